// mg_attn.cu -- attention block pieces: QK-norm + RoPE + f16 KV store, decode
// attention (split over the context, sinks, sliding ring) with its combine, and
// causal prefill attention.  Numerics follow engine/midge.c:341-400: scores
// q.k (k as stored f16) * scale, softmax whose max and denominator include the
// sink logit, output sum_t p_t * v_t.
#include "mg_attn.h"
#include "mg_common.cuh"

namespace mg {

// Per token: optional per-head RMSNorm of q and k (engine/midge.c:352-359),
// half-split RoPE (engine/midge.c:178-190), then k, v rounded to f16 with the
// subnormal flush (engine/mkern.h:261-273) into the cache slot pos % cap.
// q/k/v rows are [n_tok x dim]; tok_pos[t] = position, tok_seq[t] = sequence.
// If kv_tmp_k is non-null, k/v are (also) written to kv_tmp at row t.
__global__ void k_qkv_post(QkvPostArgs a) {
    const int t = blockIdx.x;
    const int hd = a.head_dim, half = hd >> 1;
    const int pos = a.tok_pos[t];
    const int seq = a.tok_seq ? a.tok_seq[t] : 0;
    float *q = a.q + (int64_t)t * a.ldq;
    float *k = a.k + (int64_t)t * a.ldk;
    const float *v = a.v + (int64_t)t * a.ldk;
    const int nh = a.n_heads, nkv = a.n_kv_heads;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    // qk-norm: one warp per head; sequential-order-insensitive parallel sum
    if (a.qn) {
        for (int h = warp; h < nh + nkv; h += nw) {
            float *vec = h < nh ? q + (int64_t)h * hd : k + (int64_t)(h - nh) * hd;
            const float *w = h < nh ? a.qn : a.kn;
            float ss = 0.f;
            for (int i = lane; i < hd; i += 32) ss = fmaf(vec[i], vec[i], ss);
            ss = warp_sum(ss);
            float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
            __syncwarp();
            for (int i = lane; i < hd; i += 32) vec[i] = __fmul_rn(__fmul_rn(vec[i], inv), w[i]);
        }
        __syncthreads();
    }
    const float *co = a.rope_cos + (int64_t)pos * half, *si = a.rope_sin + (int64_t)pos * half;
    for (int j = threadIdx.x; j < (nh + nkv) * half; j += blockDim.x) {
        int h = j / half, i = j - h * half;
        float *vec = h < nh ? q + (int64_t)h * hd : k + (int64_t)(h - nh) * hd;
        float x0 = vec[i], x1 = vec[i + half];
        vec[i] = __fsub_rn(__fmul_rn(x0, co[i]), __fmul_rn(x1, si[i]));
        vec[i + half] = __fadd_rn(__fmul_rn(x1, co[i]), __fmul_rn(x0, si[i]));
    }
    __syncthreads();
    const int kv_dim = nkv * hd;
    if (a.write_cache) {
        const int slot = pos % a.cap;
        uint16_t *kc = a.kc + ((int64_t)seq * a.cap + slot) * kv_dim;
        uint16_t *vc = a.vc + ((int64_t)seq * a.cap + slot) * kv_dim;
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
            kc[i] = f2h_ftz(k[i]);
            vc[i] = f2h_ftz(v[i]);
        }
    }
    if (a.tmp_k) {
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) {
            a.tmp_k[(int64_t)t * kv_dim + i] = f2h_ftz(k[i]);
            a.tmp_v[(int64_t)t * kv_dim + i] = f2h_ftz(v[i]);
        }
    }
}

int qkv_post(const QkvPostArgs &a, int n_tok, cudaStream_t st) {
    if (n_tok <= 0) return MG_OK;
    k_qkv_post<<<n_tok, 256, 0, st>>>(a);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// ------------------------------------------------------ decode attention
// Block = (kv head, sequence, split).  Scores of the split's positions for the
// gq query heads of this kv head are computed into shared memory (thread per
// position, its K row held in registers), then each thread accumulates
// (head, dim) outputs over the split.  Partials (max, sum, acc[hd]) go to
// scratch for the combine.
constexpr int ATTN_THREADS = 128;

template <int HD>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn_decode(AttnDecodeArgs a) {
    extern __shared__ __align__(16) float asm_[];
    const int kh = blockIdx.x, si = blockIdx.y, sp = blockIdx.z;
    const int seq = a.seq_ids[si];
    const int gq = a.n_heads / a.n_kv_heads, kv_dim = a.n_kv_heads * HD;
    const int pos = a.pos[si];
    const int nctx = pos + 1 < a.cap ? pos + 1 : a.cap;
    const int t0 = sp * a.split_len;
    int t1 = t0 + a.split_len;
    if (t1 > nctx) t1 = nctx;
    const int np = t1 - t0;
    float *qs = asm_;          // [gq][HD]
    float *sc = qs + gq * HD;  // [gq][split_len]
    const int64_t pstride = (int64_t)a.max_splits * (HD + 2);  // between heads
    float *part = a.partial + ((int64_t)si * a.n_heads + kh * gq) * pstride + (int64_t)sp * (HD + 2);
    if (np <= 0) {
        for (int h = threadIdx.x; h < gq; h += blockDim.x) {
            part[h * pstride + 0] = -INFINITY;
            part[h * pstride + 1] = 0.f;
        }
        return;
    }
    for (int i = threadIdx.x; i < gq * HD; i += blockDim.x)
        qs[i] = a.q[(int64_t)si * a.ldq + (int64_t)kh * gq * HD + i];
    __syncthreads();
    const uint16_t *kc = a.kc + (int64_t)seq * a.cap * kv_dim + (int64_t)kh * HD;
    const uint16_t *vc = a.vc + (int64_t)seq * a.cap * kv_dim + (int64_t)kh * HD;
    for (int p = threadIdx.x; p < np; p += blockDim.x) {
        const uint16_t *kr = kc + (int64_t)(t0 + p) * kv_dim;
        float kf[HD];
#pragma unroll
        for (int i = 0; i < HD; i += 8) {
            uint4 raw = *reinterpret_cast<const uint4 *>(kr + i);
            const __half2 *k2 = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float2 f = __half22float2(k2[j]);
                kf[i + 2 * j] = f.x;
                kf[i + 2 * j + 1] = f.y;
            }
        }
        for (int h = 0; h < gq; h++) {
            const float *qh = qs + h * HD;
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < HD; i++) d = fmaf(qh[i], kf[i], d);
            sc[h * a.split_len + p] = d * a.scale;
        }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int h = warp; h < gq; h += nw) {
        float m = -INFINITY;
        for (int p = lane; p < np; p += 32) m = fmaxf(m, sc[h * a.split_len + p]);
        m = warp_max(m);
        float s = 0.f;
        for (int p = lane; p < np; p += 32) {
            float e = expf(sc[h * a.split_len + p] - m);
            sc[h * a.split_len + p] = e;
            s += e;
        }
        s = warp_sum(s);
        if (lane == 0) {
            part[h * pstride + 0] = m;
            part[h * pstride + 1] = s;
        }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < gq * HD; j += blockDim.x) {
        int h = j / HD, i = j - h * HD;
        const float *e = sc + h * a.split_len;
        float acc = 0.f;
        for (int p = 0; p < np; p++) acc = fmaf(e[p], h2f(vc[(int64_t)(t0 + p) * kv_dim + i]), acc);
        part[h * pstride + 2 + i] = acc;
    }
}

// Combine splits and the sink:
//   out = sum_s acc_s e^(m_s-M) / (e^(sink-M) + sum_s l_s e^(m_s-M)),  M = max(sink, m_s)
__global__ void k_attn_combine(AttnDecodeArgs a) {
    const int h = blockIdx.x, si = blockIdx.y;
    const int hd = a.head_dim;
    const int pos = a.pos[si];
    const int nctx = pos + 1 < a.cap ? pos + 1 : a.cap;
    const int nsplit = (nctx + a.split_len - 1) / a.split_len;
    const float *part = a.partial + ((int64_t)si * a.n_heads + h) * (int64_t)a.max_splits * (hd + 2);
    float M = a.sinks ? a.sinks[h] : -1e30f;
    for (int s = 0; s < nsplit; s++) M = fmaxf(M, part[s * (hd + 2)]);
    float L = a.sinks ? expf(a.sinks[h] - M) : 0.f;
    for (int s = 0; s < nsplit; s++) L += part[s * (hd + 2) + 1] * expf(part[s * (hd + 2)] - M);
    float inv = 1.0f / L;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < nsplit; s++) o = fmaf(part[s * (hd + 2) + 2 + i], expf(part[s * (hd + 2)] - M), o);
        a.out[(int64_t)si * a.ldo + (int64_t)h * hd + i] = o * inv;
    }
}

template <typename K>
static int attn_smem_cfg(K kfn, size_t smem) {
    return ensure_smem(kfn, smem);
}

template <int HD>
static int attn_decode_t(const AttnDecodeArgs &a, int n_seqs, cudaStream_t st) {
    int gq = a.n_heads / a.n_kv_heads;
    size_t smem = (size_t)(gq * HD + gq * a.split_len) * 4;
    int rc = attn_smem_cfg(k_attn_decode<HD>, smem);
    if (rc) return rc;
    dim3 g1(a.n_kv_heads, n_seqs, a.max_splits);
    k_attn_decode<HD><<<g1, ATTN_THREADS, smem, st>>>(a);
    MG_CHECK_LAUNCH();
    dim3 g2(a.n_heads, n_seqs);
    k_attn_combine<<<g2, 64, 0, st>>>(a);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int attn_decode(const AttnDecodeArgs &a, int n_seqs, cudaStream_t st) {
    if (n_seqs <= 0) return MG_OK;
    switch (a.head_dim) {
    case 16: return attn_decode_t<16>(a, n_seqs, st);
    case 32: return attn_decode_t<32>(a, n_seqs, st);
    case 64: return attn_decode_t<64>(a, n_seqs, st);
    case 128: return attn_decode_t<128>(a, n_seqs, st);
    }
    set_error("attention: head_dim %d unsupported (16/32/64/128)", a.head_dim);
    return MG_ERR_ARG;
}

// ------------------------------------------------------ prefill attention
// Causal attention of n query tokens at positions pos0..pos0+n-1 of one
// sequence.  Key j is read from the chunk's own f16 K/V (tmp, rows j-pos0)
// when j >= pos0, else from the cache ring slot j % cap.  The query at
// position p sees keys max(0, p-cap+1) .. p (cap = ctx for full layers, the
// window for sliding ones: exactly the ring's valid entries when the
// reference reaches p token by token, engine/midge.c:363-370).
// Block = (tile of PF_Q query positions, q head); TPR threads per query row
// hold its q and output accumulator in registers (online softmax); K/V tiles
// are staged in shared memory as f32.
constexpr int PF_Q = 64, PF_K = 64;

template <int HD>
__global__ void __launch_bounds__(PF_Q *(HD > 64 ? 2 : 1)) k_attn_prefill(AttnPrefillArgs a) {
    constexpr int TPR = HD > 64 ? 2 : 1;
    constexpr int DPT = HD / TPR;
    extern __shared__ __align__(16) float psm[];
    const int kv_dim = a.n_kv_heads * HD;
    const int h = blockIdx.y, kh = h / (a.n_heads / a.n_kv_heads);
    const int row = threadIdx.x / TPR, part = threadIdx.x % TPR;
    const int qi = blockIdx.x * PF_Q + row;
    float *ks = psm, *vs = psm + PF_K * HD;
    const bool active = qi < a.n;
    const int p = a.pos0 + (active ? qi : 0);
    float q[DPT], acc[DPT];
#pragma unroll
    for (int i = 0; i < DPT; i++) {
        q[i] = active ? a.q[(int64_t)qi * a.ldq + (int64_t)h * HD + part * DPT + i] : 0.f;
        acc[i] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int p_first = a.pos0 + blockIdx.x * PF_Q;
    const int p_last = a.pos0 + min(a.n, (int)(blockIdx.x + 1) * PF_Q) - 1;
    const int j_lo = max(0, p_first - a.cap + 1);
    const int my_lo = max(0, p - a.cap + 1);
    for (int jb = j_lo; jb <= p_last; jb += PF_K) {
        const int nk = min(PF_K, p_last - jb + 1);
        __syncthreads();
        for (int i = threadIdx.x; i < nk * HD; i += blockDim.x) {
            int jj = i / HD, d = i - jj * HD;
            int j = jb + jj;
            const uint16_t *kr, *vr;
            if (j >= a.pos0) {
                kr = a.tmp_k + (int64_t)(j - a.pos0) * kv_dim;
                vr = a.tmp_v + (int64_t)(j - a.pos0) * kv_dim;
            } else {
                int slot = j % a.cap;
                kr = a.kc + ((int64_t)a.seq * a.cap + slot) * kv_dim;
                vr = a.vc + ((int64_t)a.seq * a.cap + slot) * kv_dim;
            }
            ks[jj * HD + d] = h2f(kr[kh * HD + d]);
            vs[jj * HD + d] = h2f(vr[kh * HD + d]);
        }
        __syncthreads();
        for (int jj = 0; jj < nk; jj++) {
            const int j = jb + jj;
            const float *kr = ks + jj * HD + part * DPT;
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < DPT; i++) d = fmaf(q[i], kr[i], d);
            if (TPR == 2) d += __shfl_xor_sync(0xffffffffu, d, 1);
            if (!active || j < my_lo || j > p) continue;
            d *= a.scale;
            const float mn = fmaxf(m, d);
            const float corr = expf(m - mn), e = expf(d - mn);
            l = l * corr + e;
            const float *vr = vs + jj * HD + part * DPT;
#pragma unroll
            for (int i = 0; i < DPT; i++) acc[i] = fmaf(e, vr[i], acc[i] * corr);
            m = mn;
        }
    }
    if (!active) return;
    const float sink = a.sinks ? a.sinks[h] : -1e30f;
    const float M = fmaxf(m, sink);
    const float corr = expf(m - M);
    const float L = l * corr + (a.sinks ? expf(sink - M) : 0.f);
    const float inv = 1.0f / L;
#pragma unroll
    for (int i = 0; i < DPT; i++) a.out[(int64_t)qi * a.ldo + (int64_t)h * HD + part * DPT + i] = acc[i] * corr * inv;
}

template <int HD>
static int attn_prefill_t(const AttnPrefillArgs &a, cudaStream_t st) {
    constexpr int TPR = HD > 64 ? 2 : 1;
    size_t smem = (size_t)2 * PF_K * HD * 4;
    int rc = attn_smem_cfg(k_attn_prefill<HD>, smem);
    if (rc) return rc;
    dim3 grid(ceil_div(a.n, PF_Q), a.n_heads);
    k_attn_prefill<HD><<<grid, PF_Q * TPR, smem, st>>>(a);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int attn_prefill(const AttnPrefillArgs &a, cudaStream_t st) {
    if (a.n <= 0) return MG_OK;
    switch (a.head_dim) {
    case 16: return attn_prefill_t<16>(a, st);
    case 32: return attn_prefill_t<32>(a, st);
    case 64: return attn_prefill_t<64>(a, st);
    case 128: return attn_prefill_t<128>(a, st);
    }
    set_error("prefill attention: head_dim %d unsupported (16/32/64/128)", a.head_dim);
    return MG_ERR_ARG;
}

}  // namespace mg

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

// The same steps with the K-split sum in front (decode): warp = (token, head)
// over the q, k and v heads.  The head's values are the planes' sum in plane
// order from 0 (as k_sum_parts), written back to q / k / v_out after the
// per-head RMSNorm and RoPE of k_qkv_post, then k and v into the cache.
constexpr int QP_WARPS = 8;
constexpr int QP_PLANES = 4;  // K-split planes summed with their loads issued together
__global__ void __launch_bounds__(QP_WARPS * 32) k_qkv_post_parts(QkvPostArgs a) {
    __shared__ float hv[QP_WARPS][128];
    const int t = blockIdx.x, w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.y * QP_WARPS + w;
    const int hd = a.head_dim, half = hd >> 1, nh = a.n_heads, nkv = a.n_kv_heads;
    if (h >= nh + 2 * nkv) {  // warp-uniform; no block barrier follows
        pdl_wait();
        return;
    }
    const int kind = h < nh ? 0 : (h < nh + nkv ? 1 : 2);  // q, k, v
    const int hh = kind == 0 ? h : (kind == 1 ? h - nh : h - nh - nkv);
    const float *src = kind == 0 ? a.q : (kind == 1 ? a.k : a.v);
    const int64_t ld = kind == 0 ? a.ldq : a.ldk;
    const int64_t off = (int64_t)t * ld + (int64_t)hh * hd;
    const float *ps = a.parts + (src - a.q) + off;  // parts rows are laid out as q / k / v
    float *vec = hv[w];
    // The position first and the RoPE values it selects (this lane's
    // dimensions lane and lane + 32 of the half); none of these comes from the
    // GEMV before this kernel, so a programmatic launch reads them before its
    // wait.  Then the plane loads, all issued together (up to QP_PLANES).
    const int pos = a.tok_pos[t];
    const int seq = a.tok_seq ? a.tok_seq[t] : 0;
    float rc[2] = {0.f, 0.f}, rsn[2] = {0.f, 0.f};
    if (kind < 2)
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const int i = lane + 32 * r;
            if (i < half) {
                rc[r] = a.rope_cos[(int64_t)pos * half + i];
                rsn[r] = a.rope_sin[(int64_t)pos * half + i];
            }
        }
    pdl_wait();
    float ss = 0.f;
    const int ks = a.ks;
#pragma unroll
    for (int r = 0; r < 4; r++) {  // dimensions lane + 32 r (head_dim <= 128)
        const int i = lane + 32 * r;
        if (i >= hd) break;
        float v = 0.f;
        if (ks <= QP_PLANES) {
            float yv[QP_PLANES];
#pragma unroll
            for (int k = 0; k < QP_PLANES; k++) yv[k] = k < ks ? ps[(int64_t)k * a.plane + i] : 0.f;
#pragma unroll
            for (int k = 0; k < QP_PLANES; k++)
                if (k < ks) v += yv[k];
        } else {
            for (int k = 0; k < ks; k++) v += ps[(int64_t)k * a.plane + i];
        }
        vec[i] = v;
        ss = fmaf(v, v, ss);
    }
    __syncwarp();
    const int kv_dim = nkv * hd;
    const int slot = pos % a.cap;
    if (kind < 2) {
        if (a.qn) {
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
            const float *nw = kind == 0 ? a.qn : a.kn;
            for (int i = lane; i < hd; i += 32) vec[i] = __fmul_rn(__fmul_rn(vec[i], inv), nw[i]);
            __syncwarp();
        }
        float *dst = (kind == 0 ? a.q : a.k) + off;
#pragma unroll
        for (int r = 0; r < 2; r++) {  // half <= 64
            const int i = lane + 32 * r;
            if (i >= half) break;
            const float x0 = vec[i], x1 = vec[i + half];
            const float y0 = __fsub_rn(__fmul_rn(x0, rc[r]), __fmul_rn(x1, rsn[r]));
            const float y1 = __fadd_rn(__fmul_rn(x1, rc[r]), __fmul_rn(x0, rsn[r]));
            dst[i] = y0;
            dst[i + half] = y1;
            if (kind == 1) {
                const int64_t c = (int64_t)hh * hd + i;
                if (a.write_cache) {
                    uint16_t *kc = a.kc + ((int64_t)seq * a.cap + slot) * kv_dim;
                    kc[c] = f2h_ftz(y0);
                    kc[c + half] = f2h_ftz(y1);
                }
                if (a.tmp_k) {
                    a.tmp_k[(int64_t)t * kv_dim + c] = f2h_ftz(y0);
                    a.tmp_k[(int64_t)t * kv_dim + c + half] = f2h_ftz(y1);
                }
            }
        }
    } else {
        for (int i = lane; i < hd; i += 32) {
            const float v = vec[i];
            const int64_t c = (int64_t)hh * hd + i;
            if (a.v_out) a.v_out[off + i] = v;
            if (a.write_cache) a.vc[((int64_t)seq * a.cap + slot) * kv_dim + c] = f2h_ftz(v);
            if (a.tmp_v) a.tmp_v[(int64_t)t * kv_dim + c] = f2h_ftz(v);
        }
    }
}

int qkv_post_parts(const QkvPostArgs &a, int n_tok, cudaStream_t st) {
    if (n_tok <= 0) return MG_OK;
    MG_REQUIRE(a.parts && a.ks >= 1 && a.head_dim <= 128 && a.ldq == a.ldk && a.k >= a.q && a.v >= a.k &&
                   (a.v - a.q) + (int64_t)a.n_kv_heads * a.head_dim <= a.ldq,
               MG_ERR_ARG, "qkv_post_parts: q, k, v must share one row of stride ldq");
    dim3 g(n_tok, (a.n_heads + 2 * a.n_kv_heads + QP_WARPS - 1) / QP_WARPS);
    MG_CUDA(launch_k(a.pdl != 0, k_qkv_post_parts, g, dim3(QP_WARPS * 32), 0, st, a));
    return MG_OK;
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
// ---- shared helpers of the tensor-core attention kernels
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {  // (lo -> low half, hi -> high half)
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}
// f16 hi/lo pair of two values: hi = f16(v), lo = f16(v - hi)
__device__ __forceinline__ void split2(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
    __half2 H = __halves2half2(ha, hb), L = __halves2half2(la, lb);
    hi = *reinterpret_cast<uint32_t *>(&H);
    lo = *reinterpret_cast<uint32_t *>(&L);
}

constexpr int ATTN_THREADS = 128;

template <int HD>
__global__ void __launch_bounds__(ATTN_THREADS) k_attn_decode(AttnDecodeArgs a) {
    extern __shared__ __align__(16) float asm_[];
    pdl_trigger();  // the combine may start and wait for this grid
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

// Decode attention on the tensor cores (head_dim 64, up to 8 query heads per
// KV head).  Block = one warp = (kv head, sequence, split of split_len
// positions, a multiple of 64), walking the split in tiles of 64 positions
// with an online softmax: the next tile's K and V (64 positions x 64 dims of
// f16, as cached) come in by cp.async into 128-byte-swizzled shared memory
// while the current one is multiplied.  The A operand of every MMA stacks
// the f16 hi halves of the group's query rows (rows 0..7) over their lo
// halves (rows 8..15), so D rows g and g + 8 are the two halves of the same
// (head, position) and sum exactly in fp32:
//   S = [q_hi; q_lo] K^T, softmax pieces in fp32 against the running maximum
//   M (earlier tiles' sums and outputs rescaled by e^(M_old - M)),
//   O += [P_hi; P_lo] V.
// Writes per-split partials (max, sum, acc) for the combine.
constexpr int TCD_POS = 64;

// MULTI = false: one tile per split (split_len 64), compiled without the
// loop-carried rescaling so that it keeps the register count of a single tile.
template <bool MULTI>
__global__ void __launch_bounds__(32) k_attn_decode_tc(AttnDecodeArgs a) {
    constexpr int HD = 64;
    pdl_trigger();  // the combine may start and wait for this grid
    // [buffer][K, V] tiles: two buffers when a split has more than one tile
    extern __shared__ __align__(128) uint16_t kv[];
    const int kh = blockIdx.x, si = blockIdx.y, sp = blockIdx.z;
    const int seq = a.seq_ids[si];
    const int gq = a.n_heads / a.n_kv_heads, kv_dim = a.n_kv_heads * HD;
    const int pos = a.pos[si];
    const int nctx = pos + 1 < a.cap ? pos + 1 : a.cap;
    const int t0 = sp * a.split_len;
    const int npa = min(a.split_len, nctx - t0);  // positions of this split
    const int lane = threadIdx.x, g = lane >> 2, t = lane & 3;
    const int64_t pstride = (int64_t)a.max_splits * (HD + 2);
    float *part = a.partial + ((int64_t)si * a.n_heads + kh * gq) * pstride + (int64_t)sp * (HD + 2);
    if (npa <= 0) {
        if (lane < gq) {
            part[lane * pstride + 0] = -INFINITY;
            part[lane * pstride + 1] = 0.f;
        }
        return;
    }
    const int ntile = MULTI ? (npa + TCD_POS - 1) / TCD_POS : 1;
    const uint32_t sb = (uint32_t)__cvta_generic_to_shared(kv);
    auto swz = [](int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); };
    const uint16_t *kc = a.kc + (int64_t)seq * a.cap * kv_dim + (int64_t)kh * HD;
    const uint16_t *vc = a.vc + (int64_t)seq * a.cap * kv_dim + (int64_t)kh * HD;
    constexpr uint32_t MAT = TCD_POS * HD * 2;  // bytes of one 64 x 64 f16 tile
    // positions [t0 + 64 i, + np) of the ring into buffer b, rows beyond np zero-filled
    auto load_tile = [&](int i, int b) {
        const int p0 = t0 + i * TCD_POS, np = min(TCD_POS, npa - i * TCD_POS);
        const uint32_t kb = sb + (uint32_t)b * 2 * MAT, vb = kb + MAT;
#pragma unroll
        for (int j = 0; j < 16; j++) {  // 512 chunks of 16 bytes per matrix, 16 per lane
            const int c = lane + 32 * j, r = c >> 3, part8 = c & 7;
            const uint32_t dk = kb + swz(r, part8), dv = vb + swz(r, part8);
            if (r < np) {
                cp_async16(dk, kc + (int64_t)(p0 + r) * kv_dim + part8 * 8);
                cp_async16(dv, vc + (int64_t)(p0 + r) * kv_dim + part8 * 8);
            } else {
                asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dk), "r"(0) : "memory");
                asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dv), "r"(0) : "memory");
            }
        }
        cp_async_commit();
    };
    // MULTI: three buffers, two tiles in flight ahead of the one multiplied
    constexpr int NBUF = MULTI ? 3 : 1;
    load_tile(0, 0);
    if (MULTI && ntile > 1) load_tile(1, 1);
    // A fragments of [q_hi; q_lo] for the 4 k-steps (row g = head g)
    uint32_t qa[4][4];
    {
        const bool hv = g < gq;
        const float *qp = a.q + (int64_t)si * a.ldq + (int64_t)(kh * gq + (hv ? g : 0)) * HD;
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            const int d0 = ks * 16 + 2 * t, d1 = d0 + 8;
            const float x0 = hv ? qp[d0] : 0.f, x1 = hv ? qp[d0 + 1] : 0.f;
            const float x2 = hv ? qp[d1] : 0.f, x3 = hv ? qp[d1 + 1] : 0.f;
            split2(x0, x1, qa[ks][0], qa[ks][1]);  // a0: row g (hi), a1: row g + 8 (lo)
            split2(x2, x3, qa[ks][2], qa[ks][3]);
        }
    }
    float M = -INFINITY, lsum = 0.f;
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) o[i][j] = 0.f;
#pragma unroll 1
    for (int it = 0; it < ntile; it++) {
        // tile it must be complete; the groups committed after it may pend
        if (MULTI && it + 2 < ntile) {
            load_tile(it + 2, (it + 2) % NBUF);  // into the buffer tile it - 1 left
            cp_async_wait<2>();
        } else if (MULTI && it + 1 < ntile) {
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncwarp();
        const int np = min(TCD_POS, npa - it * TCD_POS);
        const uint32_t kb = sb + (uint32_t)(it % NBUF) * 2 * MAT, vb = kb + MAT;
        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll
        for (int np2 = 0; np2 < 4; np2++) {
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {
                const int mi = lane >> 3, rr = lane & 7;
                const int r = np2 * 16 + (mi >> 1) * 8 + rr, chunk = ks * 2 + (mi & 1);
                uint32_t b00, b01, b10, b11;
                ldsm_x4(kb + swz(r, chunk), b00, b01, b10, b11);
                mma_16816(sc[2 * np2], qa[ks], b00, b01);
                mma_16816(sc[2 * np2 + 1], qa[ks], b10, b11);
            }
        }
        // head g's scores at positions 8 nt + 2t (+1): hi part in c0/c1, lo part in c2/c3
        float sv[8][2];
        float mx = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int p = nt * 8 + 2 * t + e;
                const float v = p < np ? __fadd_rn(sc[nt][e], sc[nt][2 + e]) * a.scale : -INFINITY;
                sv[nt][e] = v;
                mx = fmaxf(mx, v);
            }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float Mn = MULTI ? fmaxf(M, mx) : mx;
        const float alpha = (!MULTI || M == -INFINITY) ? 0.f : expf(M - Mn);  // rescales the earlier tiles
        float sum = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float pv = sv[nt][e] == -INFINITY ? 0.f : expf(sv[nt][e] - Mn);
                sv[nt][e] = pv;
                sum += pv;
            }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        lsum = MULTI ? lsum * alpha + sum : sum;
        M = Mn;
        if (MULTI)
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) o[i][j] *= alpha;
        // O += [P_hi; P_lo] V
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {  // positions 16 kk .. 16 kk + 15
            uint32_t pa[4];
            split2(sv[2 * kk][0], sv[2 * kk][1], pa[0], pa[1]);
            split2(sv[2 * kk + 1][0], sv[2 * kk + 1][1], pa[2], pa[3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {
                const int mi = lane >> 3, rr = lane & 7;
                const int r = kk * 16 + (mi & 1) * 8 + rr, chunk = dp * 2 + (mi >> 1);
                uint32_t b00, b01, b10, b11;
                ldsm_x4_t(vb + swz(r, chunk), b00, b01, b10, b11);
                mma_16816(o[2 * dp], pa, b00, b01);
                mma_16816(o[2 * dp + 1], pa, b10, b11);
            }
        }
        __syncwarp();  // every lane is done with this buffer before the next load refills it
    }
    if (g < gq) {
        float *ph = part + (int64_t)g * pstride;
        if (t == 0) {
            ph[0] = M;
            ph[1] = lsum;
        }
#pragma unroll
        for (int dt = 0; dt < 8; dt++) {
            const int d = dt * 8 + 2 * t;
            ph[2 + d] = __fadd_rn(o[dt][0], o[dt][2]);
            ph[2 + d + 1] = __fadd_rn(o[dt][1], o[dt][3]);
        }
    }
}

// Combine splits and the sink:
//   out = sum_s acc_s e^(m_s-M) / (e^(sink-M) + sum_s l_s e^(m_s-M)),  M = max(sink, m_s)
// One block (8 warps) per (head, sequence): the split maxima and the
// denominator are reduced once and each split's weight e^(m_s-M) is kept in
// shared memory (max_splits floats); warp w sums the splits w, w + 8, ... in
// ascending order for every output dimension (lane + 32 r), and the eight
// warp sums are added in warp order.
constexpr int AC_WARPS = 8;
__global__ void __launch_bounds__(AC_WARPS * 32) k_attn_combine(AttnDecodeArgs a, int staged) {
    extern __shared__ float cw[];  // [max_splits] split weights, then (staged) the partials
    __shared__ float red[2][AC_WARPS];
    __shared__ float ws[AC_WARPS][128];
    const int h = blockIdx.x, si = blockIdx.y, t = threadIdx.x, w = t >> 5, lane = t & 31;
    const int hd = a.head_dim, rs = hd + 2;
    const float *gpart = a.partial + ((int64_t)si * a.n_heads + h) * (int64_t)a.max_splits * rs;
    // the position and the sink (neither written by the attention grid, so a
    // programmatic launch reads them before its wait); then (staged) every
    // split slot's partial at once, without waiting for the position (the
    // slots past the context are staged too, and skipped below)
    const int pos = a.pos[si];
    const float sink = a.sinks ? a.sinks[h] : -1e30f;
    pdl_wait();
    const float *part = gpart;
    if (staged) {
        float *sp = cw + ((a.max_splits + 1) & ~1);  // 8-byte aligned
        const int n2 = a.max_splits * rs / 2;         // float pairs (head_dim even)
        const float2 *g2 = reinterpret_cast<const float2 *>(gpart);
        float2 *s2 = reinterpret_cast<float2 *>(sp);
        constexpr int U = 10;
        for (int b = t; b < n2; b += U * blockDim.x) {
            float2 r[U];
#pragma unroll
            for (int u = 0; u < U; u++)
                if (b + u * (int)blockDim.x < n2) r[u] = g2[b + u * blockDim.x];
#pragma unroll
            for (int u = 0; u < U; u++)
                if (b + u * (int)blockDim.x < n2) s2[b + u * blockDim.x] = r[u];
        }
        __syncthreads();
        part = sp;
    }
    const int nctx = pos + 1 < a.cap ? pos + 1 : a.cap;
    const int nsplit = (nctx + a.split_len - 1) / a.split_len;
    float mx = sink;
    for (int s = t; s < nsplit; s += blockDim.x) mx = fmaxf(mx, part[s * rs]);
    mx = warp_max(mx);
    if (lane == 0) red[0][w] = mx;
    __syncthreads();
    float M = red[0][0];
#pragma unroll
    for (int i = 1; i < AC_WARPS; i++) M = fmaxf(M, red[0][i]);
    float ls = 0.f;
    for (int s = t; s < nsplit; s += blockDim.x) {
        const float e = expf(part[s * rs] - M);
        cw[s] = e;
        ls += part[s * rs + 1] * e;
    }
    ls = warp_sum(ls);
    if (lane == 0) red[1][w] = ls;
    __syncthreads();
    float lsum = red[1][0];
#pragma unroll
    for (int i = 1; i < AC_WARPS; i++) lsum += red[1][i];
    const float L = (a.sinks ? expf(sink - M) : 0.f) + lsum;
    float o[4] = {0.f, 0.f, 0.f, 0.f};  // dimensions lane + 32 r (head_dim <= 128)
    for (int s = w; s < nsplit; s += AC_WARPS) {
        const float c = cw[s];
        const float *ps = part + s * rs + 2;
#pragma unroll
        for (int r = 0; r < 4; r++)
            if (lane + 32 * r < hd) o[r] = fmaf(ps[lane + 32 * r], c, o[r]);
    }
#pragma unroll
    for (int r = 0; r < 4; r++)
        if (lane + 32 * r < hd) ws[w][lane + 32 * r] = o[r];
    __syncthreads();
    const float inv = 1.0f / L;
    for (int i = t; i < hd; i += blockDim.x) {
        float v = ws[0][i];
#pragma unroll
        for (int k = 1; k < AC_WARPS; k++) v += ws[k][i];
        a.out[(int64_t)si * a.ldo + (int64_t)h * hd + i] = v * inv;
    }
}

// the partials staged in shared memory when they fit in AC_STAGE_BYTES
constexpr size_t AC_STAGE_BYTES = 64 * 1024;
static int attn_combine(const AttnDecodeArgs &a, int n_seqs, cudaStream_t st) {
    dim3 g2(a.n_heads, n_seqs);
    const size_t cw = (size_t)((a.max_splits + 1) & ~1) * 4;
    const size_t staged = cw + (size_t)a.max_splits * (a.head_dim + 2) * 4;
    const bool stage = a.head_dim % 2 == 0 && staged <= AC_STAGE_BYTES;
    const size_t cs = stage ? staged : cw;
    if (cs > 48 * 1024 && ensure_smem(k_attn_combine, cs)) return MG_ERR_CUDA;
    MG_CUDA(launch_k(a.pdl != 0, k_attn_combine, g2, dim3(AC_WARPS * 32), cs, st, a, stage ? 1 : 0));
    return MG_OK;
}

template <typename K>
static int attn_smem_cfg(K kfn, size_t smem) {
    return ensure_smem(kfn, smem);
}

template <int HD>
static int attn_decode_t(const AttnDecodeArgs &a, int n_seqs, cudaStream_t st) {
    int gq = a.n_heads / a.n_kv_heads;
    if (HD == 64 && a.use_tc && gq <= 8 && a.split_len % TCD_POS == 0) {
        dim3 g1(a.n_kv_heads, n_seqs, a.max_splits);
        const bool multi = a.split_len > TCD_POS;
        const size_t ts = (size_t)(multi ? 3 : 1) * 2 * TCD_POS * 64 * 2;  // K and V tiles per buffer
        if (multi) k_attn_decode_tc<true><<<g1, 32, ts, st>>>(a);
        else k_attn_decode_tc<false><<<g1, 32, ts, st>>>(a);
        MG_CHECK_LAUNCH();
        return attn_combine(a, n_seqs, st);
    }
    size_t smem = (size_t)(gq * HD + gq * a.split_len) * 4;
    int rc = attn_smem_cfg(k_attn_decode<HD>, smem);
    if (rc) return rc;
    dim3 g1(a.n_kv_heads, n_seqs, a.max_splits);
    k_attn_decode<HD><<<g1, ATTN_THREADS, smem, st>>>(a);
    MG_CHECK_LAUNCH();
    return attn_combine(a, n_seqs, st);
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

// ---------------------------------------------- prefill attention, tensor cores
// Flash-attention form on mma.sync (head_dim 64): block = 64 queries of one
// head, 4 warps x 16 query rows; 64-key tiles of K and V (f16, exactly as
// cached) double-buffered in 128-byte-swizzled shared memory by cp.async.
//   S = Q K^T with Q split into f16 hi + lo (products exact, fp32 sums), the
//   scale, the causal / sliding-window mask, online softmax in fp32 (row max
//   and sum over the quad of lanes holding a row), then O += P V with P split
//   into hi + lo the same way.  The sink joins the normaliser at the end, as
//   engine/midge.c:376-398 does.  Agrees with the fp32 scalar kernel to ~1e-6.
constexpr int TCA_Q = 64, TCA_K = 64, TCA_THREADS = 128;

__global__ void __launch_bounds__(TCA_THREADS) k_attn_prefill_tc(AttnPrefillArgs a) {
    constexpr int HD = 64;
    __shared__ __align__(128) uint16_t kv_s[2][2][TCA_K * HD];  // [buffer][K, V][key][dim], swizzled
    const int kv_dim = a.n_kv_heads * HD;
    const int h = blockIdx.y, kh = h / (a.n_heads / a.n_kv_heads);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int q0 = blockIdx.x * TCA_Q;  // first query (chunk index) of the block
    const int qr0 = q0 + warp * 16 + g, qr1 = qr0 + 8;
    const bool act0 = qr0 < a.n, act1 = qr1 < a.n;
    const int p0 = a.pos0 + qr0, p1 = a.pos0 + qr1;
    // Q fragments (rows qr0, qr1; 4 k-steps of 16 dims), hi and lo
    uint32_t qh[4][4], ql[4][4];
#pragma unroll
    for (int ks = 0; ks < 4; ks++) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = (i & 1) ? qr1 : qr0;
            const bool ok = (i & 1) ? act1 : act0;
            const int d = ks * 16 + 2 * t + (i >> 1) * 8;
            const float *qp = a.q + (int64_t)(ok ? r : 0) * a.ldq + (int64_t)h * HD + d;
            v[2 * i] = ok ? qp[0] : 0.f;
            v[2 * i + 1] = ok ? qp[1] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) split2(v[2 * i], v[2 * i + 1], qh[ks][i], ql[ks][i]);
    }
    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) o[i][j] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    const int p_first = a.pos0 + q0;
    const int p_last = a.pos0 + min(a.n, q0 + TCA_Q) - 1;
    const int j_lo = max(0, p_first - a.cap + 1);
    const int ntile = (p_last - j_lo) / TCA_K + 1;
    const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(&kv_s[0][0][0]);
    auto swz = [](int key, int chunk) { return (uint32_t)(key * 128 + ((chunk ^ (key & 7)) << 4)); };
    auto load_tile = [&](int tile, int buf) {
        const int jb = j_lo + tile * TCA_K;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int c = threadIdx.x + TCA_THREADS * i;  // 512 chunks of 16 bytes per matrix
            const int key = c >> 3, part = c & 7;
            const int j = jb + key;
            const uint32_t dk = sbase + (uint32_t)((buf * 2 + 0) * TCA_K * HD * 2) + swz(key, part);
            const uint32_t dv = sbase + (uint32_t)((buf * 2 + 1) * TCA_K * HD * 2) + swz(key, part);
            if (j <= p_last) {
                const uint16_t *kr, *vr;
                if (j >= a.pos0) {
                    kr = a.tmp_k + (int64_t)(j - a.pos0) * kv_dim;
                    vr = a.tmp_v + (int64_t)(j - a.pos0) * kv_dim;
                } else {
                    const int slot = j % a.cap;
                    kr = a.kc + ((int64_t)a.seq * a.cap + slot) * kv_dim;
                    vr = a.vc + ((int64_t)a.seq * a.cap + slot) * kv_dim;
                }
                cp_async16(dk, kr + kh * HD + part * 8);
                cp_async16(dv, vr + kh * HD + part * 8);
            } else {  // beyond the block's last key: zeros (their P is 0, V must be finite)
                asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dk), "r"(0) : "memory");
                asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dv), "r"(0) : "memory");
            }
        }
        cp_async_commit();
    };
    load_tile(0, 0);
    for (int tile = 0; tile < ntile; tile++) {
        const int buf = tile & 1;
        if (tile + 1 < ntile) {
            load_tile(tile + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int jb = j_lo + tile * TCA_K;
        const uint32_t kb = sbase + (uint32_t)((buf * 2 + 0) * TCA_K * HD * 2);
        const uint32_t vb = sbase + (uint32_t)((buf * 2 + 1) * TCA_K * HD * 2);
        // S = Q K^T: 8 n-tiles of 8 keys
        float sc[8][4];
#pragma unroll
        for (int i = 0; i < 8; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) sc[i][j] = 0.f;
#pragma unroll
        for (int np = 0; np < 4; np++) {      // keys 16 np .. 16 np + 15
#pragma unroll
            for (int ks = 0; ks < 4; ks++) {  // dims 16 ks .. 16 ks + 15
                // matrices: (keys +0..7, dims +0..7), (keys +0..7, dims +8..15), (keys +8..15, dims +0..7), (+8..15, +8..15)
                const int mi = lane >> 3, rr = lane & 7;
                const int key = np * 16 + (mi >> 1) * 8 + rr, chunk = ks * 2 + (mi & 1);
                uint32_t b00, b01, b10, b11;
                ldsm_x4(kb + swz(key, chunk), b00, b01, b10, b11);
                mma_16816(sc[2 * np], qh[ks], b00, b01);
                mma_16816(sc[2 * np], ql[ks], b00, b01);
                mma_16816(sc[2 * np + 1], qh[ks], b10, b11);
                mma_16816(sc[2 * np + 1], ql[ks], b10, b11);
            }
        }
        // scale, mask, online softmax (row g: elements 0,1; row g + 8: elements 2,3)
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int j = jb + nt * 8 + 2 * t + (e & 1);
                const int p = (e < 2) ? p0 : p1;
                const bool ok = ((e < 2) ? act0 : act1) && j <= p && j > p - a.cap;
                const float v = ok ? sc[nt][e] * a.scale : -INFINITY;
                sc[nt][e] = v;
                if (e < 2) mx0 = fmaxf(mx0, v);
                else mx1 = fmaxf(mx1, v);
            }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float c0 = mn0 == -INFINITY ? 1.f : expf(m0 - mn0), c1 = mn1 == -INFINITY ? 1.f : expf(m1 - mn1);
        float s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float mref = e < 2 ? mn0 : mn1;
                const float pv = sc[nt][e] == -INFINITY ? 0.f : expf(sc[nt][e] - mref);
                sc[nt][e] = pv;
                if (e < 2) s0 += pv;
                else s1 += pv;
            }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s0 += __shfl_xor_sync(0xffffffffu, s0, 2);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 2);
        l0 = l0 * c0 + s0;
        l1 = l1 * c1 + s1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int dt = 0; dt < 8; dt++) {
            o[dt][0] *= c0;
            o[dt][1] *= c0;
            o[dt][2] *= c1;
            o[dt][3] *= c1;
        }
        // O += P V: k-steps of 16 keys, 8 n-tiles of 8 dims
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
            uint32_t ph[4], pl[4];
            split2(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
            split2(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
            split2(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
            split2(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
            for (int dp = 0; dp < 4; dp++) {  // dims 16 dp .. 16 dp + 15
                // transposed matrices: (keys +0..7, dims +0..7), (keys +8..15, dims +0..7), (keys +0..7, dims +8..15), (+8.., +8..)
                const int mi = lane >> 3, rr = lane & 7;
                const int key = kk * 16 + (mi & 1) * 8 + rr, chunk = dp * 2 + (mi >> 1);
                uint32_t b00, b01, b10, b11;
                ldsm_x4_t(vb + swz(key, chunk), b00, b01, b10, b11);
                mma_16816(o[2 * dp], ph, b00, b01);
                mma_16816(o[2 * dp], pl, b00, b01);
                mma_16816(o[2 * dp + 1], ph, b10, b11);
                mma_16816(o[2 * dp + 1], pl, b10, b11);
            }
        }
        __syncthreads();  // the buffer is refilled by the next iteration's prefetch
    }
    const float sink = a.sinks ? a.sinks[h] : -INFINITY;
#pragma unroll
    for (int half = 0; half < 2; half++) {
        const bool ok = half ? act1 : act0;
        if (!ok) continue;
        const float m = half ? m1 : m0, l = half ? l1 : l0;
        const float M = fmaxf(m, sink);
        const float corr = expf(m - M);
        const float L = l * corr + (a.sinks ? expf(sink - M) : 0.f);
        const float inv = 1.0f / L;
        const int r = half ? qr1 : qr0;
        float *op = a.out + (int64_t)r * a.ldo + (int64_t)h * HD;
#pragma unroll
        for (int dt = 0; dt < 8; dt++) {
            const int d = dt * 8 + 2 * t;
            op[d] = o[dt][2 * half] * corr * inv;
            op[d + 1] = o[dt][2 * half + 1] * corr * inv;
        }
    }
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
    case 64:
        if (a.use_tc) {
            dim3 grid(ceil_div(a.n, TCA_Q), a.n_heads);
            k_attn_prefill_tc<<<grid, TCA_THREADS, 0, st>>>(a);
            MG_CHECK_LAUNCH();
            return MG_OK;
        }
        return attn_prefill_t<64>(a, st);
    case 128: return attn_prefill_t<128>(a, st);
    }
    set_error("prefill attention: head_dim %d unsupported (16/32/64/128)", a.head_dim);
    return MG_ERR_ARG;
}

}  // namespace mg

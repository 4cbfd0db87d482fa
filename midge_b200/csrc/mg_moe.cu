// mg_moe.cu -- router (rmsnorm + f32 logits in the reference's AVX2 lane order +
// top-k + routing weights + usage counts) and the decode routed-expert FFN.
#include "mg_gemv.cuh"
#include "mg_kernels.h"

namespace mg {

constexpr int ROUTER_THREADS = 1024;
constexpr int MAX_TOPK = 16;      // engine/midge.c:44
constexpr int MAX_SLOTS = 256;    // n_tok * top_k handled by one decode MoE call

// ------------------------------------------------------------- router
// One block per token.  Logit e is computed by 8 consecutive threads exactly
// as mv_f32_avx2 (engine/mkern.h:85-99): lane l accumulates fma(w[c+l], x[c+l])
// over c = 0, 8, 16, ...; the 8 lanes are combined in hsum256's tree order
// ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)) (engine/mkern.h:76-82); the scalar
// tail adds w*x with separate rounding; then the bias (engine/mkern.h:245).
__global__ void __launch_bounds__(ROUTER_THREADS) k_router(RouterArgs a) {
    extern __shared__ __align__(16) float rsm[];
    const int64_t H = a.hidden;
    float *xs = rsm;                  // [H]
    float *rl = rsm + H;              // [E]
    __shared__ float scratch[32];
    __shared__ int taken[2048 / 32];
    __shared__ int s_sel[MAX_TOPK];
    __shared__ float s_val[MAX_TOPK];
    const int tok = blockIdx.x;
    const float *xr = a.x + (int64_t)tok * H;
    if (a.x_parts) {  // attention output partials join the residual first
        float *xw = const_cast<float *>(xr);
        for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
            float v = 0.f;
            for (int k = 0; k < a.x_parts_ks; k++) v += a.x_parts[(int64_t)k * a.x_parts_stride + (int64_t)tok * H + i];
            xw[i] = __fadd_rn(xw[i], v);
        }
        __syncthreads();
    }

    if (a.norm_w) {
        float ss = 0.f;
        for (int64_t i = threadIdx.x; i < H; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
        ss = block_sum(ss, scratch);
        float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
        for (int64_t i = threadIdx.x; i < H; i += blockDim.x) {
            float v = __fmul_rn(__fmul_rn(xr[i], inv), a.norm_w[i]);
            xs[i] = v;
            if (a.xb_out) a.xb_out[(int64_t)tok * H + i] = v;
        }
    } else {
        for (int64_t i = threadIdx.x; i < H; i += blockDim.x) xs[i] = xr[i];
    }
    for (int i = threadIdx.x; i < (a.n_experts + 31) / 32; i += blockDim.x) taken[i] = 0;
    __syncthreads();

    const int64_t H8 = H & ~(int64_t)7;
    const int lane8 = threadIdx.x & 7;
    for (int e0 = 0; e0 < a.n_experts; e0 += blockDim.x / 8) {
        int e = e0 + (int)(threadIdx.x >> 3);
        bool ok = e < a.n_experts;
        const float *wr = a.rw + (int64_t)(ok ? e : 0) * H;
        float acc = 0.f;
        if (ok)
            for (int64_t c = 0; c < H8; c += 8) acc = fmaf(wr[c + lane8], xs[c + lane8], acc);
        float s1 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
        float s2 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
        float s3 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
        if (ok && lane8 == 0) {
            float r = s3;
            for (int64_t c = H8; c < H; c++) r = __fadd_rn(r, __fmul_rn(wr[c], xs[c]));
            r = __fadd_rn(r, a.rb[e]);
            rl[e] = r;
            if (a.logits) a.logits[(int64_t)tok * a.n_experts + e] = r;
        }
    }
    __syncthreads();

    // top-k by (value desc, index asc) among logits > -1e30 (NaN never wins),
    // the selection both reference insertion sorts produce
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        for (int j = 0; j < a.top_k; j++) {
            float bv = -1e30f;
            int bi = 0x7fffffff;
            for (int e = lane; e < a.n_experts; e += 32) {
                if (taken[e >> 5] & (1 << (e & 31))) continue;
                float v = rl[e];
                if (v > bv) { bv = v; bi = e; }  // ascending e per lane: first max kept
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
            }
            if (lane == 0) {
                if (bi != 0x7fffffff && bv > -1e30f) {
                    s_sel[j] = bi;
                    s_val[j] = bv;
                    taken[bi >> 5] |= 1 << (bi & 31);
                } else {
                    s_sel[j] = a.variant == 0 ? -1 : 0;
                    s_val[j] = -1e30f;
                }
            }
            __syncwarp();
        }
        // routing weights (engine/midge.c:423-433, :502-512)
        float fmx = 0.f, fden = 0.f;
        if (!a.router_norm) {
            float m = -INFINITY;
            for (int e = lane; e < a.n_experts; e += 32) m = fmaxf(m, rl[e]);
            fmx = warp_max(m);
            float d = 0.f;
            for (int e = lane; e < a.n_experts; e += 32) d += expf(rl[e] - fmx);
            fden = warp_sum(d);
        }
        if (lane == 0) {
            float w[MAX_TOPK];
            const int k = a.top_k;
            if (a.router_norm) {
                float mx = s_val[0], den = 0.f;
                for (int i = 0; i < k; i++) { w[i] = expf(s_val[i] - mx); den = __fadd_rn(den, w[i]); }
                for (int i = 0; i < k; i++) w[i] = __fdiv_rn(w[i], den);
            } else {
                for (int i = 0; i < k; i++) w[i] = __fdiv_rn(expf(s_val[i] - fmx), fden);
            }
            for (int i = 0; i < k; i++) {
                a.sel[(int64_t)tok * k + i] = s_sel[i];
                a.weights[(int64_t)tok * k + i] = w[i];
                if (a.usage && s_sel[i] >= 0 && s_val[i] > -1e30f) atomicAdd(&a.usage[s_sel[i]], 1u);
            }
        }
    }
}

// Decode router in two launches.
//   k_router_prep (block per token): residual = x + the attention-output
//   K-split partials (summed in plane order), written to x_out; its RMS norm
//   -> xb_out.
//   k_router_logits (block per 4 experts, all tokens): the 4 weight rows and
//   the tokens' normed rows are bulk-copied into shared memory (row stride
//   padded so the 8-lane groups of a warp hit distinct banks) and every logit
//   is reduced in the AVX2 lane order (engine/mkern.h:85-99); the last block
//   to finish (atomic ticket) runs the top-k, routing weights and usage for
//   all tokens.
constexpr int RG = 4;  // experts per logits block (32 blocks stream the 128 rows of the 120b router)

constexpr int RP_PLANES = 8;  // K-split planes whose loads k_router_prep issues together
__global__ void __launch_bounds__(1024) k_router_prep(RouterArgs a) {
    __shared__ float scratch[32];
    pdl_trigger();  // the logits blocks may start staging their weight rows
    const int64_t H = a.hidden;
    const int tok = blockIdx.x;
    const float *xr = a.x + (int64_t)tok * H;
    constexpr int PER = 4;  // elements per thread per pass (loads issued together)
    float v[PER];
    float ss = 0.f;
    if (H <= (int64_t)blockDim.x * PER) {  // one pass: the row stays in registers through the norm
        // every load issued together (residual, norm weight, partial planes):
        // one round trip to memory before the block reduction
        float nw[PER];
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            v[j] = c < H ? xr[c] : 0.f;
            nw[j] = c < H ? a.norm_w[c] : 0.f;
        }
        if (a.x_parts) {
            float p[PER] = {0.f, 0.f, 0.f, 0.f};
            const int ks = a.x_parts_ks;
            if (ks <= RP_PLANES) {  // planes added in plane order, as below
                float yv[RP_PLANES][PER];
#pragma unroll
                for (int k = 0; k < RP_PLANES; k++) {
                    const float *pp = a.x_parts + (int64_t)k * a.x_parts_stride + (int64_t)tok * H;
#pragma unroll
                    for (int j = 0; j < PER; j++) {
                        const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
                        yv[k][j] = (k < ks && c < H) ? pp[c] : 0.f;
                    }
                }
#pragma unroll
                for (int k = 0; k < RP_PLANES; k++)
#pragma unroll
                    for (int j = 0; j < PER; j++)
                        if (k < ks) p[j] += yv[k][j];
            } else {
                for (int k = 0; k < ks; k++) {
                    const float *pp = a.x_parts + (int64_t)k * a.x_parts_stride + (int64_t)tok * H;
#pragma unroll
                    for (int j = 0; j < PER; j++) {
                        const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
                        if (c < H) p[j] += pp[c];
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
                v[j] = __fadd_rn(v[j], p[j]);
                if (c < H) a.x_out[(int64_t)tok * H + c] = v[j];
            }
        }
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            if (c < H) ss = fmaf(v[j], v[j], ss);
        }
        ss = block_sum(ss, scratch);
        const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            if (c < H) a.xb_out[(int64_t)tok * H + c] = __fmul_rn(__fmul_rn(v[j], inv), nw[j]);
        }
        return;
    }
    for (int64_t c0 = threadIdx.x; c0 < H; c0 += (int64_t)blockDim.x * PER) {
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = c0 + (int64_t)j * blockDim.x;
            v[j] = c < H ? xr[c] : 0.f;
        }
        if (a.x_parts) {
            float p[PER] = {0.f, 0.f, 0.f, 0.f};
            for (int k = 0; k < a.x_parts_ks; k++) {
                const float *pp = a.x_parts + (int64_t)k * a.x_parts_stride + (int64_t)tok * H;
#pragma unroll
                for (int j = 0; j < PER; j++) {
                    const int64_t c = c0 + (int64_t)j * blockDim.x;
                    if (c < H) p[j] += pp[c];
                }
            }
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int64_t c = c0 + (int64_t)j * blockDim.x;
                v[j] = __fadd_rn(v[j], p[j]);
                if (c < H) a.x_out[(int64_t)tok * H + c] = v[j];
            }
        }
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = c0 + (int64_t)j * blockDim.x;
            if (c < H) {
                ss = fmaf(v[j], v[j], ss);
                a.xb_out[(int64_t)tok * H + c] = v[j];  // raw for now, scaled below
            }
        }
    }
    ss = block_sum(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
    __syncthreads();
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
        const int64_t o = (int64_t)tok * H + c;
        a.xb_out[o] = __fmul_rn(__fmul_rn(a.xb_out[o], inv), a.norm_w[c]);
    }
}

// top-k by (value desc, index asc) among logits > -1e30, routing weights and
// usage for token `tok`; one warp
__device__ void router_topk_warp(const RouterArgs &a, const float *rl, int tok, int *taken, int *s_sel,
                                 float *s_val) {
    const int lane = threadIdx.x & 31;
    for (int i = lane; i < (a.n_experts + 31) / 32; i += 32) taken[i] = 0;
    __syncwarp();
    for (int j = 0; j < a.top_k; j++) {
        float bv = -1e30f;
        int bi = 0x7fffffff;
        for (int e = lane; e < a.n_experts; e += 32) {
            if (taken[e >> 5] & (1 << (e & 31))) continue;
            const float v = rl[e];
            if (v > bv) { bv = v; bi = e; }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            if (bi != 0x7fffffff && bv > -1e30f) {
                s_sel[j] = bi;
                s_val[j] = bv;
                taken[bi >> 5] |= 1 << (bi & 31);
            } else {
                s_sel[j] = a.variant == 0 ? -1 : 0;
                s_val[j] = -1e30f;
            }
        }
        __syncwarp();
    }
    float fmx = 0.f, fden = 0.f;
    if (!a.router_norm) {
        float mx = -INFINITY;
        for (int e = lane; e < a.n_experts; e += 32) mx = fmaxf(mx, rl[e]);
        fmx = warp_max(mx);
        float d = 0.f;
        for (int e = lane; e < a.n_experts; e += 32) d += expf(rl[e] - fmx);
        fden = warp_sum(d);
    }
    if (lane == 0) {
        float w[MAX_TOPK];
        const int k = a.top_k;
        if (a.router_norm) {
            const float mx = s_val[0];
            float den = 0.f;
            for (int i = 0; i < k; i++) { w[i] = expf(s_val[i] - mx); den = __fadd_rn(den, w[i]); }
            for (int i = 0; i < k; i++) w[i] = __fdiv_rn(w[i], den);
        } else {
            for (int i = 0; i < k; i++) w[i] = __fdiv_rn(expf(s_val[i] - fmx), fden);
        }
        for (int i = 0; i < k; i++) {
            a.sel[(int64_t)tok * k + i] = s_sel[i];
            a.weights[(int64_t)tok * k + i] = w[i];
            if (a.usage && s_sel[i] >= 0 && s_val[i] > -1e30f) atomicAdd(&a.usage[s_sel[i]], 1u);
        }
    }
    __syncwarp();
}

__global__ void k_router_topk(RouterArgs a, const float *logits) {
    __shared__ int taken[2048 / 32];
    __shared__ int s_sel[MAX_TOPK];
    __shared__ float s_val[MAX_TOPK];
    router_topk_warp(a, logits + (int64_t)blockIdx.x * a.n_experts, blockIdx.x, taken, s_sel, s_val);
}

constexpr int RL_THREADS = RG * 8 * 8;  // groups of 8 lanes: RG experts x 8 tokens

// blockIdx.y: group of 8 tokens; ticket null: no top-k here (a separate
// per-token kernel runs it)
__global__ void __launch_bounds__(RL_THREADS) k_router_logits(RouterArgs a, float *logits, unsigned *ticket) {
    extern __shared__ __align__(16) float rs_[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ unsigned s_last;
    __shared__ int taken[16][2048 / 32];
    __shared__ int s_sel[16][MAX_TOPK];
    __shared__ float s_val[16][MAX_TOPK];
    const int64_t H = a.hidden;
    const int64_t ld = ((H + 31) / 32) * 32 + 8;  // row stride: 8-lane groups of a warp in distinct banks
    float *ws = rs_;                 // [RG][ld]
    float *xs = rs_ + RG * ld;       // [n_tok][ld]
    const int e0 = blockIdx.x * RG;
    const int ne = min(RG, a.n_experts - e0);
    const int tok0 = blockIdx.y * 8, ntk = min(8, a.n_tok - tok0);
    const uint32_t rowb = (uint32_t)(H * 4);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, rowb * (uint32_t)(ne + ntk));
        for (int j = 0; j < ne; j++) bulk_g2s(ws + j * ld, a.rw + (int64_t)(e0 + j) * H, rowb, &bar);
    }
    // the normed rows come from the norm kernel: after its grid (a no-op
    // unless this launch is programmatic; the weights above are constant)
    pdl_wait();
    if (threadIdx.x == 0)
        for (int t = 0; t < ntk; t++) bulk_g2s(xs + t * ld, a.xb_out + (int64_t)(tok0 + t) * H, rowb, &bar);
    bool ok = true;
    if (threadIdx.x == 0) ok = mbar_wait(&bar, 0);
    if (!__syncthreads_and(ok)) {  // rows never arrived: report; the experts of this step are stale
        if (threadIdx.x == 0 && a.err) atomicExch(a.err, 3);
        return;
    }
    const int gi = threadIdx.x >> 3, lane8 = threadIdx.x & 7;
    const int j = gi % RG, t = gi / RG;
    const int64_t H8 = H & ~(int64_t)7;
    float acc = 0.f;
    const bool live = j < ne && t < ntk;
    if (live) {
        const float *wr = ws + j * ld + lane8, *xr8 = xs + t * ld + lane8;
#pragma unroll 8
        for (int64_t c = 0; c < H8; c += 8) acc = fmaf(wr[c], xr8[c], acc);
    }
    const float s1 = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    const float s2 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
    const float s3 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
    if (live && lane8 == 0) {
        float r = s3;
        for (int64_t c = H8; c < H; c++) r = __fadd_rn(r, __fmul_rn(ws[j * ld + c], xs[t * ld + c]));
        logits[(int64_t)(tok0 + t) * a.n_experts + e0 + j] = __fadd_rn(r, a.rb[e0 + j]);
    }
    if (!ticket) return;
    // the last block to finish selects the experts of every token
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1u) % gridDim.x == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    // every token's logits into shared memory once (the weight and token rows
    // are no longer needed), so the top-k rounds do not go back to L2
    const int nl = a.n_tok * a.n_experts;
    const bool stage = nl <= (RG + a.n_tok) * (int)ld;
    if (stage) {
        for (int i = threadIdx.x; i < nl; i += RL_THREADS) rs_[i] = logits[i];
        __syncthreads();
    }
    const float *lsrc = stage ? rs_ : logits;
    const int w = threadIdx.x >> 5;
    for (int tok = w; tok < a.n_tok; tok += RL_THREADS / 32)
        router_topk_warp(a, lsrc + (int64_t)tok * a.n_experts, tok, taken[w], s_sel[w], s_val[w]);
    if (threadIdx.x == 0) *ticket = 0;  // ready for the next launch
}

int router_split(const RouterArgs &a, float *logits_scratch, unsigned *ticket, cudaStream_t st) {
    MG_REQUIRE(a.x && a.norm_w && a.xb_out && a.rw && a.rb && a.sel && a.weights && logits_scratch && ticket &&
                   (!a.x_parts || (a.x_out && a.x_out != a.x)),
               MG_ERR_ARG, "router: bad arguments");
    MG_REQUIRE(a.top_k >= 1 && a.top_k <= MAX_TOPK && a.top_k <= a.n_experts && a.n_experts <= 2048 &&
                   a.n_tok <= 16,
               MG_ERR_ARG, "router: top_k %d / n_experts %d / n_tok %d unsupported", a.top_k, a.n_experts, a.n_tok);
    MG_REQUIRE((a.hidden * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.rw) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.xb_out) & 15) == 0,
               MG_ERR_ARG, "router: rows must be 16-byte aligned");
    if (a.n_tok == 0) return MG_OK;
    k_router_prep<<<a.n_tok, 1024, 0, st>>>(a);
    MG_CHECK_LAUNCH();
    const int64_t ld = ((a.hidden + 31) / 32) * 32 + 8;
    if (a.n_tok <= 8) {
        const size_t smem = (size_t)(RG + a.n_tok) * ld * 4;
        if (smem <= 200 * 1024) {
            int rc = ensure_smem(k_router_logits, smem);
            if (rc) return rc;
            MG_CUDA(launch_k(a.pdl != 0, k_router_logits, dim3((a.n_experts + RG - 1) / RG), dim3(RL_THREADS), smem,
                             st, a, logits_scratch, ticket));
            return MG_OK;
        }
    }
    // more tokens than one block's groups: logits per token through the
    // one-block-per-token router on the normed rows
    RouterArgs b = a;
    b.x = a.xb_out;
    b.norm_w = nullptr;
    b.x_parts = nullptr;
    b.logits = nullptr;
    return router(b, st);
}

// Prefill router: norm (block per token), logits (8 experts x 8 tokens per
// block, the AVX2 lane order), top-k per token with the prefill insertion
// variant.  logits_scratch: [n_tok x E].
int router_batch(const RouterArgs &a, float *logits_scratch, cudaStream_t st) {
    MG_REQUIRE(a.x && a.norm_w && a.xb_out && a.rw && a.rb && a.sel && a.weights && logits_scratch && !a.x_parts,
               MG_ERR_ARG, "router: bad arguments");
    MG_REQUIRE(a.top_k >= 1 && a.top_k <= MAX_TOPK && a.top_k <= a.n_experts && a.n_experts <= 2048, MG_ERR_ARG,
               "router: top_k %d / n_experts %d unsupported", a.top_k, a.n_experts);
    MG_REQUIRE((a.hidden * 4) % 16 == 0 && (reinterpret_cast<uintptr_t>(a.rw) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.xb_out) & 15) == 0,
               MG_ERR_ARG, "router: rows must be 16-byte aligned");
    if (a.n_tok == 0) return MG_OK;
    const int64_t ld = ((a.hidden + 31) / 32) * 32 + 8;
    const size_t smem = (size_t)(RG + 8) * ld * 4;
    if (smem > 200 * 1024) return router(a, st);
    k_router_prep<<<a.n_tok, 1024, 0, st>>>(a);
    MG_CHECK_LAUNCH();
    int rc = ensure_smem(k_router_logits, smem);
    if (rc) return rc;
    dim3 g((a.n_experts + RG - 1) / RG, (a.n_tok + 7) / 8);
    k_router_logits<<<g, RL_THREADS, smem, st>>>(a, logits_scratch, nullptr);
    MG_CHECK_LAUNCH();
    k_router_topk<<<a.n_tok, 32, 0, st>>>(a, logits_scratch);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int router(const RouterArgs &a, cudaStream_t st) {
    MG_REQUIRE(a.x && a.rw && a.rb && a.sel && a.weights && a.n_tok >= 0 && a.hidden > 0, MG_ERR_ARG,
               "router: bad arguments");
    MG_REQUIRE(a.top_k >= 1 && a.top_k <= MAX_TOPK && a.top_k <= a.n_experts && a.n_experts <= 2048, MG_ERR_ARG,
               "router: top_k %d / n_experts %d unsupported", a.top_k, a.n_experts);
    if (a.n_tok == 0) return MG_OK;
    size_t smem = (size_t)(a.hidden + a.n_experts) * 4;
    MG_REQUIRE(smem <= 160 * 1024, MG_ERR_ARG, "router: hidden %lld too large", (long long)a.hidden);
    int rc0 = ensure_smem(k_router, smem);
    if (rc0) return rc0;
    int threads = a.n_experts * 8;
    threads = threads < 256 ? 256 : threads > ROUTER_THREADS ? ROUTER_THREADS : (threads + 31) / 32 * 32;
    k_router<<<a.n_tok, threads, smem, st>>>(a);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// ----------------------------------------------- decode expert grouping
// Distinct experts of the n slots (sel[i] valid), in ascending expert id.
// Every block recomputes it from the (tiny) selection array, so no extra
// launch or global scratch is needed.  Returns the count; list[j] holds the
// j-th expert.  n <= MAX_SLOTS.
__device__ int distinct_experts(const int32_t *sel, int n, int n_experts, int *list) {
    __shared__ uint32_t bm[64];    // bitmap over <= 2048 experts
    __shared__ int wpre[65];       // set bits before each word
    for (int i = threadIdx.x; i < 64; i += blockDim.x) bm[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        int e = sel[i];
        if (e >= 0 && e < n_experts) atomicOr(&bm[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int c = 0;
        for (int w = 0; w < 64; w++) { wpre[w] = c; c += __popc(bm[w]); }
        wpre[64] = c;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < n_experts; e += blockDim.x) {
        uint32_t word = bm[e >> 5], bit = 1u << (e & 31);
        if (word & bit) list[wpre[e >> 5] + __popc(word & (bit - 1))] = e;
    }
    __syncthreads();
    return wpre[64];
}

// slots (ascending) routed to expert e; returns their count (<= 16 kept)
__device__ int expert_slots(const int32_t *sel, int n, int e, int *slots) {
    __shared__ int c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int k = 0;
        for (int i = 0; i < n && k < 16; i++) if (sel[i] == e) slots[k++] = i;
        c = k;
    }
    __syncthreads();
    return c;
}

__device__ __forceinline__ float act_fn(float g, float u, int plain, float alpha, float limit) {
    if (plain) return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);  // silu(g)*u, engine/midge.c:528
    if (g > limit) g = limit;                                                  // engine/midge.c:532-537
    if (u > limit) u = limit;
    if (u < -limit) u = -limit;
    float act = __fdiv_rn(g, __fadd_rn(1.0f, expf(__fmul_rn(-alpha, g))));
    return __fmul_rn(act, __fadd_rn(u, 1.0f));
}

// gate+up tile of one routed expert -> activation -> h rows of its slots
template <int DT, int SC, int NT>
__global__ void __launch_bounds__(GEMV_THREADS) k_moe_gateup(MoeArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int list[MAX_SLOTS];
    __shared__ int slots[16];
    const int n = a.n_tok * a.top_k;
    int nd = distinct_experts(a.sel, n, a.n_experts, list);
    if ((int)blockIdx.y >= nd) return;
    const int e = list[blockIdx.y];
    const int ne = min(expert_slots(a.sel, n, e, slots), NT * 4);  // > NT*4 only with degenerate routing
    const mg_expert_layout *L = &a.L;
    const int H = (int)L->hidden, F = (int)L->ffn;
    const int ncol = NT * 8, xs_stride = H + XS_PAD;
    __half *xs = reinterpret_cast<__half *>(smem);
    float *red = reinterpret_cast<float *>(smem + (size_t)ncol * xs_stride * 2);

    const uint8_t *eb = a.experts_layer + (int64_t)e * L->expert_stride;
    const int64_t rbase = (int64_t)blockIdx.x * 16;
    using Tile = GemvTile<DT, SC, 2, NT>;
    int c0, c1;
    warp_chunk_range(H / Tile::CHUNK, c0, c1);
    prefetch_tile<DT, SC>(eb + L->off[0][0], eb + L->off[0][1], rbase, F, H, c0, c1);
    prefetch_tile<DT, SC>(eb + L->off[1][0], eb + L->off[1][1], rbase, F, H, c0, c1);
    // stage xb of the routed tokens (column 2j/2j+1 = token of slot j)
    for (int j = 0; j < ne; j++)
        stage_x<DT>(a.xb + (int64_t)(slots[j] / a.top_k) * H, H, 1, H, xs + 2 * j * xs_stride, xs_stride);
    __syncthreads();

    const uint8_t *wp[2] = {eb + L->off[0][0], eb + L->off[1][0]};
    const uint8_t *sp[2] = {eb + L->off[0][1], eb + L->off[1][1]};
    const int64_t r0[2] = {rbase, rbase};
    float acc[2][NT][4];
#pragma unroll
    for (int m = 0; m < 2; m++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[m][nt][i] = 0.f;
    Tile::run(wp, sp, r0, F, H, c0, c1, xs, xs_stride, (ne + 3) >> 2, acc);
    gemv_block_reduce<2, NT>(acc, red);

    const float *bg = reinterpret_cast<const float *>(eb + L->off[0][2]);
    const float *bu = reinterpret_cast<const float *>(eb + L->off[1][2]);
    const float *sg = reinterpret_cast<const float *>(eb + L->off[0][1]);
    const float *su = reinterpret_cast<const float *>(eb + L->off[1][1]);
    for (int j = threadIdx.x; j < 16 * ne; j += blockDim.x) {
        int s = j >> 4, rl = j & 15;
        int64_t r = rbase + rl;
        if (r >= F) continue;
        float g = gemv_out<NT>(red, 0, rl, s), u = gemv_out<NT>(red, 1, rl, s);
        if (DT == MG_Q8R) { g = __fmul_rn(g, sg[r]); u = __fmul_rn(u, su[r]); }
        g = __fadd_rn(g, bg[r]);
        u = __fadd_rn(u, bu[r]);
        a.h[(int64_t)slots[s] * F + r] = act_fn(g, u, a.act_plain, a.alpha, a.limit);
    }
}

// down tile over every routed expert, then the rank-order weighted combine
// into the residual (engine/midge.c:542-548)
template <int DT, int SC, int NT>
__global__ void __launch_bounds__(GEMV_THREADS) k_moe_down(MoeArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int list[MAX_SLOTS];
    __shared__ int slots[16];
    const int n = a.n_tok * a.top_k;
    const mg_expert_layout *L = &a.L;
    const int H = (int)L->hidden, F = (int)L->ffn;
    const int ncol = NT * 8, xs_stride = F + XS_PAD;
    __half *xs = reinterpret_cast<__half *>(smem);
    float *red = reinterpret_cast<float *>(smem + (size_t)ncol * xs_stride * 2);
    float *ys = red + GEMV_WARPS * NT * 32 * 4;  // [n][16]
    const int64_t rbase = (int64_t)blockIdx.x * 16;
    int nd = distinct_experts(a.sel, n, a.n_experts, list);
    for (int i = threadIdx.x; i < n * 16; i += blockDim.x) ys[i] = 0.f;

    for (int d = 0; d < nd; d++) {
        const int e = list[d];
        const int ne = min(expert_slots(a.sel, n, e, slots), NT * 4);  // syncs before and after
        const uint8_t *eb = a.experts_layer + (int64_t)e * L->expert_stride;
        using Tile = GemvTile<DT, SC, 1, NT>;
        int c0, c1;
        warp_chunk_range(F / Tile::CHUNK, c0, c1);
        prefetch_tile<DT, SC>(eb + L->off[2][0], eb + L->off[2][1], rbase, H, F, c0, c1);
        for (int j = 0; j < ne; j++)
            stage_x<DT>(a.h + (int64_t)slots[j] * F, F, 1, F, xs + 2 * j * xs_stride, xs_stride);
        __syncthreads();
        const uint8_t *wp[1] = {eb + L->off[2][0]};
        const uint8_t *sp[1] = {eb + L->off[2][1]};
        const int64_t r0[1] = {rbase};
        float acc[1][NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[0][nt][i] = 0.f;
        Tile::run(wp, sp, r0, H, F, c0, c1, xs, xs_stride, (ne + 3) >> 2, acc);
        gemv_block_reduce<1, NT>(acc, red);
        const float *bd = reinterpret_cast<const float *>(eb + L->off[2][2]);
        const float *sd = reinterpret_cast<const float *>(eb + L->off[2][1]);
        for (int j = threadIdx.x; j < 16 * ne; j += blockDim.x) {
            int s = j >> 4, rl = j & 15;
            int64_t r = rbase + rl;
            if (r >= H) continue;
            float v = gemv_out<NT>(red, 0, rl, s);
            if (DT == MG_Q8R) v = __fmul_rn(v, sd[r]);
            ys[slots[s] * 16 + rl] = __fadd_rn(v, bd[r]);
        }
        __syncthreads();
    }
    for (int j = threadIdx.x; j < a.n_tok * 16; j += blockDim.x) {
        int t = j >> 4, rl = j & 15;
        int64_t r = rbase + rl;
        if (r >= H) continue;
        float moe = 0.f;
        for (int i = 0; i < a.top_k; i++) {
            int e = a.sel[t * a.top_k + i];
            if (e < 0 || e >= a.n_experts) continue;
            moe = __fadd_rn(moe, __fmul_rn(a.weights[t * a.top_k + i], ys[(t * a.top_k + i) * 16 + rl]));
        }
        float *xp = a.x + (int64_t)t * a.ldx + r;
        *xp = __fadd_rn(*xp, moe);
    }
}

template <int DT, int SC, int NT>
static int moe_decode_t(const MoeArgs &a, cudaStream_t st) {
    const int H = (int)a.L.hidden, F = (int)a.L.ffn;
    size_t s1 = (size_t)NT * 8 * (H + XS_PAD) * 2 + (size_t)GEMV_WARPS * 2 * NT * 32 * 4 * 4;
    int rc = ensure_smem(k_moe_gateup<DT, SC, NT>, s1);
    if (rc) return rc;
    dim3 g1(ceil_div(F, 16), a.n_tok * a.top_k);
    k_moe_gateup<DT, SC, NT><<<g1, GEMV_THREADS, s1, st>>>(a);
    MG_CHECK_LAUNCH();
    size_t s2 = (size_t)NT * 8 * (F + XS_PAD) * 2 + (size_t)GEMV_WARPS * NT * 32 * 4 * 4 +
                (size_t)a.n_tok * a.top_k * 16 * 4;
    rc = ensure_smem(k_moe_down<DT, SC, NT>, s2);
    if (rc) return rc;
    k_moe_down<DT, SC, NT><<<ceil_div(H, 16), GEMV_THREADS, s2, st>>>(a);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

template <int DT, int SC>
static int moe_decode_nt(const MoeArgs &a, cudaStream_t st) {
    if (a.n_tok <= 4) return moe_decode_t<DT, SC, 1>(a, st);
    if (a.n_tok <= 8) return moe_decode_t<DT, SC, 2>(a, st);
    return moe_decode_t<DT, SC, 4>(a, st);
}

// f32 experts (test containers): one warp per output row, lanes over columns.
__global__ void k_moe_f32_gateup(MoeArgs a) {
    const int slot = blockIdx.y, t = slot / a.top_k, e = a.sel[slot];
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t H = a.L.hidden, F = a.L.ffn;
    if (e < 0 || e >= a.n_experts || r >= F) return;
    const uint8_t *eb = a.experts_layer + (int64_t)e * a.L.expert_stride;
    const float *wg = reinterpret_cast<const float *>(eb + a.L.off[0][0]) + r * H;
    const float *wu = reinterpret_cast<const float *>(eb + a.L.off[1][0]) + r * H;
    const float *xb = a.xb + (int64_t)t * H;
    float g = 0.f, u = 0.f;
    for (int64_t c = lane; c < H; c += 32) { g = fmaf(wg[c], xb[c], g); u = fmaf(wu[c], xb[c], u); }
    g = warp_sum(g);
    u = warp_sum(u);
    if (lane == 0) {
        g = __fadd_rn(g, reinterpret_cast<const float *>(eb + a.L.off[0][2])[r]);
        u = __fadd_rn(u, reinterpret_cast<const float *>(eb + a.L.off[1][2])[r]);
        a.h[(int64_t)slot * F + r] = act_fn(g, u, a.act_plain, a.alpha, a.limit);
    }
}

__global__ void k_moe_f32_down(MoeArgs a) {
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int64_t H = a.L.hidden, F = a.L.ffn;
    if (r >= H) return;
    float moe = 0.f;
    for (int i = 0; i < a.top_k; i++) {
        const int slot = t * a.top_k + i, e = a.sel[slot];
        if (e < 0 || e >= a.n_experts) continue;
        const uint8_t *eb = a.experts_layer + (int64_t)e * a.L.expert_stride;
        const float *wd = reinterpret_cast<const float *>(eb + a.L.off[2][0]) + r * F;
        const float *hr = a.h + (int64_t)slot * F;
        float y = 0.f;
        for (int64_t c = lane; c < F; c += 32) y = fmaf(wd[c], hr[c], y);
        y = __fadd_rn(warp_sum(y), reinterpret_cast<const float *>(eb + a.L.off[2][2])[r]);
        moe = __fadd_rn(moe, __fmul_rn(a.weights[slot], y));
    }
    if (lane == 0) {
        float *xp = a.x + (int64_t)t * a.ldx + r;
        *xp = __fadd_rn(*xp, moe);
    }
}

int moe_decode(const MoeArgs &a, cudaStream_t st) {
    MG_REQUIRE(a.experts_layer && a.xb && a.sel && a.weights && a.h && a.x, MG_ERR_ARG, "moe: null argument");
    MG_REQUIRE(a.n_tok >= 1 && a.n_tok <= 16 && a.top_k >= 1 && a.top_k <= MAX_TOPK &&
                   a.n_tok * a.top_k <= MAX_SLOTS,
               MG_ERR_ARG, "moe: n_tok %d top_k %d unsupported", a.n_tok, a.top_k);
    const mg_expert_layout *L = &a.L;
    switch (L->dt) {
    case MG_MXFP4:
        MG_REQUIRE(L->hidden % 32 == 0 && L->ffn % 32 == 0, MG_ERR_ARG, "moe: dims must be multiples of 32");
        return L->scale_fmt == MG_SCALE_UE8M0 ? moe_decode_nt<MG_MXFP4, MG_SCALE_UE8M0>(a, st)
                                              : moe_decode_nt<MG_MXFP4, MG_SCALE_F16>(a, st);
    case MG_Q4G32:
        MG_REQUIRE(L->hidden % 32 == 0 && L->ffn % 32 == 0, MG_ERR_ARG, "moe: dims must be multiples of 32");
        return L->scale_fmt == MG_SCALE_UE8M0 ? moe_decode_nt<MG_Q4G32, MG_SCALE_UE8M0>(a, st)
                                              : moe_decode_nt<MG_Q4G32, MG_SCALE_F16>(a, st);
    case MG_Q8R:
        if (L->hidden % 64 == 0 && L->ffn % 64 == 0) return moe_decode_nt<MG_Q8R, MG_SCALE_F16>(a, st);
        break;
    case MG_F32: {
        dim3 g1(ceil_div(L->ffn, 8), a.n_tok * a.top_k), g2(ceil_div(L->hidden, 8), a.n_tok);
        k_moe_f32_gateup<<<g1, 256, 0, st>>>(a);
        MG_CHECK_LAUNCH();
        k_moe_f32_down<<<g2, 256, 0, st>>>(a);
        MG_CHECK_LAUNCH();
        return MG_OK;
    }
    default:
        break;
    }
    set_error("moe: expert dtype %d has no decode kernel", L->dt);
    return MG_ERR_ARG;
}

}  // namespace mg

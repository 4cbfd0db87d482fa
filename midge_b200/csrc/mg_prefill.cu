// mg_prefill.cu -- expert-major batched prefill of the routed experts
// (engine/midge.c:576-622 restated for the tensor cores): route every token,
// group the (token, rank) slots by expert, run each expert's gate/up and down
// projections as grouped tcgen05 GEMMs over its tokens, then add
// w * y into every token's residual in ascending expert order, as the
// reference's expert loop does (engine/midge.c:595-611).
#include "mg_common.cuh"
#include "mg_gemm.h"
#include "mg_kernels.h"
#include "mg_prefill.h"
#include "mg_ep_xchg.h"

namespace mg {

constexpr int PF_TILE_N = 128;

// histogram of the slots over this rank's experts (local index e - e0)
__global__ void k_pf_count(const int32_t *__restrict__ sel, int nslots, int e0, int n_local, int *counts) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nslots; i += gridDim.x * blockDim.x) {
        const int e = sel[i] - e0;
        if (e >= 0 && e < n_local) atomicAdd(&counts[e], 1);
    }
}

// offsets of each expert's rows, N-tile list (one thread: E is small)
__global__ void k_pf_tiles(const int *counts, int n_experts, int *offs, int *cursor, XgTile *tiles, int *ntiles,
                           int max_tiles) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int off = 0, nt = 0;
    for (int e = 0; e < n_experts; e++) {
        offs[e] = off;
        cursor[e] = 0;
        const int c = counts[e];
        for (int r = 0; r < c && nt < max_tiles; r += PF_TILE_N) tiles[nt++] = XgTile{e, r, min(PF_TILE_N, c - r)};
        off += c;
    }
    offs[n_experts] = off;
    *ntiles = nt;
}

// expert-major position of every slot (order inside an expert is arbitrary:
// every row of a GEMM tile is computed independently of the others)
__global__ void k_pf_scatter(const int32_t *__restrict__ sel, int nslots, int e0, int n_local, const int *offs,
                             int *cursor, int *pos_of_slot, int *slot_of_pos) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nslots; i += gridDim.x * blockDim.x) {
        const int e = sel[i] - e0;
        if (e >= 0 && e < n_local) {
            const int p = offs[e] + atomicAdd(&cursor[e], 1);
            pos_of_slot[i] = p;
            slot_of_pos[p] = i;
        } else {
            pos_of_slot[i] = -1;
        }
    }
}

// X rows in expert-major order as f16 hi/lo
__global__ void k_pf_gather(const float *__restrict__ xb, int64_t ldx, int64_t H, int top_k,
                            const int *__restrict__ slot_of_pos, const int *offs_end, __half *hi, __half *lo) {
    const int64_t P = *offs_end;
    const int64_t n8 = H / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < P * n8; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t p = i / n8, c = (i - p * n8) * 8;
        const int t = slot_of_pos[p] / top_k;
        const float4 *src = reinterpret_cast<const float4 *>(xb + (int64_t)t * ldx + c);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        __half h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; j++) split_f16(v[j], h[j], l[j]);
        *reinterpret_cast<uint4 *>(hi + p * H + c) = *reinterpret_cast<uint4 *>(h);
        *reinterpret_cast<uint4 *>(lo + p * H + c) = *reinterpret_cast<uint4 *>(l);
    }
}

// dense activations [n x K] -> f16 hi/lo (rows of x at stride ldx)
__global__ void k_split_rows(const float *__restrict__ x, int64_t ldx, int n, int64_t K, __half *hi, __half *lo) {
    const int64_t n8 = K / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)n * n8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n8, c = (i - r * n8) * 8;
        const float4 *src = reinterpret_cast<const float4 *>(x + r * ldx + c);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        __half h[8], l[8];
#pragma unroll
        for (int j = 0; j < 8; j++) split_f16(v[j], h[j], l[j]);
        *reinterpret_cast<uint4 *>(hi + r * K + c) = *reinterpret_cast<uint4 *>(h);
        *reinterpret_cast<uint4 *>(lo + r * K + c) = *reinterpret_cast<uint4 *>(l);
    }
}

// x[t] += w * y per routed expert in ascending expert id (engine/midge.c:595-611, :466);
// Y is slot-major (row t*top_k + i)
__global__ void k_pf_combine(float *x, int64_t H, const int32_t *__restrict__ sel, const float *__restrict__ w,
                             int top_k, int n_experts, const float *__restrict__ Y, const int *__restrict__ slot_row) {
    const int t = blockIdx.x;
    int ord[16];
    int k = 0;
    for (int i = 0; i < top_k; i++) {  // slots of this token sorted by expert id (stable)
        const int e = sel[t * top_k + i];
        if (e < 0 || e >= n_experts) continue;
        int j = k++;
        while (j > 0 && sel[t * top_k + ord[j - 1]] > e) { ord[j] = ord[j - 1]; j--; }
        ord[j] = i;
    }
    float *xr = x + (int64_t)t * H;
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
        float acc = xr[c];
        for (int j = 0; j < k; j++) {
            const int i = ord[j];
            const int64_t row = slot_row ? slot_row[t * top_k + i] : t * top_k + i;
            acc = __fadd_rn(acc, __fmul_rn(w[t * top_k + i], Y[row * H + c]));
        }
        xr[c] = acc;
    }
}

// largest nonzero ue8m0 code of each (layer, expert, matrix) scale blob ->
// rebase exponent (code - 127 - 12); counts matrices whose codes span more
// than 35 binades (their smallest values would not survive the f16 rebase)
__global__ void k_pf_rebase(const uint8_t *experts, mg_expert_layout L, int n_experts, int *rebase, int *inexact) {
    const int idx = blockIdx.x;  // (layer * E + e) * 3 + m
    const int m = idx % 3;
    const int64_t le = idx / 3;
    const uint8_t *sc = experts + le * L.expert_stride + L.off[m][1];
    const int64_t rows = m == 2 ? L.hidden : L.ffn, cols = m == 2 ? L.ffn : L.hidden;
    const int64_t n = rows * (cols / 32);
    int mx = 0, mn = 255;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int u = sc[i];
        if (u) { mx = max(mx, u); mn = min(mn, u); }
    }
    __shared__ int smx, smn;
    if (threadIdx.x == 0) { smx = 0; smn = 255; }
    __syncthreads();
    atomicMax(&smx, mx);
    atomicMin(&smn, mn);
    __syncthreads();
    if (threadIdx.x == 0) {
        rebase[idx] = smx ? smx - 127 - 12 : 0;
        if (smx && smx - smn > 35) atomicAdd(inexact, 1);
    }
}

int pf_rebase(const uint8_t *experts, const mg_expert_layout &L, int n_layers, int n_experts, int *rebase, int *inexact,
              cudaStream_t st) {
    k_pf_rebase<<<n_layers * n_experts * 3, 256, 0, st>>>(experts, L, n_experts, rebase, inexact);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int split_rows(const float *x, int64_t ldx, int n, int64_t K, __half *hi, __half *lo, cudaStream_t st) {
    MG_REQUIRE(K % 8 == 0 && ldx % 4 == 0, MG_ERR_ARG, "split_rows: K %% 8");
    int64_t tot = (int64_t)n * (K / 8);
    int grid = ceil_div(tot, 256);
    if (grid > 148 * 16) grid = 148 * 16;
    if (grid < 1) grid = 1;
    k_split_rows<<<grid, 256, 0, st>>>(x, ldx, n, K, hi, lo);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// dense q8r GEMM over n token rows: y[n x rows] (=|+=) W x + bias
int dense_gemm(const DenseGemm &d, cudaStream_t st) {
    XgLaunch l{};
    l.args.dense_w = (const uint8_t *)d.w;
    l.args.dense_s = (const uint8_t *)d.scales;
    l.args.dense_bias = d.bias;
    l.args.M = d.rows;
    l.args.K = d.cols;
    l.args.n_rows = d.n;
    l.args.y = d.y;
    l.args.ldy = d.ldy;
    l.args.accumulate = d.accumulate;
    l.args.err = d.err;
    l.x_hi = d.x_hi;
    l.x_lo = d.x_lo;
    l.x_rows = d.n;
    l.max_tiles = (d.n + PF_TILE_N - 1) / PF_TILE_N;
    return xgemm(XG_DENSE, MG_Q8R, l, st);
}

int moe_prefill_experts(const MoePrefill &a, cudaStream_t st) {
    const int nslots = a.n * a.top_k;
    const int E = a.n_local;
    if (nslots <= 0) return MG_OK;
    const int64_t ldx = a.ldx ? a.ldx : a.L.hidden;
    MG_REQUIRE(ldx % 4 == 0, MG_ERR_ARG, "moe_prefill: activation stride %lld not a multiple of 4", (long long)ldx);
    MG_CUDA(cudaMemsetAsync(a.counts, 0, (size_t)E * sizeof(int), st));
    int g = ceil_div(nslots, 256);
    k_pf_count<<<g, 256, 0, st>>>(a.sel, nslots, a.e0, E, a.counts);
    MG_CHECK_LAUNCH();
    const int max_tiles = (nslots + PF_TILE_N - 1) / PF_TILE_N + E;
    k_pf_tiles<<<1, 32, 0, st>>>(a.counts, E, a.offs, a.cursor, a.tiles, a.ntiles, max_tiles);
    MG_CHECK_LAUNCH();
    k_pf_scatter<<<g, 256, 0, st>>>(a.sel, nslots, a.e0, E, a.offs, a.cursor, a.pos_of_slot, a.slot_of_pos);
    MG_CHECK_LAUNCH();
    int gg = ceil_div((int64_t)nslots * (a.L.hidden / 8), 256);
    if (gg > 148 * 16) gg = 148 * 16;
    k_pf_gather<<<gg, 256, 0, st>>>(a.xb, ldx, a.L.hidden, a.top_k, a.slot_of_pos, a.offs + E, a.x_hi, a.x_lo);
    MG_CHECK_LAUNCH();
    XgLaunch l{};
    l.args.L = a.L;
    l.args.experts_layer = a.experts_layer;
    l.args.tiles = a.tiles;
    l.args.ntiles = a.ntiles;
    l.args.offs = a.offs;
    l.args.rebase = a.rebase;
    l.args.act_plain = a.act_plain;
    l.args.alpha = a.alpha;
    l.args.limit = a.limit;
    l.args.err = a.err;
    l.max_tiles = max_tiles;
    // gate/up -> h (f16 hi/lo)
    l.args.M = a.L.ffn;
    l.args.K = a.L.hidden;
    l.args.out_hi = a.h_hi;
    l.args.out_lo = a.h_lo;
    l.x_hi = a.x_hi;
    l.x_lo = a.x_lo;
    l.x_rows = nslots;
    int rc = xgemm(XG_GATEUP, a.L.dt, l, st);
    if (rc) return rc;
    // down -> y: slot-major, or at out_row[slot] (expert parallel: the return rows)
    const int *slot_rows = a.slot_of_pos;
    if (a.out_row) {
        MG_REQUIRE(a.slot2, MG_ERR_ARG, "moe_prefill: out_row needs slot2 scratch");
        rc = ep_pf_remap(a.slot_of_pos, a.offs + E, a.out_row, nslots, a.slot2, st);
        if (rc) return rc;
        slot_rows = a.slot2;
    }
    l.args.M = a.L.hidden;
    l.args.K = a.L.ffn;
    l.args.slot_of_pos = slot_rows;
    l.args.y = a.y;
    l.args.ldy = a.L.hidden;
    l.x_hi = a.h_hi;
    l.x_lo = a.h_lo;
    return xgemm(XG_DOWN, a.L.dt, l, st);
}

int pf_combine(float *x, int64_t H, const int32_t *sel, const float *w, int n, int top_k, int n_experts, const float *Y,
               const int *slot_row, cudaStream_t st) {
    if (n <= 0) return MG_OK;
    k_pf_combine<<<n, 256, 0, st>>>(x, H, sel, w, top_k, n_experts, Y, slot_row);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int moe_prefill(const MoePrefill &a, cudaStream_t st) {
    int rc = moe_prefill_experts(a, st);
    if (rc) return rc;
    return pf_combine(a.x, a.L.hidden, a.sel, a.w, a.n, a.top_k, a.n_experts, a.y, nullptr, st);
}

}  // namespace mg

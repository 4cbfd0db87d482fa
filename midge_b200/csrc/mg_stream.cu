// mg_stream.cu -- launchers of the streamed (bulk-copy ring) decode GEMV.
#include <cstring>

#include "mg_kernels.h"
#include "mg_bsmoe.h"
#include "mg_stream.cuh"

namespace mg {

// Error word of the streamed kernels (bounded mbarrier waits), one per device.
static int *sw_err_ptr() {
    static int *p[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!p[dev]) {
        if (cudaMalloc(&p[dev], sizeof(int)) != cudaSuccess) return nullptr;
        cudaMemset(p[dev], 0, sizeof(int));
    }
    return p[dev];
}

int stream_error_check() {
    int *e = sw_err_ptr();
    MG_REQUIRE(e, MG_ERR_CUDA, "stream: no error word");
    int h = 0;
    MG_CUDA(cudaMemcpy(&h, e, sizeof(int), cudaMemcpyDeviceToHost));
    if (h) {
        cudaMemset(e, 0, sizeof(int));
        set_error("streamed GEMV: a bounded wait timed out (code %d)", h);
        return MG_ERR_TIMEOUT;
    }
    return MG_OK;
}

int stream_prepare() { return sw_err_ptr() ? MG_OK : MG_ERR_OOM; }

int *stream_error_word() { return sw_err_ptr(); }

int stream_ksplit(int dt, int64_t cols, int want) {
    const int64_t segb = SW_SEGB;
    const int64_t rowbytes = dt == MG_Q8R ? cols : cols / 2;
    const int64_t nseg = (rowbytes + segb - 1) / segb;
    int ks = want > 0 ? want : 1;
    if (ks > nseg) ks = (int)nseg;
    const int64_t sps = (nseg + ks - 1) / ks;
    return (int)((nseg + sps - 1) / sps);
}

// Shared memory: [alignment slack][barriers][ring of nstages][sw_nslot scale slots of
// ssb bytes][partial-sum hand-over][activations].  Scale slots are dropped (ssb = 0: per-lane scale
// loads) when they would leave fewer than 4 ring stages.
template <int DT, class P>
static int launch_policy(void (*kfn)(SwMaps, P, int, int, int *), const SwMaps &maps, P &pol, size_t xs_bytes,
                         size_t ssb, int grid, cudaStream_t st) {
    cudaFuncAttributes fa{};
    MG_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(kfn)));
    const size_t budget = 227 * 1024 - fa.sharedSizeBytes - 1024;  // static shared memory and the alignment slack
    ssb = (ssb + 127) & ~(size_t)127;
    xs_bytes += SW_RED_BYTES;  // the partial-sum hand-over sits just before the activations
    constexpr size_t NS = sw_nslot(DT);
    if (ssb && budget < 1024 + xs_bytes + NS * ssb + 4 * (size_t)SW_STAGE_BYTES) ssb = 0;
    MG_REQUIRE(budget > 1024 + xs_bytes + NS * ssb, MG_ERR_ARG, "streamed kernel: activations leave no room for a ring");
    int nstages = (int)((budget - 1024 - xs_bytes - NS * ssb) / SW_STAGE_BYTES);
    if (nstages > SW_MAX_STAGES) nstages = SW_MAX_STAGES;
    MG_REQUIRE(nstages >= 2, MG_ERR_ARG, "streamed kernel: activations leave no room for a ring");
    const size_t smem = 1024 + 1024 + (size_t)nstages * SW_STAGE_BYTES + NS * ssb + xs_bytes;
    int rc = ensure_smem_attr(reinterpret_cast<const void *>(kfn), smem);
    if (rc) return rc;
    int *err = sw_err_ptr();
    MG_REQUIRE(err, MG_ERR_OOM, "streamed kernel: no error word");
    kfn<<<grid, SW_THREADS, smem, st>>>(maps, pol, nstages, (int)ssb, err);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

template <int DT, int SC, int NT>
static int launch_stream_gemv(const StreamGemvArgs &a, cudaStream_t st) {
    PolGemv<DT, SC> pol{};
    SwMaps maps;
    memset(&maps, 0, sizeof(maps));
    const int64_t rowbytes = DT == MG_Q8R ? a.cols : a.cols / 2;
    int64_t tiles = 0;
    for (int i = 0; i < a.nmat; i++) {
        if (a.mat[i].map) {
            maps.m[i] = *a.mat[i].map;
        } else {
            int rc = map_weights_2d(&maps.m[i], a.mat[i].w, rowbytes, a.mat[i].rows, SW_ROWS);
            if (rc) return rc;
        }
        pol.m[i].sc = (const uint8_t *)a.mat[i].scales;
        pol.m[i].bias = a.mat[i].bias;
        pol.m[i].rows = a.mat[i].rows;
        pol.m[i].y = a.mat[i].y;
        pol.m[i].ldy = a.mat[i].ldy;
        pol.m[i].tile0 = tiles;
        tiles += (a.mat[i].rows + SW_ROWS - 1) / SW_ROWS;
    }
    pol.nmat = a.nmat;
    pol.cols = (int)a.cols;
    pol.ntiles = tiles;
    const int ks = stream_ksplit(DT, a.cols, a.ksplit);
    const int64_t nseg = (rowbytes + SW_SEGB - 1) / SW_SEGB;
    pol.ks_count = ks;
    pol.kbytes_per_split = ((nseg + ks - 1) / ks) * SW_SEGB;
    pol.x = a.x;
    pol.ldx = a.ldx;
    pol.n_tok = a.n_tok;
    pol.accumulate = a.accumulate;
    pol.part_stride = a.part_stride;
    pol.amax = ks == 1 ? a.amax : nullptr;
    const size_t xs_bytes = (size_t)NT * 8 * sw_xs_stride<DT>(a.cols) * 2;
    const int64_t units = tiles * ks;
    const int nsm = num_sms();
    // scale slots need every matrix's scale blob 16-byte aligned and a whole
    // number of 16-byte pieces long (the last tile's copy ends at the blob's end)
    size_t ssb = 0;
    if (DT == MG_Q8R) {  // row scales (+ biases) through the scale slots: 16-byte aligned, rows % 4 == 0
        bool fits = true;
        for (int i = 0; i < a.nmat; i++)
            fits = fits && (reinterpret_cast<uintptr_t>(a.mat[i].scales) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.mat[i].bias) & 15) == 0 && a.mat[i].rows % 4 == 0;
        if (fits) ssb = (size_t)SW_ROWS * 4 * 2;
    } else {
        const int64_t sb = SC == MG_SCALE_UE8M0 ? 1 : 2;
        bool fits = true;
        for (int i = 0; i < a.nmat; i++)
            fits = fits && (reinterpret_cast<uintptr_t>(a.mat[i].scales) & 15) == 0 &&
                   (a.mat[i].rows * (a.cols / 32) * sb) % 16 == 0;
        if (fits) ssb = (size_t)SW_ROWS * (a.cols / 32) * sb;
    }
    return launch_policy<DT>(k_stream<DT, SC, NT, PolGemv<DT, SC>>, maps, pol, xs_bytes, ssb,
                             (int)(units < nsm ? units : nsm), st);
}

template <int DT, int SC>
static int stream_gemv_nt(const StreamGemvArgs &a, cudaStream_t st) {
    if (a.n_tok <= 4) return launch_stream_gemv<DT, SC, 1>(a, st);
    return launch_stream_gemv<DT, SC, 2>(a, st);
}

int stream_gemv(const StreamGemvArgs &a, cudaStream_t st) {
    MG_REQUIRE(a.nmat >= 1 && a.nmat <= 3 && a.x && a.n_tok >= 1 && a.n_tok <= 8 && a.cols > 0, MG_ERR_ARG,
               "streamed gemv: bad arguments");
    for (int i = 0; i < a.nmat; i++)
        MG_REQUIRE(a.mat[i].w && a.mat[i].y && a.mat[i].rows > 0 && a.mat[i].scales, MG_ERR_ARG,
                   "streamed gemv: matrix %d incomplete", i);
    MG_REQUIRE(((reinterpret_cast<uintptr_t>(a.x) & 15) == 0) && (a.ldx % 4 == 0), MG_ERR_ARG,
               "streamed gemv: activations must be 16-byte aligned");
    switch (a.dt) {
    case MG_MXFP4:
        MG_REQUIRE(a.cols % 32 == 0, MG_ERR_ARG, "streamed gemv: cols %% 32");
        return a.scale_fmt == MG_SCALE_UE8M0 ? stream_gemv_nt<MG_MXFP4, MG_SCALE_UE8M0>(a, st)
                                             : stream_gemv_nt<MG_MXFP4, MG_SCALE_F16>(a, st);
    case MG_Q4G32:
        MG_REQUIRE(a.cols % 32 == 0, MG_ERR_ARG, "streamed gemv: cols %% 32");
        return a.scale_fmt == MG_SCALE_UE8M0 ? stream_gemv_nt<MG_Q4G32, MG_SCALE_UE8M0>(a, st)
                                             : stream_gemv_nt<MG_Q4G32, MG_SCALE_F16>(a, st);
    case MG_Q8R:
        MG_REQUIRE(a.cols % 64 == 0, MG_ERR_ARG, "streamed gemv: q8r cols %% 64");
        return stream_gemv_nt<MG_Q8R, MG_SCALE_F16>(a, st);
    }
    set_error("streamed gemv: dtype %d unsupported", a.dt);
    return MG_ERR_ARG;
}

// ------------------------------------------------------- routed experts
template <int DT, int SC, int NT>
static int moe_stream_t(const MoeStreamArgs &a, cudaStream_t st) {
    const int nsm = num_sms();
    SwMaps maps;
    for (int i = 0; i < 3; i++) maps.m[i] = a.maps[i];
    PolMoeGateUp<DT, SC> pg{};
    pg.L = a.L;
    pg.experts_layer = a.experts_layer;
    pg.layer = a.layer;
    pg.e0 = a.e0;
    pg.n_experts = a.n_experts;
    pg.n_tok = a.n_tok;
    pg.top_k = a.top_k;
    pg.sel = a.sel;
    pg.xb = a.xb;
    pg.act_plain = a.act_plain;
    pg.alpha = a.alpha;
    pg.limit = a.limit;
    pg.h = a.h;
    // scale slots: the expert blob's scale regions are 64-byte aligned and
    // padded, so a copy rounded up to 16 bytes stays inside them
    const size_t sb = SC == MG_SCALE_UE8M0 ? 1 : 2;
    // (+ the tile's biases, whose runs are whole 16-byte pieces when the row
    // counts are multiples of 4)
    pg.bias_ss = DT != MG_Q8R && a.L.ffn % 4 == 0;
    const size_t ssb_gu = DT == MG_Q8R ? 0 : 2 * 64 * (size_t)(a.L.hidden / 32) * sb + (pg.bias_ss ? 512 : 0);
    const size_t ssb_dn =
        DT == MG_Q8R ? 0 : (size_t)SW_ROWS * (a.L.ffn / 32) * sb + (a.L.hidden % 4 == 0 ? SW_ROWS * 4 : 0);
    int rc = launch_policy<DT>(k_stream<DT, SC, NT, PolMoeGateUp<DT, SC>>, maps, pg,
                               (size_t)NT * 8 * sw_xs_stride<DT>(a.L.hidden) * 2, ssb_gu, nsm, st);
    if (rc) return rc;
    PolMoeDown<DT, SC> pd{};
    pd.L = a.L;
    pd.experts_layer = a.experts_layer;
    pd.layer = a.layer;
    pd.e0 = a.e0;
    pd.n_experts = a.n_experts;
    pd.n_tok = a.n_tok;
    pd.top_k = a.top_k;
    pd.sel = a.sel;
    pd.h = a.h;
    pd.y = a.y;
    pd.bias_ss = DT != MG_Q8R && a.L.hidden % 4 == 0;
    const int64_t rowbytes = DT == MG_Q8R ? a.L.ffn : a.L.ffn / 2;
    const int64_t nseg = (rowbytes + SW_SEGB - 1) / SW_SEGB;
    const int ks = moe_down_ksplit(a.L, a.down_ksplit);
    MG_REQUIRE(ks == a.down_ksplit_out, MG_ERR_ARG, "moe stream: down K split %d != caller's %d", ks,
               a.down_ksplit_out);
    pd.ks_count = ks;
    pd.kbytes_per_split = ((nseg + ks - 1) / ks) * SW_SEGB;
    return launch_policy<DT>(k_stream<DT, SC, NT, PolMoeDown<DT, SC>>, maps, pd,
                             (size_t)NT * 8 * sw_xs_stride<DT>(a.L.ffn) * 2, ssb_dn, nsm, st);
}

int moe_down_ksplit(const mg_expert_layout &L, int want) { return stream_ksplit(L.dt, L.ffn, want); }

int moe_stream(const MoeStreamArgs &a, cudaStream_t st) {
    MG_REQUIRE(a.n_tok >= 1 && a.n_tok <= 8 && a.n_tok * a.top_k <= SW_MAX_SLOTS && a.n_experts <= 2048 && a.maps,
               MG_ERR_ARG, "moe stream: n_tok %d top_k %d unsupported", a.n_tok, a.top_k);
    const mg_expert_layout &L = a.L;
    if (a.bs && bsmoe_supported(L)) return moe_bs(a, st);
    switch (L.dt) {
    case MG_MXFP4:
        if (L.scale_fmt == MG_SCALE_UE8M0)
            return a.n_tok <= 4 ? moe_stream_t<MG_MXFP4, MG_SCALE_UE8M0, 1>(a, st)
                                : moe_stream_t<MG_MXFP4, MG_SCALE_UE8M0, 2>(a, st);
        return a.n_tok <= 4 ? moe_stream_t<MG_MXFP4, MG_SCALE_F16, 1>(a, st)
                            : moe_stream_t<MG_MXFP4, MG_SCALE_F16, 2>(a, st);
    case MG_Q4G32:
        if (L.scale_fmt == MG_SCALE_UE8M0)
            return a.n_tok <= 4 ? moe_stream_t<MG_Q4G32, MG_SCALE_UE8M0, 1>(a, st)
                                : moe_stream_t<MG_Q4G32, MG_SCALE_UE8M0, 2>(a, st);
        return a.n_tok <= 4 ? moe_stream_t<MG_Q4G32, MG_SCALE_F16, 1>(a, st)
                            : moe_stream_t<MG_Q4G32, MG_SCALE_F16, 2>(a, st);
    case MG_Q8R:
        MG_REQUIRE(L.hidden % 64 == 0 && L.ffn % 64 == 0, MG_ERR_ARG, "moe stream: q8r dims %% 64");
        return a.n_tok <= 4 ? moe_stream_t<MG_Q8R, MG_SCALE_F16, 1>(a, st) : moe_stream_t<MG_Q8R, MG_SCALE_F16, 2>(a, st);
    }
    set_error("moe stream: dtype %d unsupported", L.dt);
    return MG_ERR_ARG;
}

// ----------------------------------------------- MoE combine + RMSNorm
// x[t] += sum_i w[t][i] * sum_ks y[ks][t*k+i]   (rank order, engine/midge.c:544-548)
// then xb[t] = rmsnorm(x[t]) * nw.  One block per token; with one plane, rows
// of up to 4 x 1024 values stay in registers (all of a thread's loads issue
// before any store), otherwise a strided loop.
template <int KS>
__device__ __forceinline__ float cn_value(const CombineNormArgs &a, const float *xi, int64_t c, int64_t H,
                                          int64_t plane, int nk, const int *s_slot, const float *s_w) {
    float v = xi[c];
    if (!a.y) return v;
    // all of this element's plane values first (independent loads), then the
    // reference's order: per slot the planes in order, slots in rank order
    float moe = 0.f;
    if (nk <= 8) {
        float yv[8][KS];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float *yp = a.y + (int64_t)s_slot[i < nk ? i : 0] * H + c;
#pragma unroll
            for (int ks = 0; ks < KS; ks++) yv[i][ks] = i < nk ? yp[ks * plane] : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            float yy = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ks++) yy += yv[i][ks];
            if (i < nk) moe = __fadd_rn(moe, __fmul_rn(s_w[i], yy));
        }
    } else {
        for (int i = 0; i < nk; i++) {
            const float *yp = a.y + (int64_t)s_slot[i] * H + c;
            float yy = 0.f;
            for (int ks = 0; ks < KS; ks++) yy += yp[ks * plane];
            moe = __fadd_rn(moe, __fmul_rn(s_w[i], yy));
        }
    }
    return __fadd_rn(v, moe);
}

template <int KS>  // K-split planes of the expert outputs (compile time so their loads issue together)
__global__ void __launch_bounds__(1024) k_combine_norm(CombineNormArgs a) {
    __shared__ float scratch[32];
    __shared__ float s_w[16];
    __shared__ int s_slot[16], s_k;
    const int t = blockIdx.x;
    const int64_t H = a.hidden;
    float *x = a.x + (int64_t)t * H;
    const float *xi = (a.x_in ? a.x_in : a.x) + (int64_t)t * H;
    if (threadIdx.x < 32) {  // this token's valid routing slots in rank order (ballot prefix)
        const int i = threadIdx.x;
        bool valid = false;
        float wv = 0.f;
        if (a.y && i < a.top_k && i < 16) {
            const int e = a.sel[t * a.top_k + i];
            valid = e >= 0 && e < a.n_experts;
            if (valid) wv = a.w[t * a.top_k + i];
        }
        const unsigned m = __ballot_sync(0xffffffffu, valid);
        if (valid) {
            const int r = __popc(m & ((1u << i) - 1u));
            s_slot[r] = t * a.top_k + i;
            s_w[r] = wv;
        }
        if (i == 0) s_k = __popc(m);
    }
    __syncthreads();
    const int nk = s_k;
    const int64_t plane = a.plane ? a.plane : (int64_t)a.n_tok * a.top_k * H;
    float ss = 0.f;
    constexpr int PER = 4;
    if (KS == 1 && H <= (int64_t)blockDim.x * PER) {  // (more planes would spill registers)
        float v[PER];
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            v[j] = c < H ? cn_value<KS>(a, xi, c, H, plane, nk, s_slot, s_w) : 0.f;
        }
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            if (c < H) {
                if (a.y) x[c] = v[j];
                ss = fmaf(v[j], v[j], ss);
            }
        }
        ss = block_sum(ss, scratch);
        const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
        if (a.xb)
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
                if (c < H) a.xb[(int64_t)t * H + c] = __fmul_rn(__fmul_rn(v[j], inv), a.nw[c]);
            }
        return;
    }
    for (int64_t c = threadIdx.x; c < H; c += blockDim.x) {
        const float v = cn_value<KS>(a, xi, c, H, plane, nk, s_slot, s_w);
        if (a.y) x[c] = v;
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
    if (a.xb)
        for (int64_t c = threadIdx.x; c < H; c += blockDim.x)
            a.xb[(int64_t)t * H + c] = __fmul_rn(__fmul_rn(x[c], inv), a.nw[c]);
}

// The same for one plane of expert outputs (or none), top_k <= MK and hidden
// <= 1024 PER, with one round trip to memory before the norm's reduction:
// every thread loads the token's routing slots and weights, its columns'
// outputs of every slot (valid or not: the buffer holds all n_tok x top_k
// rows), the residual and the norm weight together, then adds the valid
// slots in rank order exactly as k_combine_norm.
template <int MK, int PER>
__global__ void __launch_bounds__(1024) k_combine_norm1(CombineNormArgs a) {
    __shared__ float scratch[32];
    const int t = blockIdx.x;
    const int64_t H = a.hidden;
    float *x = a.x + (int64_t)t * H;
    const float *xi = (a.x_in ? a.x_in : a.x) + (int64_t)t * H;
    const int k = a.top_k;
    int ev[MK];
    float wv[MK];
#pragma unroll
    for (int i = 0; i < MK; i++) {
        const bool s = a.y && i < k;
        ev[i] = s ? a.sel[t * k + i] : -1;
        wv[i] = s ? a.w[t * k + i] : 0.f;
    }
    float v[PER], nw[PER], yv[MK][PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
        v[j] = c < H ? xi[c] : 0.f;
        nw[j] = (a.xb && c < H) ? a.nw[c] : 0.f;
    }
    // the expert outputs come from the MoE grid: after it (a no-op unless
    // this launch is programmatic; the slots, weights and residual above
    // were written by kernels that completed before the MoE grid started)
    pdl_wait();
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
#pragma unroll
        for (int i = 0; i < MK; i++) yv[i][j] = (a.y && i < k && c < H) ? a.y[(int64_t)(t * k + i) * H + c] : 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
        if (a.y) {
            float moe = 0.f;
#pragma unroll
            for (int i = 0; i < MK; i++) {
                float yy = 0.f;
                yy += yv[i][j];
                if (i < k && ev[i] >= 0 && ev[i] < a.n_experts) moe = __fadd_rn(moe, __fmul_rn(wv[i], yy));
            }
            v[j] = __fadd_rn(v[j], moe);
            if (c < H) x[c] = v[j];
        }
        if (c < H) ss = fmaf(v[j], v[j], ss);
    }
    ss = block_sum(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / (float)H + a.eps);
    if (a.xb)
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t c = threadIdx.x + (int64_t)j * blockDim.x;
            if (c < H) a.xb[(int64_t)t * H + c] = __fmul_rn(__fmul_rn(v[j], inv), nw[j]);
        }
}

template <int MK, int PER>
static cudaError_t launch_cn1(const CombineNormArgs &a, cudaStream_t st) {
    return launch_k(a.pdl != 0, k_combine_norm1<MK, PER>, dim3(a.n_tok), dim3(1024), 0, st, a);
}

// false: no instance for this shape (the caller falls back)
template <int MK>
static bool launch_combine_norm1(const CombineNormArgs &a, int per, cudaStream_t st, cudaError_t *e) {
    switch (per) {
    case 1: *e = launch_cn1<MK, 1>(a, st); return true;
    case 2: *e = launch_cn1<MK, 2>(a, st); return true;
    case 3: *e = launch_cn1<MK, 3>(a, st); return true;
    }
    if constexpr (MK <= 4)
        if (per == 4) { *e = launch_cn1<MK, 4>(a, st); return true; }
    return false;
}

int combine_norm(const CombineNormArgs &a, cudaStream_t st) {
    if (a.n_tok <= 0) return MG_OK;
    // one plane of expert outputs (or none): the single-round-trip kernel
    const int per = (int)((a.hidden + 1023) / 1024);
    if ((!a.y || a.ksplit == 1) && a.top_k <= 8 && per <= 4) {
        cudaError_t e = cudaSuccess;
        const bool done =
            a.top_k <= 4 || !a.y ? launch_combine_norm1<4>(a, per, st, &e) : launch_combine_norm1<8>(a, per, st, &e);
        if (done) {
            MG_CUDA(e);
            return MG_OK;
        }
    }
    switch (a.y ? a.ksplit : 1) {
    case 1: k_combine_norm<1><<<a.n_tok, 1024, 0, st>>>(a); break;
    case 2: k_combine_norm<2><<<a.n_tok, 1024, 0, st>>>(a); break;
    case 3: k_combine_norm<3><<<a.n_tok, 1024, 0, st>>>(a); break;
    case 4: k_combine_norm<4><<<a.n_tok, 1024, 0, st>>>(a); break;
    default: set_error("combine_norm: %d K-split planes unsupported", a.ksplit); return MG_ERR_ARG;
    }
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// sum K-split partial planes: out[t][r] (=|+=) sum_ks part[ks][t][r]
__global__ void k_sum_parts(const float *__restrict__ part, int ks, int64_t plane, int n_tok, int64_t rows, int64_t ldp,
                            float *out, int64_t ldo, int accumulate) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_tok * rows; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / rows, r = i - t * rows;
        float v = 0.f;
        for (int k = 0; k < ks; k++) v += part[(int64_t)k * plane + t * ldp + r];
        float *o = out + t * ldo + r;
        *o = accumulate ? *o + v : v;
    }
}

int sum_parts(const float *part, int ks, int64_t plane, int n_tok, int64_t rows, int64_t ldp, float *out, int64_t ldo,
              int accumulate, cudaStream_t st) {
    const int64_t n = (int64_t)n_tok * rows;
    int grid = ceil_div(n, 256);
    if (grid > 1184) grid = 1184;
    k_sum_parts<<<grid, 256, 0, st>>>(part, ks, plane, n_tok, rows, ldp, out, ldo, accumulate);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

}  // namespace mg

// mg_stream.cuh -- warp-specialized streamed dequant-GEMV for decode.
//
// One CTA = 8 consumer warps + 1 producer warp.  The producer streams weight
// rows into a ring of shared-memory stages with cp.async.bulk (one bulk copy
// per row segment, completion counted on an mbarrier); the consumers decode
// and multiply out of shared memory on the tensor cores (mma.sync, f16 hi/lo
// activations, f32 accumulation) and hand each stage back through a second
// mbarrier.  Memory parallelism is therefore set by the ring depth, not by
// registers.
//
// A stage holds 128 "MMA rows" (16 per consumer warp) x up to SEGB bytes of
// each row.  Work is a list of units; a unit is a tile of MMA rows times a
// range of each row's bytes (a K split), streamed as consecutive segments.
// Each consumer warp accumulates its own 16 rows over the unit's segments and
// runs the policy's epilogue itself: no cross-warp reduction.
//
// Every wait is bounded; on timeout a kernel records an error code and stops.
#pragma once
#include "mg_common.cuh"
#include "mg_gemv.cuh"

namespace mg {

constexpr int SW_CONS = 8;                    // consumer warps
constexpr int SW_THREADS = (SW_CONS + 1) * 32;
constexpr int SW_ROWS = SW_CONS * 16;         // MMA rows per stage
constexpr int SW_MAX_STAGES = 6;
constexpr int SW_ERR_TIMEOUT = 1;

template <int DT>
struct SwGeom {
    static constexpr int CB = DT == MG_Q8R ? 64 : 16;    // bytes of one chunk of one row
    static constexpr int COLS_PER_CHUNK = DT == MG_Q8R ? 64 : 32;
    static constexpr int SEGB = 256;                      // bytes per row per stage
    // smem row stride: conflict-free fragment loads (LDS.32 / LDS.128)
    static constexpr int STRIDE = DT == MG_Q8R ? SEGB + 64 : SEGB + 16;
    static constexpr int STAGE_BYTES = SW_ROWS * STRIDE;
};

// Shared-memory bookkeeping common to all streamed kernels.
struct SwShared {
    uint64_t full[SW_MAX_STAGES];
    uint64_t empty[SW_MAX_STAGES];
};

// -------------------------------------------------------------- producer
// Policy interface (device):
//   int64_t units() const
//   void unit(int64_t u, UnitInfo &ui) const  -> byte range [b0, b1) of each row
//   const uint8_t *row_ptr(const UnitInfo &, int mma_row) const  (null = no row)
struct UnitInfo {
    int64_t tile;
    int ks;
    int64_t b0, b1;  // byte range of every row handled by this unit
    int aux;          // policy-defined (e.g. expert index)
};

template <int DT, class P>
__device__ void sw_producer(const P &pol, int64_t u0, int64_t u1, uint8_t *ring, int nstages, SwShared *sh,
                            int *err) {
    using G = SwGeom<DT>;
    const int lane = threadIdx.x & 31;
    int64_t it = 0;
    for (int64_t u = u0; u < u1; u++) {
        UnitInfo ui;
        pol.unit(u, ui);
        const uint8_t *rp[SW_ROWS / 32];
        int nvalid = 0;
#pragma unroll
        for (int j = 0; j < SW_ROWS / 32; j++) {
            rp[j] = pol.row_ptr(ui, lane + 32 * j);
            nvalid += __popc(__ballot_sync(0xffffffffu, rp[j] != nullptr));
        }
        for (int64_t b = ui.b0; b < ui.b1; b += G::SEGB, it++) {
            const int s = (int)(it % nstages);
            const uint32_t bytes = (uint32_t)min((int64_t)G::SEGB, ui.b1 - b);
            if (it >= nstages) {  // wait until the consumers released this stage
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&sh->empty[s], (uint32_t)(((it / nstages) - 1) & 1));
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) atomicExch(err, SW_ERR_TIMEOUT);
                    return;
                }
            }
            if (lane == 0) mbar_arrive_expect_tx(&sh->full[s], bytes * (uint32_t)nvalid);
            __syncwarp();
            uint8_t *st = ring + (size_t)s * G::STAGE_BYTES;
#pragma unroll
            for (int j = 0; j < SW_ROWS / 32; j++)
                if (rp[j]) bulk_g2s(st + (size_t)(lane + 32 * j) * G::STRIDE, rp[j] + b, bytes, &sh->full[s]);
        }
    }
}

// -------------------------------------------------------------- consumer
// One warp's share of one segment: 16 MMA rows (stage rows 16w..16w+15),
// `nch` chunks starting at row byte `b` (column col0 of the activations).
template <int DT, int SC, int NT, class P>
__device__ __forceinline__ void sw_consume_seg(const P &pol, const UnitInfo &ui, const uint8_t *st, int w, int64_t b,
                                               int nch, const __half *xs, int xs_stride, int nt_active,
                                               float acc[NT][4]) {
    using G = SwGeom<DT>;
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const uint8_t *ra = st + (size_t)(16 * w + g) * G::STRIDE;
    const uint8_t *rb = ra + (size_t)8 * G::STRIDE;
    const int64_t col0 = b / G::CB * G::COLS_PER_CHUNK;
    if constexpr (DT == MG_Q8R) {
#pragma unroll 2
        for (int c = 0; c < nch; c++) {
            uint4 wa = *reinterpret_cast<const uint4 *>(ra + c * 64 + 16 * t);
            uint4 wb = *reinterpret_cast<const uint4 *>(rb + c * 64 + 16 * t);
            uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w}, wbv[4] = {wb.x, wb.y, wb.z, wb.w};
            uint32_t fa[4][4];
#pragma unroll
            for (int s = 0; s < 4; s++) {
                s8x4_to_h2(wav[s], fa[s][0], fa[s][2]);
                s8x4_to_h2(wbv[s], fa[s][1], fa[s][3]);
            }
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                if (nt >= nt_active) break;
                const __half *xp = xs + (nt * 8 + g) * xs_stride + col0 + c * 64 + 16 * t;
                uint4 x0 = *reinterpret_cast<const uint4 *>(xp);
                uint4 x1 = *reinterpret_cast<const uint4 *>(xp + 8);
                uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int s = 0; s < 4; s++) mma_16816(acc[nt], fa[s], bx[2 * s], bx[2 * s + 1]);
            }
        }
    } else {
        const int64_t gchunk0 = b / G::CB;  // group index of the segment's first chunk
#pragma unroll 2
        for (int c = 0; c < nch; c++) {
            const uint32_t wa = lds32(ra + c * 16 + 4 * t), wb = lds32(rb + c * 16 + 4 * t);
            const float sa = pol.scale(ui, g, gchunk0 + c), sb = pol.scale(ui, g + 8, gchunk0 + c);
            uint32_t fa[4], fb[4];
            if (DT == MG_MXFP4) {
                e2m1x8_to_h2(wa, fa);
                e2m1x8_to_h2(wb, fb);
            } else {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    fa[i] = u4pair_minus8_h2(wa >> (4 * i));
                    fb[i] = u4pair_minus8_h2(wb >> (4 * i));
                }
            }
            const uint32_t a0[4] = {fa[0], fb[0], fa[1], fb[1]};
            const uint32_t a1[4] = {fa[2], fb[2], fa[3], fb[3]};
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                if (nt >= nt_active) break;
                const uint4 bx =
                    *reinterpret_cast<const uint4 *>(xs + (nt * 8 + g) * xs_stride + col0 + c * 32 + 8 * t);
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                mma_16816(d, a0, bx.x, bx.y);
                mma_16816(d, a1, bx.z, bx.w);
                acc[nt][0] = fmaf(sa, d[0], acc[nt][0]);
                acc[nt][1] = fmaf(sa, d[1], acc[nt][1]);
                acc[nt][2] = fmaf(sb, d[2], acc[nt][2]);
                acc[nt][3] = fmaf(sb, d[3], acc[nt][3]);
            }
        }
    }
}

// Consumer warps: per unit, accumulate its segments, then the policy epilogue.
// Policy:  void stage(int64_t u, ...) is done outside; here:
//   bool restage(int64_t u)  -> the activations must be re-staged before u
//   void stage_x(int64_t u, __half *xs, int xs_stride)   (consumer threads, synced by caller)
//   void epilogue(const UnitInfo&, int warp, const float acc[NT][4])
template <int DT, int SC, int NT, class P>
__device__ void sw_consumers(P &pol, int64_t u0, int64_t u1, uint8_t *ring, int nstages, SwShared *sh, __half *xs,
                             int xs_stride, int *err) {
    using G = SwGeom<DT>;
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t it = 0;
    for (int64_t u = u0; u < u1; u++) {
        if (pol.restage(u, u0)) {
            named_bar_sync(1, SW_CONS * 32);  // everyone is done with the old activations
            pol.stage_x(u, xs, xs_stride);
            named_bar_sync(1, SW_CONS * 32);
        }
        UnitInfo ui;
        pol.unit(u, ui);
        const int nt_active = pol.nt_active(ui);
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
        const bool live = pol.warp_live(ui, w);
        for (int64_t b = ui.b0; b < ui.b1; b += G::SEGB, it++) {
            const int s = (int)(it % nstages);
            const int64_t bytes = min((int64_t)G::SEGB, ui.b1 - b);
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&sh->full[s], (uint32_t)((it / nstages) & 1));
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) atomicExch(err, SW_ERR_TIMEOUT);
                return;
            }
            if (live)
                sw_consume_seg<DT, SC, NT>(pol, ui, ring + (size_t)s * G::STAGE_BYTES, w, b, (int)(bytes / G::CB), xs,
                                           xs_stride, nt_active, acc);
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->empty[s]);
        }
        if (live) pol.template epilogue<NT>(ui, w, acc);
    }
}

// The kernel shell: barrier setup, block's unit range, role split.
template <int DT, int SC, int NT, class P>
__global__ void __launch_bounds__(SW_THREADS, 1) k_stream(P pol, int nstages, int *err) {
    extern __shared__ __align__(128) uint8_t sw_smem[];
    using G = SwGeom<DT>;
    SwShared *sh = reinterpret_cast<SwShared *>(sw_smem);
    uint8_t *ring = sw_smem + 128;
    __half *xs = reinterpret_cast<__half *>(ring + (size_t)nstages * G::STAGE_BYTES);
    const int xs_stride = pol.xs_stride();
    const int64_t nunits = pol.units();
    const int64_t per = (nunits + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = (int64_t)blockIdx.x * per, u1 = min(nunits, u0 + per);
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstages; s++) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], SW_CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (u0 >= u1) return;
    const int w = threadIdx.x >> 5;
    if (w == SW_CONS) {
        sw_producer<DT>(pol, u0, u1, ring, nstages, sh, err);
    } else {
        pol.stage_x(u0, xs, xs_stride);
        named_bar_sync(1, SW_CONS * 32);
        sw_consumers<DT, SC, NT>(pol, u0, u1, ring, nstages, sh, xs, xs_stride, err);
    }
}

// ------------------------------------------------------------- policies
// Plain GEMV over up to 3 row-concatenated matrices sharing cols and the
// activations; K split KS ways.  Unit = (tile of 128 rows of one matrix, ks).
// Output: KS == 1 -> y = W x (+bias) (store or accumulate); KS > 1 -> part[ks]
// holds the partial sums (bias added by ks 0) for a later reduction.
struct GemvMat {
    const uint8_t *w, *sc;
    const float *bias;
    int64_t rows;
    float *y;      // [n_tok x ldy] (KS == 1) or partials [KS x n_tok x ldy]
    int64_t ldy;
    int64_t tile0;  // first tile index of this matrix
};

template <int DT, int SC>
struct PolGemv {
    GemvMat m[3];
    int nmat;
    int cols;
    int ks_count;
    int64_t kbytes_per_split;  // row bytes per K split (multiple of SEGB)
    int64_t ntiles;
    const float *x;
    int64_t ldx;
    int n_tok;
    int accumulate;
    int64_t part_stride;  // floats between K-split partial planes

    __device__ int64_t rowbytes() const { return DT == MG_Q8R ? cols : cols / 2; }
    __device__ int xs_stride() const { return cols + XS_PAD; }
    __device__ int64_t units() const { return ntiles * ks_count; }
    __device__ int mat_of(int64_t tile) const {
        int k = 0;
        while (k + 1 < nmat && tile >= m[k + 1].tile0) k++;
        return k;
    }
    __device__ void unit(int64_t u, UnitInfo &ui) const {
        ui.tile = u / ks_count;
        ui.ks = (int)(u % ks_count);
        ui.b0 = (int64_t)ui.ks * kbytes_per_split;
        ui.b1 = min(rowbytes(), ui.b0 + kbytes_per_split);
        ui.aux = mat_of(ui.tile);
    }
    __device__ int64_t row_of(const UnitInfo &ui, int r) const { return (ui.tile - m[ui.aux].tile0) * SW_ROWS + r; }
    __device__ const uint8_t *row_ptr(const UnitInfo &ui, int r) const {
        const int64_t row = row_of(ui, r);
        return row < m[ui.aux].rows ? m[ui.aux].w + row * rowbytes() : nullptr;
    }
    __device__ bool warp_live(const UnitInfo &ui, int w) const { return row_of(ui, 16 * w) < m[ui.aux].rows; }
    __device__ float scale(const UnitInfo &ui, int r16, int64_t grp) const {
        // r16 = MMA row within this warp's 16 (caller passes g or g+8)
        const int w = threadIdx.x >> 5;
        const int64_t row = row_of(ui, 16 * w + r16);
        if (row >= m[ui.aux].rows) return 0.f;
        const int64_t gpr = cols / 32;
        if (SC == MG_SCALE_UE8M0) return ue8m0_to_f32(__ldg(m[ui.aux].sc + row * gpr + grp));
        return h2f(__ldg(reinterpret_cast<const uint16_t *>(m[ui.aux].sc) + row * gpr + grp));
    }
    __device__ int nt_active(const UnitInfo &) const { return (n_tok + 3) >> 2; }
    __device__ bool restage(int64_t, int64_t) const { return false; }
    __device__ void stage_x(int64_t, __half *xs, int xs_stride) const {
        stage_x_n<DT>(x, ldx, n_tok, cols, xs, xs_stride, threadIdx.x, SW_CONS * 32);
    }
    template <int NT>
    __device__ void epilogue(const UnitInfo &ui, int w, const float acc[NT][4]) const {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        const GemvMat &mm = m[ui.aux];
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int64_t row = row_of(ui, 16 * w + g + 8 * half);
            if (row >= mm.rows) continue;
            float rs = 1.f;
            if (DT == MG_Q8R) rs = reinterpret_cast<const float *>(mm.sc)[row];
            const float bias = (mm.bias && ui.ks == 0) ? mm.bias[row] : 0.f;
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int tok = nt * 4 + t;
                if (tok >= n_tok) continue;
                float v = acc[nt][2 * half] + acc[nt][2 * half + 1];
                if (DT == MG_Q8R) v *= rs;
                v += bias;
                if (ks_count == 1) {
                    float *yp = mm.y + (int64_t)tok * mm.ldy + row;
                    *yp = accumulate ? *yp + v : v;
                } else {
                    mm.y[(int64_t)ui.ks * part_stride + (int64_t)tok * mm.ldy + row] = v;
                }
            }
        }
    }
};

}  // namespace mg

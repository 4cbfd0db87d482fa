// mg_gemv.cuh -- dequant-GEMV tile machinery shared by the decode kernels.
//
// A weight row-tile of 16 rows is multiplied by up to 16 activation vectors
// on the tensor cores (mma.sync m16n8k16, f16 inputs, f32 accumulation):
//   * weights are decoded in registers to f16 exactly (e2m1 via the sm_100
//     cvt.f16x2.e2m1x2 instruction, int8 and biased int4 via exponent tricks);
//   * every fp32 activation is split into an f16 pair hi + lo (~22 significant
//     bits), the two halves occupying adjacent MMA columns, so the product is
//     the fp32 GEMV to ~1e-6 relative;
//   * 4-bit group scales (one per 32 columns) are applied in fp32 to a fresh
//     per-group accumulator, so the scale never passes through f16;
//   * q8r row scales are applied after the full sum (as engine/mkern.h:116).
// MMA K order is free, so each thread's k-slots are chosen to be the columns
// it loaded; the activation tile in shared memory is laid out to match.
#pragma once
#include "mg_common.cuh"

namespace mg {

constexpr int GEMV_THREADS = 256;  // 8 warps per block split K
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int XS_PAD = 8;          // halves of padding per staged column (16 B)

// Column permutation applied when staging activations for q4g32: the biased
// int4 decode pairs nibbles (i, i+4) of a 32-bit word.
__device__ __forceinline__ int q4_stage_perm(int p) {  // position p in an 8-col block -> source column
    return ((p & 1) << 2) | (p >> 1);
}

// Stage n_tok fp32 activation rows (row t at x + t*ldx) into xs as f16 hi/lo
// columns: column 2t = hi, 2t+1 = lo.  Columns of tokens >= n_tok are left
// as they are: an MMA output column depends only on its own B column, and
// those outputs are never read.  Vector path: 8 columns per step (two 16-byte
// loads, two 16-byte stores); needs x 16-byte aligned and ldx % 4 == 0.
template <int DT>
__device__ __forceinline__ void stage_x_n(const float *x, int64_t ldx, int n_tok, int cols, __half *xs,
                                          int xs_stride, int tid, int nthr) {
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((ldx & 3) == 0);
    if (vec) {
        const int q = cols >> 3;
        const int total = n_tok * q;
#pragma unroll 2
        for (int i = tid; i < total; i += nthr) {
            const int t = i / q, c8 = (i - t * q) << 3;
            const float4 *src = reinterpret_cast<const float4 *>(x + (int64_t)t * ldx + c8);
            float4 a = __ldg(src), b = __ldg(src + 1);
            float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
            __half hi[8], lo[8];
#pragma unroll
            for (int p = 0; p < 8; p++) {
                const int srcc = DT == MG_Q4G32 ? q4_stage_perm(p) : p;
                split_f16(v[srcc], hi[p], lo[p]);
            }
            *reinterpret_cast<uint4 *>(xs + (2 * t) * xs_stride + c8) = *reinterpret_cast<uint4 *>(hi);
            *reinterpret_cast<uint4 *>(xs + (2 * t + 1) * xs_stride + c8) = *reinterpret_cast<uint4 *>(lo);
        }
    } else {
        const int total = n_tok * cols;
        for (int i = tid; i < total; i += nthr) {
            const int t = i / cols, c = i - t * cols;
            const int src = DT == MG_Q4G32 ? ((c & ~7) | q4_stage_perm(c & 7)) : c;
            __half hi, lo;
            split_f16(x[(int64_t)t * ldx + src], hi, lo);
            xs[(2 * t) * xs_stride + c] = hi;
            xs[(2 * t + 1) * xs_stride + c] = lo;
        }
    }
}

template <int DT>
__device__ __forceinline__ void stage_x(const float *x, int64_t ldx, int n_tok, int cols, __half *xs,
                                        int xs_stride) {
    stage_x_n<DT>(x, ldx, n_tok, cols, xs, xs_stride, threadIdx.x, blockDim.x);
}

__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Ask L2 for this warp's slice of a row tile (rows row0..row0+15 of w, byte
// range of chunks [c0, c1)) and, from warp 0, the tile's scales, so that the
// weight stream overlaps the activation staging.  Only in-bounds, 16-byte
// aligned ranges are requested.
template <int DT, int SC>
__device__ __forceinline__ void prefetch_tile(const uint8_t *w, const uint8_t *sc, int64_t row0, int64_t rows,
                                              int cols, int c0, int c1) {
    const int lane = threadIdx.x & 31;
    constexpr int CB = DT == MG_Q8R ? 64 : 16;  // bytes per row per chunk
    const int64_t rowbytes = DT == MG_Q8R ? cols : cols / 2;
    if (lane < 16 && row0 + lane < rows && c1 > c0)
        prefetch_l2_bulk(w + (row0 + lane) * rowbytes + (int64_t)c0 * CB, (uint32_t)((c1 - c0) * CB));
    if (DT != MG_Q8R && (threadIdx.x >> 5) == 0 && lane == 16) {
        const int64_t sb = SC == MG_SCALE_UE8M0 ? cols / 32 : cols / 16;  // scale bytes per row
        int64_t nr = rows - row0 < 16 ? rows - row0 : 16;
        uint32_t bytes = (uint32_t)((nr * sb) & ~(int64_t)15);
        const uint8_t *sp = sc + row0 * sb;
        if (bytes && ((reinterpret_cast<uintptr_t>(sp) & 15) == 0)) prefetch_l2_bulk(sp, bytes);
    }
}

// Per-thread partial sums of one warp over chunk range [c0, c1) for MT row
// tiles (rows row0[mt] + 0..15 of matrix w[mt]) and NT n-tiles.
// 4-bit: chunk = one 32-column group; q8r: chunk = 64 columns.
// acc[mt][nt][0..3] follow the m16n8 accumulator layout.  The loop is
// software-pipelined: the loads of batch b+1 (U chunks) are issued before the
// tensor-core work of batch b.
template <int DT, int SC, int MT, int NT>
struct GemvTile {
    static constexpr int CHUNK = (DT == MG_Q8R) ? 64 : 32;
    static constexpr int U = (DT == MG_Q8R) ? 2 : 4;  // chunks per batch
    static constexpr int WW = (DT == MG_Q8R) ? 4 : 1; // 32-bit words per row per chunk per thread

    struct Batch {
        uint32_t wa[U][MT][WW], wb[U][MT][WW];
        float sa[U][MT], sb[U][MT];
    };

    __device__ __forceinline__ static void load(Batch &bt, const uint8_t *const w[MT], const uint8_t *const sc[MT],
                                                const int64_t ra[MT], const int64_t rb[MT], const bool va[MT],
                                                const bool vb[MT], int64_t rowbytes, int gpr, int cb, int c1, int t) {
#pragma unroll
        for (int u = 0; u < U; u++)
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const int c = cb + u;
                const bool oka = c < c1 && va[m], okb = c < c1 && vb[m];
                if constexpr (DT == MG_Q8R) {
                    const uint8_t *pa = w[m] + ra[m] * rowbytes + (int64_t)c * 64 + 16 * t;
                    const uint8_t *pb = w[m] + rb[m] * rowbytes + (int64_t)c * 64 + 16 * t;
                    uint4 x = oka ? ldg_nc_u128(pa) : make_uint4(0, 0, 0, 0);
                    uint4 y = okb ? ldg_nc_u128(pb) : make_uint4(0, 0, 0, 0);
                    bt.wa[u][m][0] = x.x; bt.wa[u][m][1] = x.y; bt.wa[u][m][2] = x.z; bt.wa[u][m][3] = x.w;
                    bt.wb[u][m][0] = y.x; bt.wb[u][m][1] = y.y; bt.wb[u][m][2] = y.z; bt.wb[u][m][3] = y.w;
                } else {
                    const uint8_t *pa = w[m] + ra[m] * rowbytes + (int64_t)c * 16 + 4 * t;
                    const uint8_t *pb = w[m] + rb[m] * rowbytes + (int64_t)c * 16 + 4 * t;
                    bt.wa[u][m][0] = oka ? ldg_u32_l1(pa) : 0u;
                    bt.wb[u][m][0] = okb ? ldg_u32_l1(pb) : 0u;
                    if (SC == MG_SCALE_UE8M0) {
                        bt.sa[u][m] = oka ? ue8m0_to_f32(__ldg(sc[m] + ra[m] * gpr + c)) : 0.f;
                        bt.sb[u][m] = okb ? ue8m0_to_f32(__ldg(sc[m] + rb[m] * gpr + c)) : 0.f;
                    } else {
                        const uint16_t *s16 = reinterpret_cast<const uint16_t *>(sc[m]);
                        bt.sa[u][m] = oka ? h2f(__ldg(s16 + ra[m] * gpr + c)) : 0.f;
                        bt.sb[u][m] = okb ? h2f(__ldg(s16 + rb[m] * gpr + c)) : 0.f;
                    }
                }
            }
    }

    __device__ __forceinline__ static void compute(const Batch &bt, int cb, int c1, const __half *xs, int xs_stride,
                                                   int nt_active, int g, int t, float acc[MT][NT][4]) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int c = cb + u;
            if (c >= c1) break;
            if constexpr (DT == MG_Q8R) {
                uint32_t fa[MT][4][4];  // [m][k-step][a-register]
#pragma unroll
                for (int m = 0; m < MT; m++)
#pragma unroll
                    for (int s = 0; s < 4; s++) {
                        s8x4_to_h2(bt.wa[u][m][s], fa[m][s][0], fa[m][s][2]);
                        s8x4_to_h2(bt.wb[u][m][s], fa[m][s][1], fa[m][s][3]);
                    }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    if (nt >= nt_active) break;
                    const __half *xp = xs + (nt * 8 + g) * xs_stride + c * 64 + 16 * t;
                    uint4 x0 = *reinterpret_cast<const uint4 *>(xp);
                    uint4 x1 = *reinterpret_cast<const uint4 *>(xp + 8);
                    uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int m = 0; m < MT; m++)
#pragma unroll
                        for (int s = 0; s < 4; s++) mma_16816(acc[m][nt], fa[m][s], bx[2 * s], bx[2 * s + 1]);
                }
            } else {
                uint32_t fa[MT][4], fb[MT][4];
#pragma unroll
                for (int m = 0; m < MT; m++) {
                    if (DT == MG_MXFP4) {
                        e2m1x8_to_h2(bt.wa[u][m][0], fa[m]);
                        e2m1x8_to_h2(bt.wb[u][m][0], fb[m]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            fa[m][i] = u4pair_minus8_h2(bt.wa[u][m][0] >> (4 * i));
                            fb[m][i] = u4pair_minus8_h2(bt.wb[u][m][0] >> (4 * i));
                        }
                    }
                }
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    if (nt >= nt_active) break;
                    const __half *xp = xs + (nt * 8 + g) * xs_stride + c * 32 + 8 * t;
                    uint4 bx = *reinterpret_cast<const uint4 *>(xp);
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        float d[4] = {0.f, 0.f, 0.f, 0.f};
                        uint32_t a0[4] = {fa[m][0], fb[m][0], fa[m][1], fb[m][1]};
                        uint32_t a1[4] = {fa[m][2], fb[m][2], fa[m][3], fb[m][3]};
                        mma_16816(d, a0, bx.x, bx.y);
                        mma_16816(d, a1, bx.z, bx.w);
                        acc[m][nt][0] = fmaf(bt.sa[u][m], d[0], acc[m][nt][0]);
                        acc[m][nt][1] = fmaf(bt.sa[u][m], d[1], acc[m][nt][1]);
                        acc[m][nt][2] = fmaf(bt.sb[u][m], d[2], acc[m][nt][2]);
                        acc[m][nt][3] = fmaf(bt.sb[u][m], d[3], acc[m][nt][3]);
                    }
                }
            }
        }
    }

    __device__ __forceinline__ static void run(const uint8_t *const w[MT], const uint8_t *const sc[MT],
                                               const int64_t row0[MT], int64_t rows, int cols, int c0, int c1,
                                               const __half *xs, int xs_stride, int nt_active, float acc[MT][NT][4]) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        const int64_t rowbytes = (DT == MG_Q8R) ? cols : cols / 2;
        const int gpr = cols / 32;
        int64_t ra[MT], rb[MT];
        bool va[MT], vb[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) {
            ra[m] = row0[m] + g;
            rb[m] = ra[m] + 8;
            va[m] = ra[m] < rows;
            vb[m] = rb[m] < rows;
        }
        if (c0 >= c1) return;
        Batch cur, nxt;
        load(cur, w, sc, ra, rb, va, vb, rowbytes, gpr, c0, c1, t);
        for (int cb = c0; cb < c1; cb += U) {
            const bool more = cb + U < c1;
            if (more) load(nxt, w, sc, ra, rb, va, vb, rowbytes, gpr, cb + U, c1, t);
            compute(cur, cb, c1, xs, xs_stride, nt_active, g, t, acc);
            if (more) cur = nxt;
        }
    }
};

// Reduce the 8 warps' partial accumulators of a block through shared memory.
// After the call, red holds per (mt, nt, lane, i) the sum over warps, and the
// caller reads outputs with gemv_out().
template <int MT, int NT>
__device__ __forceinline__ void gemv_block_reduce(float acc[MT][NT][4], float *red) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    constexpr int PER_WARP = MT * NT * 32 * 4;
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) red[wid * PER_WARP + ((m * NT + nt) * 4 + i) * 32 + lane] = acc[m][nt][i];
    __syncthreads();
    for (int j = threadIdx.x; j < PER_WARP; j += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int wv = 0; wv < GEMV_WARPS; wv++) s += red[wv * PER_WARP + j];
        red[j] = s;
    }
    __syncthreads();
}

// Output (row r16 in 0..15 of row tile mt, token tok) from a reduced block:
// hi column + lo column.
template <int NT>
__device__ __forceinline__ float gemv_out(const float *red, int mt, int r16, int tok) {
    int nt = tok >> 2, t = tok & 3;
    int g = r16 & 7, hiRow = r16 >> 3;
    int lane = g * 4 + t;
    int i0 = hiRow * 2;
    return red[((mt * NT + nt) * 4 + i0) * 32 + lane] + red[((mt * NT + nt) * 4 + i0 + 1) * 32 + lane];
}

// Split [0, nchunks) among the block's warps.
__device__ __forceinline__ void warp_chunk_range(int nchunks, int &c0, int &c1) {
    int wid = threadIdx.x >> 5;
    c0 = (int)((int64_t)nchunks * wid / GEMV_WARPS);
    c1 = (int)((int64_t)nchunks * (wid + 1) / GEMV_WARPS);
}

}  // namespace mg

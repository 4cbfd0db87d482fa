// mg_gemm.cu -- expert-major grouped GEMM for prefill on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in TMEM, activations by TMA).
//
// D[M x N] = W[M x K] . X[N x K]^T per expert, M = weight rows (output
// features), N = the tokens routed to the expert (expert-major rows), K-major
// operands in 128-byte-swizzled shared memory:
//   * W (MXFP4 / q8r) is decoded by four converter warps straight into the
//     UMMA layout as f16, exactly: e2m1 values times 2^(k - k0) with a
//     per-matrix rebase k0 (so every group scale folds into f16 without
//     rounding), int8 values as they are; k0 (or the q8r row scale) is
//     restored in fp32 in the epilogue;
//   * X is an fp32 activation split into f16 hi + lo halves (~22 bits); the
//     two halves are two MMAs into the same accumulator;
//   * modes: GATEUP (gate and up tiles in two TMEM accumulators, the clamped /
//     plain SwiGLU in the epilogue, h written back as f16 hi/lo for the down
//     GEMM), DOWN (y = W h + bias per expert-major row), DENSE (one matrix over
//     all tokens, y = W x + bias, stored or accumulated: the trunk in prefill).
// Warp roles: warp 0 issues TMA for X, warp 1 issues the MMAs (one thread) and
// owns TMEM, warps 2-5 convert W and run the epilogue.  All waits are bounded.
#include <cuda.h>

#include "mg_gemm.h"
#include "mg_kernels.h"
#include "mg_tc.cuh"

namespace mg {

constexpr int XG_M = 128, XG_N = 128, XG_K = 64;
constexpr int XG_THREADS = 192;
constexpr int XG_TILE_BYTES = XG_M * XG_K * 2;  // 16 KB: 128 rows x 128 B
constexpr int XG_ERR = 2;

template <int MODE>
struct XgCfg {
    static constexpr int NA = MODE == XG_GATEUP ? 2 : 1;              // A tiles per stage
    static constexpr int STAGE = (NA + 2) * XG_TILE_BYTES;           // + B hi + B lo
    static constexpr int STAGES = MODE == XG_GATEUP ? 3 : 4;
    static constexpr int TMEM_COLS = NA * XG_N;                       // 256 or 128
};

// Raw bytes of one row's slice of a 128 x 64 weight tile, loaded one k-tile
// ahead of its conversion so the global-load latency overlaps the previous
// tile's conversion and MMAs.
template <int DT>
struct XgRaw {
    static constexpr int NW = DT == MG_Q8R ? 4 : 2;  // 16-byte words: 64 int8 or 64 e2m1
    uint4 w[NW];
    uint32_t s[2];  // ue8m0 codes of the two 32-column groups (MXFP4)
};

template <int DT>
__device__ __forceinline__ void xg_load(XgRaw<DT> &r, const uint8_t *w, const uint8_t *sc, int64_t rows, int64_t cols,
                                        int64_t row, int kt) {
    if (row < rows) {
        if constexpr (DT == MG_Q8R) {
            const uint4 *src = reinterpret_cast<const uint4 *>(w + row * cols + (int64_t)kt * 64);
#pragma unroll
            for (int q = 0; q < 4; q++) r.w[q] = __ldg(src + q);
        } else {
            const uint4 *src = reinterpret_cast<const uint4 *>(w + row * (cols / 2) + (int64_t)kt * 32);
            r.w[0] = __ldg(src);
            r.w[1] = __ldg(src + 1);
            const int64_t gpr = cols / 32;
            r.s[0] = sc[row * gpr + (int64_t)kt * 2];
            r.s[1] = sc[row * gpr + (int64_t)kt * 2 + 1];
        }
    } else {
#pragma unroll
        for (int q = 0; q < XgRaw<DT>::NW; q++) r.w[q] = make_uint4(0, 0, 0, 0);
        r.s[0] = r.s[1] = 0;
    }
}

// Write one row (thread r of 128) of the tile as f16 at `dst` in the
// 128B-swizzled K-major layout: e2m1 values times 2^(code - 127 - rebase),
// int8 values as they are.
template <int DT>
__device__ __forceinline__ void xg_store(uint8_t *dst, const XgRaw<DT> &raw, int rebase, int r) {
    uint8_t *drow = dst + r * 128;
    const int sw = r & 7;
    uint32_t v[32];  // 64 f16 = 32 words
    if constexpr (DT == MG_Q8R) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            s8x4_to_h2(raw.w[q].x, v[8 * q + 0], v[8 * q + 1]);
            s8x4_to_h2(raw.w[q].y, v[8 * q + 2], v[8 * q + 3]);
            s8x4_to_h2(raw.w[q].z, v[8 * q + 4], v[8 * q + 5]);
            s8x4_to_h2(raw.w[q].w, v[8 * q + 6], v[8 * q + 7]);
        }
    } else {
#pragma unroll
        for (int gi = 0; gi < 2; gi++) {  // two 32-column groups per tile
            const uint32_t u = raw.s[gi];
            const uint32_t f = u ? pow2_h2((int)u - 127 - rebase) : 0u;
            const uint32_t words[4] = {raw.w[gi].x, raw.w[gi].y, raw.w[gi].z, raw.w[gi].w};
#pragma unroll
            for (int wd = 0; wd < 4; wd++) {
                uint32_t o[4];
                e2m1x8_to_h2(words[wd], o);
#pragma unroll
                for (int i = 0; i < 4; i++) v[16 * gi + 4 * wd + i] = hmul2_u32(o[i], f);
            }
        }
    }
#pragma unroll
    for (int c = 0; c < 8; c++)  // 16-byte chunk c of the 128-byte row, swizzled
        *reinterpret_cast<uint4 *>(drow + ((c ^ sw) << 4)) = make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

template <int MODE, int DT>
__global__ void __launch_bounds__(XG_THREADS, 1)
    k_xgemm(const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_lo, XgArgs a) {
    using C = XgCfg<MODE>;
    extern __shared__ __align__(1024) uint8_t xsm[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(xsm) + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t full_a[C::STAGES], full_b[C::STAGES], empty[C::STAGES], acc_full;
    __shared__ uint32_t tmem_base;
    __shared__ XgTile tile;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (MODE == XG_DENSE) {
        if (threadIdx.x == 0) tile = XgTile{0, (int)blockIdx.y * XG_N, min(XG_N, a.n_rows - (int)blockIdx.y * XG_N)};
        __syncthreads();
        if (tile.nrows <= 0) return;
    } else {
        if (threadIdx.x == 0) tile = a.tiles[blockIdx.y];
        __syncthreads();
        if ((int)blockIdx.y >= *a.ntiles) return;  // uniform: no TMEM touched yet
    }
    const int64_t m0 = (int64_t)blockIdx.x * XG_M;
    if (m0 >= a.M) return;
    const int e = tile.e;
    // first (expert-major) activation row of the N tile
    const int64_t grow0 = (MODE == XG_DENSE ? 0 : (int64_t)a.offs[e]) + tile.row0;
    const int KT = (int)(a.K / XG_K);

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            mbar_init(&full_a[s], 128);
            mbar_init(&full_b[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&tmem_base, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    // expert (or dense) weights
    const uint8_t *wmat[2];
    const uint8_t *smat[2];
    int rebase[2] = {0, 0};
    if (MODE == XG_DENSE) {
        wmat[0] = a.dense_w;
        smat[0] = a.dense_s;
    } else {
        const uint8_t *eb = a.experts_layer + (int64_t)e * a.L.expert_stride;
        const int mm0 = MODE == XG_DOWN ? 2 : 0;
        wmat[0] = eb + a.L.off[mm0][0];
        smat[0] = eb + a.L.off[mm0][1];
        wmat[1] = eb + a.L.off[1][0];
        smat[1] = eb + a.L.off[1][1];
        if (DT != MG_Q8R) {
            rebase[0] = a.rebase[e * 3 + mm0];
            rebase[1] = a.rebase[e * 3 + 1];
        }
    }
    bool ok = true;
    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            int issued = 0;
            for (int kt = 0; kt < KT && ok; kt++) {
                const int s = kt % C::STAGES;
                if (kt >= C::STAGES) ok = mbar_wait(&empty[s], ((kt / C::STAGES) - 1) & 1);
                if (!ok) break;
                uint8_t *st = base + (size_t)s * C::STAGE;
                mbar_arrive_expect_tx(&full_b[s], 2 * XG_TILE_BYTES);
                tma_load_2d(st + C::NA * XG_TILE_BYTES, &tm_hi, kt * XG_K, (int)grow0, &full_b[s]);
                tma_load_2d(st + (C::NA + 1) * XG_TILE_BYTES, &tm_lo, kt * XG_K, (int)grow0, &full_b[s]);
                issued = kt + 1;
            }
            if (!ok) atomicExch(a.err, XG_ERR);
            // every copy this thread issued has landed before the CTA may exit
            for (int s = 0; s < C::STAGES && s < issued; s++) {
                const int kl = s + ((issued - 1 - s) / C::STAGES) * C::STAGES;
                if (!mbar_wait(&full_b[s], (kl / C::STAGES) & 1)) atomicExch(a.err, XG_ERR);
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(XG_M, XG_N);
            for (int kt = 0; kt < KT && ok; kt++) {
                const int s = kt % C::STAGES;
                const uint32_t par = (kt / C::STAGES) & 1;
                ok = mbar_wait(&full_b[s], par) && mbar_wait(&full_a[s], par);
                if (!ok) break;
                tc_fence_after();
                const uint32_t st = smem_u32(base + (size_t)s * C::STAGE);
                const uint32_t bh = st + C::NA * XG_TILE_BYTES, bl = st + (C::NA + 1) * XG_TILE_BYTES;
#pragma unroll
                for (int kk = 0; kk < XG_K / 16; kk++) {
                    const uint32_t koff = kk * 32;  // 16 f16 = 32 bytes along K inside the swizzle atom
                    const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
                    for (int na = 0; na < C::NA; na++) {
                        const uint64_t ad = umma_desc_sw128(st + na * XG_TILE_BYTES + koff);
                        const uint32_t td = tmem + na * XG_N;
                        tc_mma_f16(td, ad, umma_desc_sw128(bh + koff), idesc, acc);
                        tc_mma_f16(td, ad, umma_desc_sw128(bl + koff), idesc, 1u);
                    }
                }
                tc_commit(&empty[s]);  // stage s free once these MMAs have read it
            }
            tc_commit(&acc_full);  // also on failure: arrives once the MMAs issued so far are done
            if (!ok) atomicExch(a.err, XG_ERR);
        }
    } else {
        // ------------------------------------------- converters + epilogue
        const int tid = threadIdx.x - 64;  // 0..127: the weight row this thread converts
        // the row's raw bytes of k-tiles kt, kt + 1 and kt + 2: each load is
        // issued two k-tiles before its conversion (one ahead left the
        // converters waiting on HBM, not the tensor core)
        XgRaw<DT> cur[C::NA], nxt[C::NA], nx2[C::NA];
#pragma unroll
        for (int na = 0; na < C::NA; na++) {
            xg_load<DT>(cur[na], wmat[na], smat[na], a.M, a.K, m0 + tid, 0);
            if (KT > 1) xg_load<DT>(nxt[na], wmat[na], smat[na], a.M, a.K, m0 + tid, 1);
        }
        for (int kt = 0; kt < KT && ok; kt++) {
            if (kt + 2 < KT) {
#pragma unroll
                for (int na = 0; na < C::NA; na++) xg_load<DT>(nx2[na], wmat[na], smat[na], a.M, a.K, m0 + tid, kt + 2);
            }
            const int s = kt % C::STAGES;
            if (kt >= C::STAGES) ok = mbar_wait(&empty[s], ((kt / C::STAGES) - 1) & 1);
            if (!ok) break;
            uint8_t *st = base + (size_t)s * C::STAGE;
#pragma unroll
            for (int na = 0; na < C::NA; na++) xg_store<DT>(st + na * XG_TILE_BYTES, cur[na], rebase[na], tid);
            fence_proxy_async_smem();
            mbar_arrive(&full_a[s]);
#pragma unroll
            for (int na = 0; na < C::NA; na++) {
                cur[na] = nxt[na];
                nxt[na] = nx2[na];
            }
        }
        const bool acc_ok = mbar_wait(&acc_full, 0);  // always: TMEM is freed only after the MMAs
        ok = ok && acc_ok;
        if (!ok) {
            if (tid == 0) atomicExch(a.err, XG_ERR);
        } else {
            tc_fence_after();
            const int q = warp & 3;  // TMEM lane quarter this warp may access
            const int64_t row = m0 + 32 * q + lane;
            const bool rv = row < a.M;
            float scale0 = 1.f, scale1 = 1.f, b0 = 0.f, b1 = 0.f;
            if (rv) {
                if (DT == MG_Q8R) {
                    scale0 = reinterpret_cast<const float *>(smat[0])[row];
                    if (MODE == XG_GATEUP) scale1 = reinterpret_cast<const float *>(smat[1])[row];
                } else {
                    scale0 = exp2f((float)rebase[0]);
                    scale1 = exp2f((float)rebase[1]);
                }
                if (MODE == XG_DENSE) {
                    b0 = a.dense_bias ? a.dense_bias[row] : 0.f;
                } else {
                    const uint8_t *eb = a.experts_layer + (int64_t)e * a.L.expert_stride;
                    const int mm0 = MODE == XG_DOWN ? 2 : 0;
                    b0 = reinterpret_cast<const float *>(eb + a.L.off[mm0][2])[row];
                    if (MODE == XG_GATEUP) b1 = reinterpret_cast<const float *>(eb + a.L.off[1][2])[row];
                }
            }
            for (int c0 = 0; c0 < XG_N; c0 += 16) {
                float vg[16], vu[16];
                tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c0, vg);
                if (MODE == XG_GATEUP) tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + XG_N + c0, vu);
                if (!rv) continue;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const int n = c0 + j;
                    if (n >= tile.nrows) break;
                    const int64_t p = grow0 + n;
                    if (MODE == XG_GATEUP) {
                        float g = __fadd_rn(__fmul_rn(vg[j], scale0), b0);
                        float u = __fadd_rn(__fmul_rn(vu[j], scale1), b1);
                        float hv;
                        if (a.act_plain) {
                            hv = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                        } else {
                            if (g > a.limit) g = a.limit;
                            if (u > a.limit) u = a.limit;
                            if (u < -a.limit) u = -a.limit;
                            hv = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(__fmul_rn(-a.alpha, g)))), __fadd_rn(u, 1.0f));
                        }
                        __half hi, lo;
                        split_f16(hv, hi, lo);
                        a.out_hi[p * a.M + row] = hi;
                        a.out_lo[p * a.M + row] = lo;
                    } else {
                        const float v = __fadd_rn(__fmul_rn(vg[j], scale0), b0);
                        const int64_t yr = MODE == XG_DOWN ? (int64_t)a.slot_of_pos[p] : p;
                        float *yp = a.y + yr * a.ldy + row;
                        *yp = (MODE == XG_DENSE && a.accumulate) ? __fadd_rn(*yp, v) : v;
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------ host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// [rows x K] f16 row-major -> TMA map with a 64 x 128 box, 128-byte swizzle
static int make_map(CUtensorMap *map, const __half *ptr, int64_t rows, int64_t K) {
    EncodeTiledFn fn = encode_fn();
    MG_REQUIRE(fn, MG_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    MG_REQUIRE((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (K * 2) % 16 == 0, MG_ERR_ARG,
               "xgemm: activation buffer misaligned");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {XG_K, XG_N};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    MG_REQUIRE(r == CUDA_SUCCESS, MG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return MG_OK;
}

template <int MODE, int DT>
static int launch_xg(const XgLaunch &l, cudaStream_t st) {
    using C = XgCfg<MODE>;
    CUtensorMap mh, ml;
    int rc = make_map(&mh, l.x_hi, l.x_rows, l.args.K);
    if (rc) return rc;
    rc = make_map(&ml, l.x_lo, l.x_rows, l.args.K);
    if (rc) return rc;
    const size_t smem = (size_t)C::STAGES * C::STAGE + 1024;
    auto kfn = k_xgemm<MODE, DT>;
    rc = ensure_smem(kfn, smem);
    if (rc) return rc;
    dim3 grid((unsigned)ceil_div(l.args.M, XG_M), (unsigned)l.max_tiles);
    kfn<<<grid, XG_THREADS, smem, st>>>(mh, ml, l.args);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int xgemm(int mode, int dt, const XgLaunch &l, cudaStream_t st) {
    MG_REQUIRE(l.args.K % XG_K == 0, MG_ERR_ARG, "xgemm: K %lld not a multiple of 64", (long long)l.args.K);
    MG_REQUIRE(dt == MG_MXFP4 || dt == MG_Q8R, MG_ERR_ARG, "xgemm: dtype %d unsupported", dt);
    if (l.max_tiles <= 0) return MG_OK;
    if (mode == XG_GATEUP) return dt == MG_Q8R ? launch_xg<XG_GATEUP, MG_Q8R>(l, st) : launch_xg<XG_GATEUP, MG_MXFP4>(l, st);
    if (mode == XG_DOWN) return dt == MG_Q8R ? launch_xg<XG_DOWN, MG_Q8R>(l, st) : launch_xg<XG_DOWN, MG_MXFP4>(l, st);
    return dt == MG_Q8R ? launch_xg<XG_DENSE, MG_Q8R>(l, st) : launch_xg<XG_DENSE, MG_MXFP4>(l, st);
}

}  // namespace mg

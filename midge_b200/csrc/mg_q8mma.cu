// mg_q8mma.cu -- decode-time GEMV of int8 rows with an f32 scale per row (the
// q8r trunk: q, k, v and o; engine/mkern.h q8 rows, y = scale * sum w x + bias)
// on tcgen05.mma.kind::i8 (s8 x s8 -> s32 in TMEM).
//
// The activations become exact integers: the slice of token t's row x that
// one unit multiplies (its K split) is held as four int8 limbs under one
// power-of-two scale 2^e (2^e >= the slice's max|x| / 127):
//   x = 2^e (q0 + q1 2^-7 + q2 2^-14 + q3 2^-21) + r,  |r| <= 2^(e-22)
// (each limb the round-to-nearest of the scaled residual, |q0| <= 127 and
// |q1..3| <= 64).  The MMA sums w q_l exactly in int32 (|sum| < 2^31 for
// K < 133,000), the epilogue adds the four sums in double (exact: they span
// < 53 bits) and rounds once to f32 at 2^e; then * row scale + bias as the
// mma.sync kernels do.  The error against f32 inputs is |sum w r| <=
// 2^(e-22) sum |w|, below the f16 hi/lo split's.
//
// Units: 128-row tiles of up to three matrices (q, k, v share the input) x
// K splits of whole 128-byte segments; each K split writes its partial plane
// (bias in split 0), summed downstream in plane order.  Roles (320 threads,
// one CTA per SM, each CTA a contiguous, balanced range of units):
//   warp 0    producer: first every unit's f32 activation slice (all
//             tokens) by bulk copy, then per segment the A box (128 rows x
//             128 B) by TMA into a ring stage
//   warp 1    MMA issuer: 4 MMAs (K = 32) per stage into one of eight TMEM
//             accumulators (128 lanes x 32 columns: token t limb l = t*4+l),
//             so the MMAs never wait for the epilogue of a CTA's few units
//   warps 2-5 epilogue (TMEM lane quadrant = warp % 4): one output row each
//   warps 6-9 activation limbs of each unit's K slice (two tokens per warp;
//             the producer first bulk-copies every unit's f32 slice into
//             shared memory) into the unit's own buffer, written in the
//             128-byte swizzle the MMA reads.
// Every wait is bounded and records a code in the stream's error word.
#include <cfloat>

#include "mg_q8mma.h"
#include "mg_stream.cuh"
#include "mg_tc.cuh"

namespace mg {

constexpr int QM_TOK = 8, QM_LIMBS = 4, QM_N = QM_TOK * QM_LIMBS;  // B rows = MMA N
constexpr int QM_A = 128 * 128;                                    // A box: 128 rows x 128 B
constexpr int QM_B = QM_N * 128;                                   // limb box: 32 rows x 128 B
constexpr int QM_MAX_STAGES = 8;
constexpr int QM_THREADS = 320;
constexpr int QM_NACC = 8;                   // TMEM accumulators: the MMAs run up to 8 units ahead
constexpr int QM_TMEM_COLS = QM_NACC * QM_N;  // 256 columns
constexpr int QM_MAXU = 8;                    // units per CTA (each with its own activation buffer)
constexpr int QM_NONFINITE = 0x7fffffff;  // xe of a row with a NaN or infinity: its outputs are NaN
// error word codes (first failure kept): producer 41, MMA 42 (43 accumulator buffer, 46 activation
// buffer), epilogue 44, drain 45, activation encoders 47
__device__ __forceinline__ void qm_fail(int *err, int code) { atomicCAS(err, 0, code); }

struct QmBars {
    uint64_t full[QM_MAX_STAGES], empty[QM_MAX_STAGES], accfull[QM_NACC], accempty[QM_NACC], bfull[QM_MAXU];
    uint64_t xfull, done;
    int es[QM_MAXU][QM_TOK];  // scale exponents of the CTA's unit q's tokens
    uint32_t tmem;
};
struct QmMaps {
    CUtensorMap a[3];
};
struct QmMat {
    const float *scales, *bias;
    float *y;
    int64_t rows, ldy, tile0;
};
struct QmPol {
    QmMat m[3];
    int nmat, ks_count, sps, nseg, n_tok, accumulate;
    int64_t ntiles, part_stride, K, ldx;
    const float *x;
    int *err;
    __device__ int mat_of(int64_t tile) const {
        int k = 0;
        if (nmat > 1 && tile >= m[1].tile0) k = 1;
        if (nmat > 2 && tile >= m[2].tile0) k = 2;
        return k;
    }
};
#define QM_SEL(i, f) ((i) == 0 ? p.m[0].f : ((i) == 1 ? p.m[1].f : p.m[2].f))

// instruction descriptor, kind::i8: D s32 (2), A and B s8 (1), K-major, N, M = 128
__device__ __forceinline__ uint32_t qm_idesc(int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
__device__ __forceinline__ void qm_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}

__global__ void __launch_bounds__(QM_THREADS, 1) k_q8mma(const __grid_constant__ QmMaps maps, QmPol p, int nst,
                                                        int bbytes, int nu) {
    extern __shared__ __align__(1024) uint8_t qm_raw[];
    uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(qm_raw) + 1023) & ~(uintptr_t)1023);
    uint8_t *bbuf = ring + (size_t)nst * QM_A;  // per unit [segment][32 rows x 128 B], 1024-aligned
    float *xs = reinterpret_cast<float *>(bbuf + (size_t)nu * bbytes);  // per unit [token][sps * 128] f32
    QmBars *bb = reinterpret_cast<QmBars *>(reinterpret_cast<uint8_t *>(xs) + (size_t)nu * bbytes);
    const int xslot = p.sps * 128;  // floats of one token's slice
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int i = 0; i < nst; i++) {
            mbar_init(&bb->full[i], 1);
            mbar_init(&bb->empty[i], 1);
        }
        for (int i = 0; i < QM_NACC; i++) {
            mbar_init(&bb->accfull[i], 1);
            mbar_init(&bb->accempty[i], 4);
        }
        for (int i = 0; i < QM_MAXU; i++) mbar_init(&bb->bfull[i], 1);
        mbar_init(&bb->xfull, 1);
        mbar_init(&bb->done, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&bb->tmem, QM_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = bb->tmem;
    const int64_t nunits = p.ntiles * p.ks_count;
    const int64_t u0 = nunits * blockIdx.x / gridDim.x, u1 = nunits * (blockIdx.x + 1) / gridDim.x;
    auto unit = [&](int64_t u, int64_t &tile, int &ks, int &s0, int &s1, int &mi, int64_t &row0) {
        tile = u / p.ks_count;
        ks = (int)(u - tile * p.ks_count);
        s0 = ks * p.sps;
        s1 = min(p.nseg, s0 + p.sps);
        mi = p.mat_of(tile);
        row0 = (tile - QM_SEL(mi, tile0)) * 128;
    };
    if (warp == 0) {
        // ---------------------------------------------------------- producer
        if (lane == 0) {
            bool ok = true;
            int s = 0;
            uint32_t ph = 0, it = 0;
            {  // every unit's activation slice, all tokens, into shared memory first
                uint32_t total = 0;
                for (int64_t u = u0; u < u1; u++) {
                    int64_t tile, row0;
                    int ks, s0, s1, mi;
                    unit(u, tile, ks, s0, s1, mi, row0);
                    total += (uint32_t)(p.n_tok * (min(p.K, (int64_t)s1 * 128) - (int64_t)s0 * 128) * 4);
                }
                mbar_arrive_expect_tx(&bb->xfull, total);
                int q = 0;
                for (int64_t u = u0; u < u1; u++, q++) {
                    int64_t tile, row0;
                    int ks, s0, s1, mi;
                    unit(u, tile, ks, s0, s1, mi, row0);
                    const int64_t kbeg = (int64_t)s0 * 128, kend = min(p.K, (int64_t)s1 * 128);
                    for (int t = 0; t < p.n_tok; t++)
                        bulk_g2s(xs + (size_t)(q * QM_TOK + t) * xslot, p.x + (int64_t)t * p.ldx + kbeg,
                                 (uint32_t)((kend - kbeg) * 4), &bb->xfull);
                }
            }
            for (int64_t u = u0; u < u1 && ok; u++) {
                int64_t tile, row0;
                int ks, s0, s1, mi;
                unit(u, tile, ks, s0, s1, mi, row0);
                for (int g = s0; g < s1; g++) {
                    if (it >= (uint32_t)nst && !mbar_wait(&bb->empty[s], ph ^ 1u)) { ok = false; break; }
                    mbar_arrive_expect_tx(&bb->full[s], QM_A);
                    tma_box_2d(ring + (size_t)s * QM_A, &maps.a[mi], g * 128, (int)row0, &bb->full[s]);
                    it++;
                    if (++s == nst) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) qm_fail(p.err, 41);
            for (int64_t k = (int64_t)it - 1; k >= 0 && k >= (int64_t)it - nst; k--)
                if (!mbar_wait(&bb->full[k % nst], (uint32_t)((k / nst) & 1))) qm_fail(p.err, 45);
            if (!mbar_wait(&bb->xfull, 0)) qm_fail(p.err, 45);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = true;
            int s = 0, q = 0;
            uint32_t ph = 0;
            const uint64_t da0 = umma_desc_sw128(smem_u32(ring)), db0 = umma_desc_sw128(smem_u32(bbuf));
            const uint32_t idesc = qm_idesc(QM_N);
            for (int64_t u = u0; u < u1 && ok; u++, q++) {
                int64_t tile, row0;
                int ks, s0, s1, mi;
                unit(u, tile, ks, s0, s1, mi, row0);
                const int b = q % QM_NACC;
                if (q >= QM_NACC && !mbar_wait(&bb->accempty[b], (uint32_t)((q / QM_NACC - 1) & 1))) {
                    qm_fail(p.err, 43);
                    ok = false;
                    break;
                }
                if (!mbar_wait(&bb->bfull[q], 0)) {
                    qm_fail(p.err, 46);
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t tacc = tb + (uint32_t)(b * QM_N);
                for (int g = s0; g < s1; g++) {
                    if (!mbar_wait(&bb->full[s], ph)) { ok = false; break; }
                    tc_fence_after();
                    // descriptors: the start-address field is the low 14 bits (address >> 4)
                    const uint64_t da = da0 + (uint64_t)((s * QM_A) >> 4);
                    const uint64_t db = db0 + (uint64_t)((q * bbytes + (g - s0) * QM_B) >> 4);
#pragma unroll
                    for (int j = 0; j < 4; j++)  // K = 32 bytes per MMA
                        qm_mma(tacc, da + 2 * j, db + 2 * j, idesc, (g > s0 || j > 0) ? 1u : 0u);
                    tc_commit(&bb->empty[s]);
                    if (++s == nst) { s = 0; ph ^= 1u; }
                }
                if (ok) tc_commit(&bb->accfull[b]);  // also: the unit's activation buffer may be rewritten
            }
            if (!ok) qm_fail(p.err, 42);
            tc_commit(&bb->done);
            if (!mbar_wait(&bb->done, 0)) qm_fail(p.err, 42);
        }
    } else if (warp < 6) {
        // ---------------------------------------------------------- epilogue
        const int ew = warp & 3, r = 32 * ew + lane;  // TMEM lane quadrant = warp % 4
        bool failed = false;
        int q = 0;
        for (int64_t u = u0; u < u1; u++, q++) {
            int64_t tile, row0;
            int ks, s0, s1, mi;
            unit(u, tile, ks, s0, s1, mi, row0);
            const int b = q % QM_NACC;
            if (!failed && !mbar_wait(&bb->accfull[b], (uint32_t)((q / QM_NACC) & 1))) {
                failed = true;
                if (lane == 0) qm_fail(p.err, 44);
            }
            // the encoders' arrival publishes the unit's exponents (completed already)
            if (!failed && !mbar_wait(&bb->bfull[q], 0)) {
                failed = true;
                if (lane == 0) qm_fail(p.err, 44);
            }
            if (failed) continue;
            tc_fence_after();
            int e[QM_TOK];
#pragma unroll
            for (int t = 0; t < QM_TOK; t++) e[t] = bb->es[q][t];
            float raw[QM_N];
            tmem_ld16(tb + (uint32_t)(b * QM_N) + ((uint32_t)(32 * ew) << 16), raw);
            tmem_ld16(tb + (uint32_t)(b * QM_N + 16) + ((uint32_t)(32 * ew) << 16), raw + 16);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bb->accempty[b]);
            const int64_t row = row0 + r;
            if (row >= QM_SEL(mi, rows)) continue;
            const float rs = QM_SEL(mi, scales)[row];
            const float *mb = QM_SEL(mi, bias);
            const float bias = (mb && ks == 0) ? mb[row] : 0.f;
            float *my = QM_SEL(mi, y);
            const int64_t ldy = QM_SEL(mi, ldy);
#pragma unroll
            for (int t = 0; t < QM_TOK; t++) {
                if (t >= p.n_tok) break;
                float v;
                if (e[t] == QM_NONFINITE) {
                    v = __int_as_float(0x7fc00000);
                } else {
                    const double sum = (double)__float_as_int(raw[4 * t]) +
                                       (double)__float_as_int(raw[4 * t + 1]) * 0x1p-7 +
                                       (double)__float_as_int(raw[4 * t + 2]) * 0x1p-14 +
                                       (double)__float_as_int(raw[4 * t + 3]) * 0x1p-21;
                    // * 2^e exactly (e in [-156, 121]: a normal double), one rounding to f32
                    v = (float)(sum * __longlong_as_double((long long)(1023 + e[t]) << 52));
                }
                v = __fadd_rn(__fmul_rn(v, rs), bias);
                if (p.ks_count == 1) {
                    float *yp = my + (int64_t)t * ldy + row;
                    *yp = p.accumulate ? __fadd_rn(*yp, v) : v;
                } else {
                    my[(int64_t)ks * p.part_stride + (int64_t)t * ldy + row] = v;
                }
            }
        }
    } else {
        // ---------------------------------------------------------- activation limbs
        // warp w encodes tokens 2 (w - 6) and 2 (w - 6) + 1 of each unit's K
        // slice (in shared memory) into the unit's buffer, in the 128-byte
        // swizzle the MMA reads: row r, byte k of segment g at g*4096 +
        // (r/8)*1024 + (r%8)*128 + ((k/16) ^ (r%8))*16 + k%16; lane = 4
        // consecutive values.  After a timed-out wait the warps stop encoding
        // but keep taking part in their named barrier.
        const int ew = warp - 6;
        bool failed = false;
        if (!mbar_wait(&bb->xfull, 0)) {
            failed = true;
            if (lane == 0) qm_fail(p.err, 47);
        }
        int q = 0;
        for (int64_t u = u0; u < u1; u++, q++) {
            int64_t tile, row0;
            int ks, s0, s1, mi;
            unit(u, tile, ks, s0, s1, mi, row0);
            if (!failed) {
                uint8_t *buf = bbuf + (size_t)q * bbytes;
                const int n = (int)(min(p.K, (int64_t)s1 * 128) - (int64_t)s0 * 128);  // values in the slice
                const int nb = (s1 - s0) * 128;
#pragma unroll
                for (int tt = 0; tt < 2; tt++) {
                    const int t = 2 * ew + tt;
                    const bool live = t < p.n_tok;
                    const float *xr = xs + (size_t)(q * QM_TOK + t) * xslot;
                    float m = 0.f;
                    bool bad = false;
                    if (live)
                        for (int k = 4 * lane; k < n; k += 128) {
                            const float4 v = *reinterpret_cast<const float4 *>(xr + k);
                            const float a[4] = {fabsf(v.x), fabsf(v.y), fabsf(v.z), fabsf(v.w)};
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                if (a[i] <= FLT_MAX) m = fmaxf(m, a[i]);
                                else bad = true;
                            }
                        }
                    m = warp_max(m);
                    bad = __any_sync(0xffffffffu, bad);
                    int e = 0;
                    if (bad) {
                        e = QM_NONFINITE;
                    } else if (m > 0.f) {  // smallest e with m <= 127 * 2^e
                        int E;
                        const float f = frexpf(m, &E);  // m = f 2^E, f in [0.5, 1)
                        e = f <= 127.f / 128.f ? E - 7 : E - 6;
                    }
                    if (lane == 0) bb->es[q][t] = e;
                    // 2^-e as a float when normal (the usual case), else scalbnf
                    const bool pn = e != QM_NONFINITE && e > -127 && e < 127;
                    const float pw = pn ? __int_as_float((127 - e) << 23) : 0.f;
                    for (int kk = 4 * lane; kk < nb; kk += 128) {
                        uint32_t wd[QM_LIMBS] = {0u, 0u, 0u, 0u};
                        if (live && !bad && kk < n) {
                            const float4 v = *reinterpret_cast<const float4 *>(xr + kk);
                            const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                float y = pn ? xv[i] * pw : scalbnf(xv[i], -e);  // |y| <= 127, exact
#pragma unroll
                                for (int l = 0; l < QM_LIMBS; l++) {
                                    const float rq = rintf(y);
                                    wd[l] |= ((uint32_t)(int)rq & 0xFFu) << (8 * i);
                                    y = (y - rq) * 128.f;  // exact: the residual of a round-to-nearest
                                }
                            }
                        }
                        const int g = kk >> 7, kb = kk & 127;
#pragma unroll
                        for (int l = 0; l < QM_LIMBS; l++) {
                            const int rr = t * QM_LIMBS + l;
                            *reinterpret_cast<uint32_t *>(buf + g * QM_B + (rr >> 3) * 1024 + (rr & 7) * 128 +
                                                          ((((kb >> 4) ^ (rr & 7))) << 4) + (kb & 15)) = wd[l];
                        }
                    }
                }
                fence_proxy_async_smem();
            }
            named_bar_sync(2, 128);  // the four encoder warps
            if (ew == 0 && lane == 0 && !failed) mbar_arrive(&bb->bfull[q]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tb, QM_TMEM_COLS);
    }
}
#undef QM_SEL

// ---------------------------------------------------------------- host side
bool q8mma_supported(const StreamGemvArgs &a) {
    if (a.dt != MG_Q8R || a.amax || a.nmat < 1 || a.nmat > 3 || !a.x || a.cols <= 0 || a.cols % 16) return false;
    if (a.n_tok < 1 || a.n_tok > QM_TOK || a.ldx % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return false;
    for (int i = 0; i < a.nmat; i++)
        if (!a.mat[i].map || !a.mat[i].scales || !a.mat[i].y || a.mat[i].rows <= 0) return false;
    return true;
}

int q8mma_gemv(const StreamGemvArgs &a, cudaStream_t st) {
    MG_REQUIRE(q8mma_supported(a), MG_ERR_ARG, "int8 tensor-core gemv: unsupported call");
    int *err = stream_error_word();
    MG_REQUIRE(err, MG_ERR_OOM, "int8 tensor-core gemv: no error word");
    QmMaps maps;
    memset(&maps, 0, sizeof(maps));
    QmPol p{};
    int64_t tiles = 0;
    for (int i = 0; i < a.nmat; i++) {
        maps.a[i] = *a.mat[i].map;
        p.m[i].scales = reinterpret_cast<const float *>(a.mat[i].scales);
        p.m[i].bias = a.mat[i].bias;
        p.m[i].y = a.mat[i].y;
        p.m[i].rows = a.mat[i].rows;
        p.m[i].ldy = a.mat[i].ldy;
        p.m[i].tile0 = tiles;
        tiles += (a.mat[i].rows + 127) / 128;
    }
    p.nmat = a.nmat;
    p.ntiles = tiles;
    p.nseg = (int)((a.cols + 127) / 128);
    p.ks_count = stream_ksplit(MG_Q8R, a.cols, a.ksplit);  // the same planes as the mma.sync kernels
    p.sps = (p.nseg + p.ks_count - 1) / p.ks_count;
    p.n_tok = a.n_tok;
    p.accumulate = a.accumulate;
    p.part_stride = a.part_stride;
    p.K = a.cols;
    p.x = a.x;
    p.ldx = a.ldx;
    p.err = err;
    // per unit: its activation limbs (32 rows x the slice) and its f32 slice
    // of the 8 tokens, both sps x 4 KB
    const int bbytes = p.sps * QM_B;
    const int64_t units = tiles * p.ks_count;
    const int nsm = num_sms();
    const int grid = (int)(units < nsm ? units : nsm);
    const int nu = (int)((units + grid - 1) / grid);  // most units of a CTA
    cudaFuncAttributes fa{};
    MG_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(k_q8mma)));
    const size_t budget = 227 * 1024 - fa.sharedSizeBytes;
    const size_t fixed = 1024 + 2 * (size_t)nu * bbytes + sizeof(QmBars);
    MG_REQUIRE(nu <= QM_MAXU && budget > fixed + 2 * (size_t)QM_A, MG_ERR_ARG,
               "int8 tensor-core gemv: %d units of %d K stages per CTA do not fit", nu, p.sps);
    int nst = (int)((budget - fixed) / QM_A);
    if (nst > QM_MAX_STAGES) nst = QM_MAX_STAGES;
    const size_t smem = fixed + (size_t)nst * QM_A;
    int rc = ensure_smem_attr(reinterpret_cast<const void *>(k_q8mma), smem);
    if (rc) return rc;
    k_q8mma<<<grid, QM_THREADS, smem, st>>>(maps, p, nst, bbytes, nu);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

}  // namespace mg

// mg_tmoe.cu -- decode routed-expert FFN on the 5th-generation tensor cores.
//
// Same work split as the streamed MoE kernels (units = 64 gate+up output rows
// of one routed expert, or 128 down rows x a K split), but the arithmetic runs
// as tcgen05.mma with the weights as the A operand in tensor memory:
//   * warp 0 (one lane) streams 128-row x 128-byte weight boxes by TMA into a
//     shared-memory ring and bulk-copies each unit's ue8m0 scales;
//   * warps 2..9 (converters; TMEM lane quarter = warp % 4, stage half =
//     (warp - 2) / 4) decode their row's half of each stage -- e2m1 or int8 ->
//     f16, times 2^(scale code - 127 - k0) for MXFP4, exact with the matrix's
//     rebase k0 -- and store it to an A buffer in TMEM (tcgen05.st);
//   * warp 1 (one lane) owns TMEM and issues, per stage, the K/16 MMAs
//     D[128 x 16] += A[128 x 16] . B[16 x 16]^T, B = the tokens' activations
//     as f16 hi/lo rows (row 2t = hi, 2t+1 = lo of token t), staged once in
//     shared memory in the 128B-swizzled K-major layout;
//   * warps 10..13 (epilogue) read D back (tcgen05.ld), undo the rebase (or
//     apply the int8 row scale), add the bias and run the clamped/plain SwiGLU
//     (gate/up) or store the partial sums (down).
// Accumulation is fp32 in the tensor core, as in the prefill GEMM.  Every
// wait is bounded; a timed-out role records an error, stops waiting and
// computing, and keeps taking part in the named barriers.
#include "mg_common.cuh"
#include "mg_kernels.h"
#include "mg_stream.cuh"
#include "mg_tc.cuh"

namespace mg {

constexpr int TM_WARPS = 14, TM_THREADS = TM_WARPS * 32;
constexpr int TM_CONV0 = 2, TM_EPI0 = 10;
constexpr int TM_NA = 3;                  // A buffers in TMEM
constexpr int TM_ACOLS = 128;             // TMEM columns per A buffer (one stage of K)
constexpr int TM_D0 = TM_NA * TM_ACOLS;   // two D buffers of 16 columns from here
constexpr int TM_TCOLS = 512;             // allocation (power of two >= 416)
constexpr int TM_N = 16;                  // MMA N: 8 tokens x (hi, lo)
constexpr int TM_ERR = 4;
enum { TM_GATEUP = 0, TM_DOWN = 1 };

struct TmBars {
    uint64_t full[SW_MAX_STAGES], empty[SW_MAX_STAGES];
    uint64_t sfull[2], sempty[2];
    uint64_t afull[TM_NA], aempty[TM_NA];
    uint64_t dfull[2], dempty[2];
    uint64_t bready, fin;
    uint32_t tmem;
};

struct TmArgs {
    MoeStreamArgs a;
    const int *rebase;  // [n_local x 3] of this layer (MXFP4)
    int ks_count;       // down K split
    int64_t kbytes_per_split;
    int nstages, ssb;
    int *err;
};

// B operand: nrow (<= 16) activation rows as f16 hi/lo, K-major, 128-byte
// swizzle: row r, column k at (k/64)*2048 + r*128 + (((k%64)/8 ^ r%7)... (see addr)
__device__ __forceinline__ void tm_stage_rows(const float *const *rows, int nrow, int64_t K, uint8_t *xsb, int tid,
                                              int nthr) {
    const int64_t q8 = K / 8;
    for (int64_t i = tid; i < (int64_t)nrow * q8; i += nthr) {
        const int j = (int)(i / q8);
        const int64_t k8 = (i - (int64_t)j * q8) * 8;
        const float4 *src = reinterpret_cast<const float4 *>(rows[j] + k8);
        const float4 p = src[0], q = src[1];
        const float v[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
        __half hi[8], lo[8];
#pragma unroll
        for (int e = 0; e < 8; e++) split_f16(v[e], hi[e], lo[e]);
        const int64_t kb = k8 / 64;
        const int c = (int)((k8 % 64) / 8);
        const int rh = 2 * j, rl = 2 * j + 1;
        *reinterpret_cast<uint4 *>(xsb + kb * 2048 + rh * 128 + ((c ^ (rh & 7)) << 4)) = *reinterpret_cast<uint4 *>(hi);
        *reinterpret_cast<uint4 *>(xsb + kb * 2048 + rl * 128 + ((c ^ (rl & 7)) << 4)) = *reinterpret_cast<uint4 *>(lo);
    }
}

template <int MODE>
struct TmUnit {
    int aux;      // index into the distinct-expert list
    int64_t tile;
    int ks;
    int64_t b0, b1;
};

template <int DT, int MODE>
__global__ void __launch_bounds__(TM_THREADS, 1) k_tmoe(const __grid_constant__ SwMaps maps, TmArgs t) {
    extern __shared__ __align__(1024) uint8_t tm_raw[];
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tm_raw) + 1023) & ~(uintptr_t)1023);
    const MoeStreamArgs &a = t.a;
    const mg_expert_layout &L = a.L;
    const int64_t K = MODE == TM_GATEUP ? L.hidden : L.ffn;        // reduction length
    const int64_t M = MODE == TM_GATEUP ? L.ffn : L.hidden;        // output rows of the matrix
    const int64_t rowbytes = DT == MG_Q8R ? K : K / 2;
    const int64_t gpr = K / 32;                                     // scale groups per row (MXFP4)
    const int nst = t.nstages;
    uint8_t *ring = base;
    uint8_t *xsb = ring + (size_t)nst * SW_STAGE_BYTES;            // K/64 blocks of 16 rows x 128 B
    const size_t xsb_bytes = (size_t)((K + 63) / 64) * 2048;
    uint8_t *ss = xsb + xsb_bytes;                                 // 2 scale slots
    float *upbuf = reinterpret_cast<float *>(ss + 2 * (size_t)t.ssb);  // [64 rows][8 tokens]
    __shared__ TmBars bars;
    __shared__ MoeShared msh;
    __shared__ int s_slots[2][16], s_ne[2];

    MoeCommon mc;
    mc.L = L;
    mc.experts_layer = a.experts_layer;
    mc.layer = a.layer;
    mc.e0 = a.e0;
    mc.n_experts = a.n_experts;
    mc.n_tok = a.n_tok;
    mc.top_k = a.top_k;
    mc.sel = a.sel;
    mc.ms = &msh;
    mc.build_list();  // all threads; ends with __syncthreads

    const int64_t tpe = MODE == TM_GATEUP ? (M + 63) / 64 : ((M + 127) / 128) * t.ks_count;
    const int64_t nunits = (int64_t)msh.nd * tpe;
    const int64_t per = (nunits + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = (int64_t)blockIdx.x * per, u1 = min(nunits, u0 + per);
    if (u0 >= u1) return;  // uniform: no barrier or TMEM touched

    auto unit_of = [&](int64_t u) {
        TmUnit<MODE> ui;
        ui.aux = (int)(u / tpe);
        const int64_t r = u % tpe;
        if (MODE == TM_GATEUP) {
            ui.tile = r;
            ui.ks = 0;
            ui.b0 = 0;
            ui.b1 = rowbytes;
        } else {
            ui.tile = r / t.ks_count;
            ui.ks = (int)(r % t.ks_count);
            ui.b0 = (int64_t)ui.ks * t.kbytes_per_split;
            ui.b1 = min(rowbytes, ui.b0 + t.kbytes_per_split);
        }
        return ui;
    };
    // down: the slots routed to expert list entry aux (<= 16), for the B rows
    auto slots_of = [&](int aux, int *slots) {
        const int eg = msh.list[aux] + a.e0;
        int k = 0;
        for (int i = 0; i < a.n_tok * a.top_k && k < 8; i++)
            if (a.sel[i] == eg) slots[k++] = i;
        return k;
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- set-up: barriers, TMEM, the first unit's B rows (all threads)
    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; s++) {
            mbar_init(&bars.full[s], 1);
            mbar_init(&bars.empty[s], 8);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(&bars.sfull[s], 1);
            mbar_init(&bars.sempty[s], 8);
            mbar_init(&bars.dfull[s], 1);
            mbar_init(&bars.dempty[s], 4);
        }
        for (int s = 0; s < TM_NA; s++) {
            mbar_init(&bars.afull[s], 8);
            mbar_init(&bars.aempty[s], 1);
        }
        mbar_init(&bars.bready, 1);
        mbar_init(&bars.fin, 1);
        fence_mbar_init();
    }
    for (int64_t i = threadIdx.x; i < (int64_t)xsb_bytes / 16; i += blockDim.x)
        reinterpret_cast<uint4 *>(xsb)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();
    {
        const float *rows[8];
        int nrow;
        if (MODE == TM_GATEUP) {
            nrow = a.n_tok;
            for (int j = 0; j < nrow; j++) rows[j] = a.xb + (int64_t)j * L.hidden;
        } else {
            if (threadIdx.x == 0) s_ne[0] = slots_of(unit_of(u0).aux, s_slots[0]);
            __syncthreads();
            nrow = s_ne[0];
            for (int j = 0; j < nrow; j++) rows[j] = a.h + (int64_t)s_slots[0][j] * L.ffn;
        }
        tm_stage_rows(rows, nrow, K, xsb, threadIdx.x, blockDim.x);
    }
    fence_proxy_async_smem();
    if (warp == 1) tmem_alloc(&bars.tmem, TM_TCOLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars.tmem;
    bool failed = false;
    auto wait_b = [&](uint64_t *bar, uint32_t par) {  // one lane waits; the warp agrees
        bool ok = true;
        if (!failed) {
            if (lane == 0) ok = mbar_wait(bar, par);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) atomicExch(t.err, TM_ERR);
                failed = true;
            }
        }
        return !failed;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int64_t it = 0;
            for (int64_t u = u0; u < u1 && !failed; u++) {
                const TmUnit<MODE> ui = unit_of(u);
                const int el = msh.list[ui.aux];
                const uint8_t *eb = a.experts_layer + (int64_t)el * L.expert_stride;
                if (t.ssb) {
                    const int64_t j = u - u0;
                    const int slot = (int)(j & 1);
                    if (j >= 2 && !mbar_wait(&bars.sempty[slot], (uint32_t)(((j >> 1) - 1) & 1))) {
                        failed = true;
                        break;
                    }
                    uint8_t *dst = ss + (size_t)slot * t.ssb;
                    if (MODE == TM_GATEUP) {
                        const int64_t nr = min((int64_t)64, M - ui.tile * 64);
                        const uint32_t n = round16((uint32_t)(nr * gpr));
                        mbar_arrive_expect_tx(&bars.sfull[slot], 2 * n);
                        bulk_g2s(dst, eb + L.off[0][1] + ui.tile * 64 * gpr, n, &bars.sfull[slot]);
                        bulk_g2s(dst + 64 * gpr, eb + L.off[1][1] + ui.tile * 64 * gpr, n, &bars.sfull[slot]);
                    } else {
                        const int64_t nr = min((int64_t)128, M - ui.tile * 128);
                        const uint32_t n = round16((uint32_t)(nr * gpr));
                        mbar_arrive_expect_tx(&bars.sfull[slot], n);
                        bulk_g2s(dst, eb + L.off[2][1] + ui.tile * 128 * gpr, n, &bars.sfull[slot]);
                    }
                }
                for (int64_t b = ui.b0; b < ui.b1; b += SW_SEGB, it++) {
                    const int s = (int)(it % nst);
                    if (it >= nst && !mbar_wait(&bars.empty[s], (uint32_t)(((it / nst) - 1) & 1))) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_expect_tx(&bars.full[s], SW_STAGE_BYTES);
                    uint8_t *dst = ring + (size_t)s * SW_STAGE_BYTES;
                    if (MODE == TM_GATEUP) {
                        tma_box_4d(dst, &maps.m[0], (int)b, (int)(ui.tile * 64), el, a.layer, &bars.full[s]);
                        tma_box_4d(dst + 64 * 128, &maps.m[1], (int)b, (int)(ui.tile * 64), el, a.layer, &bars.full[s]);
                    } else {
                        tma_box_4d(dst, &maps.m[2], (int)b, (int)(ui.tile * 128), el, a.layer, &bars.full[s]);
                    }
                }
            }
            if (failed) atomicExch(t.err, TM_ERR);
            // every copy issued has landed before the CTA may exit
            for (int64_t k = it - 1; k >= 0 && k >= it - nst; k--)
                if (!mbar_wait(&bars.full[k % nst], (uint32_t)((k / nst) & 1))) atomicExch(t.err, TM_ERR);
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = umma_idesc_f16(128, TM_N);
            const uint32_t xsb_a = smem_u32(xsb);
            int64_t it = 0;
            int restages = 0;
            int prev_aux = -1;
            for (int64_t u = u0; u < u1; u++) {
                const TmUnit<MODE> ui = unit_of(u);
                const int64_t j = u - u0;
                const int d = (int)(j & 1);
                if (!failed && j >= 2 && !mbar_wait(&bars.dempty[d], (uint32_t)(((j >> 1) - 1) & 1))) failed = true;
                if (MODE == TM_DOWN && prev_aux >= 0 && ui.aux != prev_aux) {  // new expert: wait for its B rows
                    if (!failed && !mbar_wait(&bars.bready, (uint32_t)(restages & 1))) failed = true;
                    restages++;
                }
                prev_aux = ui.aux;
                bool first = true;
                for (int64_t b = ui.b0; b < ui.b1; b += SW_SEGB, it++) {
                    const int ab = (int)(it % TM_NA);
                    if (!failed && !mbar_wait(&bars.afull[ab], (uint32_t)((it / TM_NA) & 1))) failed = true;
                    tc_fence_after();
                    const int nb = (int)min((int64_t)SW_SEGB, ui.b1 - b);
                    const int64_t kg0 = DT == MG_Q8R ? b : 2 * b;     // first K column of the stage
                    const int kcount = DT == MG_Q8R ? nb : 2 * nb;     // K columns in the stage
                    if (!failed) {
                        for (int jj = 0; jj < kcount / 16; jj++) {
                            const int64_t kg = kg0 + 16 * jj;
                            const uint32_t bad = xsb_a + (uint32_t)((kg / 64) * 2048 + ((kg % 64) / 16) * 32);
                            tc_mma_f16_ts(tmem + TM_D0 + d * TM_N, tmem + ab * TM_ACOLS + jj * 8,
                                          umma_desc_sw128(bad), idesc, first ? 0u : 1u);
                            first = false;
                        }
                    }
                    tc_commit(&bars.aempty[ab]);  // the A buffer is free once these MMAs have read it
                }
                tc_commit(&bars.dfull[d]);
            }
            tc_commit(&bars.fin);
            if (!mbar_wait(&bars.fin, 0)) failed = true;
            if (failed) atomicExch(t.err, TM_ERR);
        }
    } else if (warp < TM_EPI0) {
        // ---------------------------------------------------------- converters
        const int q = warp & 3, kh = (warp - TM_CONV0) >> 2;
        const int r = 32 * q + lane;  // stage row = TMEM lane
        const uint32_t tl = tmem + ((uint32_t)(32 * q) << 16);
        int64_t it = 0;
        for (int64_t u = u0; u < u1; u++) {
            const TmUnit<MODE> ui = unit_of(u);
            const int el = msh.list[ui.aux];
            const int slot = (int)((u - u0) & 1);
            // this lane's output row, its validity, scale row and rebase
            int64_t orow;
            int mat;
            if (MODE == TM_GATEUP) {
                orow = ui.tile * 64 + (r & 63);
                mat = r < 64 ? 0 : 1;
            } else {
                orow = ui.tile * 128 + r;
                mat = 2;
            }
            const bool valid = orow < M;
            int rb = 0;
            const uint8_t *srow = nullptr;
            if (DT == MG_MXFP4) {
                rb = t.rebase[el * 3 + mat];
                if (t.ssb) {
                    wait_b(&bars.sfull[slot], (uint32_t)(((u - u0) >> 1) & 1));
                    srow = ss + (size_t)slot * t.ssb + (MODE == TM_GATEUP ? (r < 64 ? 0 : 64 * gpr) + (r & 63) * gpr
                                                                          : (int64_t)r * gpr);
                }
            }
            for (int64_t b = ui.b0; b < ui.b1; b += SW_SEGB, it++) {
                const int s = (int)(it % nst), ab = (int)(it % TM_NA);
                wait_b(&bars.full[s], (uint32_t)((it / nst) & 1));
                const uint8_t *st = ring + (size_t)s * SW_STAGE_BYTES + r * 128;
                uint4 raw[4];
#pragma unroll
                for (int p = 0; p < 4; p++) {
                    const int piece = 4 * kh + p;
                    raw[p] = *reinterpret_cast<const uint4 *>(st + ((piece ^ (r & 7)) << 4));
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars.empty[s]);  // the raw stage is in registers
                uint32_t v[32];
                if (DT == MG_Q8R) {
#pragma unroll
                    for (int p = 0; p < 4; p++) {
                        s8x4_to_h2(raw[p].x, v[8 * p + 0], v[8 * p + 1]);
                        s8x4_to_h2(raw[p].y, v[8 * p + 2], v[8 * p + 3]);
                        s8x4_to_h2(raw[p].z, v[8 * p + 4], v[8 * p + 5]);
                        s8x4_to_h2(raw[p].w, v[8 * p + 6], v[8 * p + 7]);
                    }
                    if (it >= TM_NA) wait_b(&bars.aempty[ab], (uint32_t)(((it / TM_NA) - 1) & 1));
                    if (!failed) tmem_st32(tl + ab * TM_ACOLS + kh * 32, v);
                } else {
                    // two passes of two 16-byte pieces (64 values = 32 columns each)
                    if (it >= TM_NA) wait_b(&bars.aempty[ab], (uint32_t)(((it / TM_NA) - 1) & 1));
#pragma unroll
                    for (int half = 0; half < 2; half++) {
#pragma unroll
                        for (int pp = 0; pp < 2; pp++) {
                            const int p = 2 * half + pp;
                            const int64_t grp = b / 16 + 4 * kh + p;  // 32 values per 16-byte piece
                            uint32_t f = 0u;
                            if (valid && srow) {
                                const uint32_t code = srow[grp];
                                f = code ? pow2_h2((int)code - 127 - rb) : 0u;
                            }
                            const uint32_t w4[4] = {raw[p].x, raw[p].y, raw[p].z, raw[p].w};
#pragma unroll
                            for (int wd = 0; wd < 4; wd++) {
                                uint32_t o[4];
                                e2m1x8_to_h2(w4[wd], o);
#pragma unroll
                                for (int i = 0; i < 4; i++) v[16 * pp + 4 * wd + i] = hmul2_u32(o[i], f);
                            }
                        }
                        if (!failed) tmem_st32(tl + ab * TM_ACOLS + kh * 64 + half * 32, v);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars.afull[ab]);
            }
            if (t.ssb) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars.sempty[slot]);
            }
        }
    } else {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;
        const int r = 32 * q + lane;
        const int etid = threadIdx.x - TM_EPI0 * 32;  // 0..127
        int restages = 0;
        for (int64_t u = u0; u < u1; u++) {
            const TmUnit<MODE> ui = unit_of(u);
            const int el = msh.list[ui.aux];
            const int eg = el + a.e0;
            const uint8_t *eb = a.experts_layer + (int64_t)el * L.expert_stride;
            const int64_t j = u - u0;
            const int d = (int)(j & 1);
            int64_t orow;
            int mat;
            if (MODE == TM_GATEUP) {
                orow = ui.tile * 64 + (r & 63);
                mat = r < 64 ? 0 : 1;
            } else {
                orow = ui.tile * 128 + r;
                mat = 2;
            }
            const bool valid = orow < M;
            float scale = 1.f, bias = 0.f;
            if (valid) {  // loaded before the wait for D
                if (DT == MG_Q8R) scale = reinterpret_cast<const float *>(eb + L.off[mat][1])[orow];
                else scale = exp2f((float)t.rebase[el * 3 + mat]);
                if (MODE == TM_GATEUP || ui.ks == 0) bias = reinterpret_cast<const float *>(eb + L.off[mat][2])[orow];
            }
            // the B rows' owners: tokens (gate/up) or this expert's slots (down)
            int slot_of[8];
            int nrow;
            if (MODE == TM_GATEUP) {
                nrow = a.n_tok;
                for (int tk = 0; tk < 8; tk++) {
                    slot_of[tk] = -1;
                    if (tk < a.n_tok)
                        for (int i = 0; i < a.top_k; i++)
                            if (a.sel[tk * a.top_k + i] == eg) { slot_of[tk] = tk * a.top_k + i; break; }
                }
            } else {
                int sl[8];
                nrow = slots_of(ui.aux, sl);
                for (int k = 0; k < 8; k++) slot_of[k] = k < nrow ? sl[k] : -1;
            }
            wait_b(&bars.dfull[d], (uint32_t)((j >> 1) & 1));
            tc_fence_after();
            float acc[16];
            tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + TM_D0 + d * TM_N, acc);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.dempty[d]);
            float val[8];
#pragma unroll
            for (int k = 0; k < 8; k++) val[k] = __fadd_rn(__fmul_rn(__fadd_rn(acc[2 * k], acc[2 * k + 1]), scale), bias);
            if (MODE == TM_GATEUP) {
                if (r >= 64)
                    for (int k = 0; k < 8; k++) upbuf[(r - 64) * 8 + k] = val[k];
                named_bar_sync(2, 128);
                if (r < 64 && valid && !failed) {
                    for (int k = 0; k < nrow; k++) {
                        if (slot_of[k] < 0) continue;
                        float g = val[k], uu = upbuf[r * 8 + k], hv;
                        if (a.act_plain) {
                            hv = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), uu);
                        } else {
                            if (g > a.limit) g = a.limit;
                            if (uu > a.limit) uu = a.limit;
                            if (uu < -a.limit) uu = -a.limit;
                            hv = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(__fmul_rn(-a.alpha, g)))), __fadd_rn(uu, 1.0f));
                        }
                        a.h[(int64_t)slot_of[k] * L.ffn + orow] = hv;
                    }
                }
                named_bar_sync(2, 128);  // upbuf is read before the next unit writes it
            } else {
                if (valid && !failed)
                    for (int k = 0; k < nrow; k++)
                        a.y[((int64_t)ui.ks * a.n_tok * a.top_k + slot_of[k]) * L.hidden + orow] = val[k];
                // the next unit belongs to another expert: its B rows replace these once every MMA
                // reading them is done (D of this unit is full, so they are)
                if (u + 1 < u1 && unit_of(u + 1).aux != ui.aux) {
                    if (etid == 0) s_ne[1] = slots_of(unit_of(u + 1).aux, s_slots[1]);
                    named_bar_sync(2, 128);
                    const float *rows[8];
                    const int n2 = s_ne[1];
                    for (int k = 0; k < n2; k++) rows[k] = a.h + (int64_t)s_slots[1][k] * L.ffn;
                    tm_stage_rows(rows, n2, K, xsb, etid, 128);
                    // rows of the old expert beyond n2 still hold data: their D columns are not read
                    fence_proxy_async_smem();
                    named_bar_sync(2, 128);
                    if (etid == 0) mbar_arrive(&bars.bready);
                    restages++;
                }
            }
        }
        (void)restages;
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, TM_TCOLS);
}

// ------------------------------------------------------------------ host side
bool tmoe_supported(const mg_expert_layout &L, const int *rebase) {
    if (L.dt == MG_MXFP4) return L.scale_fmt == MG_SCALE_UE8M0 && rebase && L.hidden % 64 == 0 && L.ffn % 64 == 0;
    return L.dt == MG_Q8R && L.hidden % 128 == 0 && L.ffn % 128 == 0;
}

template <int DT, int MODE>
static int launch_tmoe(const MoeStreamArgs &a, const int *rebase, int ks, int64_t kbps, cudaStream_t st) {
    const int64_t K = MODE == TM_GATEUP ? a.L.hidden : a.L.ffn;
    const int64_t gpr = K / 32;
    const size_t ssb = DT == MG_MXFP4 ? (((MODE == TM_GATEUP ? 128 : 128) * (size_t)gpr + 127) & ~(size_t)127) : 0;
    const size_t xsb = (size_t)((K + 63) / 64) * 2048;
    const size_t fixed = 1024 + xsb + 2 * ssb + 64 * 8 * 4;
    const size_t budget = 227 * 1024 - 2048;  // static shared memory
    MG_REQUIRE(budget > fixed + 2 * (size_t)SW_STAGE_BYTES, MG_ERR_ARG, "tensor-core MoE: activations too large");
    int nst = (int)((budget - fixed) / SW_STAGE_BYTES);
    if (nst > 8) nst = 8;
    const size_t smem = fixed + (size_t)nst * SW_STAGE_BYTES;
    auto kfn = k_tmoe<DT, MODE>;
    int rc = ensure_smem_attr(reinterpret_cast<const void *>(kfn), smem);
    if (rc) return rc;
    SwMaps maps;
    for (int i = 0; i < 3; i++) maps.m[i] = a.maps[i];
    TmArgs t{};
    t.a = a;
    t.rebase = rebase;
    t.ks_count = ks;
    t.kbytes_per_split = kbps;
    t.nstages = nst;
    t.ssb = (int)ssb;
    t.err = stream_error_word();
    MG_REQUIRE(t.err, MG_ERR_OOM, "tensor-core MoE: no error word");
    kfn<<<num_sms(), TM_THREADS, smem, st>>>(maps, t);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int moe_tmoe(const MoeStreamArgs &a, const int *rebase, cudaStream_t st) {
    MG_REQUIRE(a.n_tok >= 1 && a.n_tok <= 8 && a.n_tok * a.top_k <= SW_MAX_SLOTS && a.n_experts <= 2048 && a.maps,
               MG_ERR_ARG, "tensor-core MoE: n_tok %d top_k %d unsupported", a.n_tok, a.top_k);
    MG_REQUIRE(tmoe_supported(a.L, rebase), MG_ERR_ARG, "tensor-core MoE: expert format unsupported");
    const int ks = moe_down_ksplit(a.L, a.down_ksplit);
    MG_REQUIRE(ks == a.down_ksplit_out, MG_ERR_ARG, "tensor-core MoE: down K split %d != caller's %d", ks,
               a.down_ksplit_out);
    const int64_t rb_dn = a.L.dt == MG_Q8R ? a.L.ffn : a.L.ffn / 2;
    const int64_t nseg = (rb_dn + SW_SEGB - 1) / SW_SEGB;
    const int64_t kbps = ((nseg + ks - 1) / ks) * SW_SEGB;
    int rc;
    if (a.L.dt == MG_MXFP4) {
        rc = launch_tmoe<MG_MXFP4, TM_GATEUP>(a, rebase, 1, 0, st);
        if (rc) return rc;
        return launch_tmoe<MG_MXFP4, TM_DOWN>(a, rebase, ks, kbps, st);
    }
    rc = launch_tmoe<MG_Q8R, TM_GATEUP>(a, rebase, 1, 0, st);
    if (rc) return rc;
    return launch_tmoe<MG_Q8R, TM_DOWN>(a, rebase, ks, kbps, st);
}

}  // namespace mg

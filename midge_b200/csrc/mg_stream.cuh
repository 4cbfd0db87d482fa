// mg_stream.cuh -- warp-specialized streamed dequant-GEMV for decode.
//
// One CTA = 16 consumer warps + 1 producer warp.  The producer streams weight
// rows into a ring of shared-memory stages with cp.async.bulk (one bulk copy
// per row segment, completion counted on an mbarrier); the consumers decode
// and multiply out of shared memory on the tensor cores (mma.sync, f16 hi/lo
// activations, f32 accumulation) and hand each stage back through a second
// mbarrier.  Memory parallelism is therefore set by the ring depth, not by
// registers.
//
// A stage holds 128 "MMA rows" (8 row groups of 16) x up to SEGB bytes of
// each row.  Work is a list of units; a unit is a tile of MMA rows times a
// range of each row's bytes (a K split), streamed as consecutive segments.
// Two consumer warps share a row group and take the unit's stages in turn
// (more warps per scheduler to hide the decode and MMA latencies); at the
// end of a unit the second warp hands its sums to the first through shared
// memory and the first runs the policy's epilogue.
//
// Every wait is bounded; on timeout a kernel records an error code and stops.
#pragma once
#include "mg_common.cuh"
#include <cuda.h>

#include "mg_gemv.cuh"

namespace mg {

constexpr int SW_RG = 8;                      // row groups of 16 MMA rows per stage
constexpr int SW_KH = 2;                      // consumer warps per row group (taking alternate stages)
constexpr int SW_CONS = SW_RG * SW_KH;        // consumer warps
constexpr int SW_THREADS = (SW_CONS + 1) * 32;
constexpr int SW_ROWS = SW_RG * 16;           // MMA rows per stage
constexpr int SW_BAR_PAIR0 = 4;               // named barriers 4..11: the two warps of a row group
constexpr int SW_RED_BYTES = SW_RG * 32 * 8 * 4;  // hand-over of partial sums (NT <= 2)
constexpr int SW_MAX_STAGES = 12;
constexpr int SW_ERR_TIMEOUT = 1;
constexpr int SW_SCALE_SLOTS = 8;
// per-unit scale slots: 4-bit weights carry the tile's group scales (tens of
// KB: two slots); int8 only its row scales and biases (1 KB: eight, so that
// the producer runs as far ahead as the ring allows)
__host__ __device__ constexpr int sw_nslot(int dt) { return dt == MG_Q8R ? SW_SCALE_SLOTS : 2; }
constexpr int SW_SEGB = 128;                  // bytes of each row per stage: one 128-byte swizzle row
constexpr int SW_STAGE_BYTES = SW_ROWS * SW_SEGB;  // 16 KB: one TMA box of 128 rows x 128 B

template <int DT>
struct SwGeom {
    static constexpr int CB = DT == MG_Q8R ? 64 : 16;    // bytes of one chunk of one row
    static constexpr int COLS_PER_CHUNK = DT == MG_Q8R ? 64 : 32;
};

// byte address of 16-byte piece `p` (0..7) of stage row `r` (128-byte swizzle:
// piece p of row r lives at piece p ^ (r % 8))
__device__ __forceinline__ uint32_t sw_addr(int r, int p) { return (uint32_t)(r * 128 + ((p ^ (r & 7)) << 4)); }

// Up to three tensor maps per launch, passed as __grid_constant__ so that TMA
// reads them from parameter space.
struct SwMaps {
    CUtensorMap m[3];
};

// Shared-memory bookkeeping common to all streamed kernels.
struct SwShared {
    uint64_t full[SW_MAX_STAGES];
    uint64_t empty[SW_MAX_STAGES];
    uint64_t sfull[SW_SCALE_SLOTS], sempty[SW_SCALE_SLOTS];  // the per-unit scale slots (sw_nslot of them)
};

// Group scales of 4-bit weights: when the launch gives scale slots (ssb > 0),
// the producer bulk-copies each unit's scales into one of two shared-memory
// slots ahead of its weight stages, so the consumers never wait on a global
// load inside a stage.  sb = bytes per scale (1 for ue8m0, 2 for f16).
template <int SC>
__device__ __forceinline__ float scale_at(const uint8_t *p) {
    if (SC == MG_SCALE_UE8M0) return ue8m0_to_f32(*p);
    return h2f(*reinterpret_cast<const uint16_t *>(p));
}
__device__ __forceinline__ uint32_t round16(uint32_t v) { return (v + 15u) & ~15u; }
// row group of the calling consumer warp
__device__ __forceinline__ int sw_rg() { return (threadIdx.x >> 5) & (SW_RG - 1); }

struct UnitInfo {
    int64_t tile;
    int ks;
    int64_t b0, b1;  // byte range of every row handled by this unit
    int aux;          // policy-defined (e.g. expert index)
};

// -------------------------------------------------------------- producer
// Policy interface (device):
//   int64_t units() const;  void unit(int64_t u, UnitInfo &ui) const;
//   void issue(const SwMaps &, const UnitInfo &, int64_t b, void *dst, uint64_t *bar) const
//     -- issues the TMA boxes of row bytes [b, b+128) of the unit's rows into dst
template <int DT, class P>
__device__ void sw_producer(const P &pol, const SwMaps &maps, int64_t u0, int64_t u1, uint8_t *ring, int nstages,
                            uint8_t *ss, int ssb, SwShared *sh, int *err) {
    if ((threadIdx.x & 31) != 0) return;
    int64_t it = 0, nu = 0;  // stages and scale slots issued
    int s = 0;               // it % nstages
    uint32_t ph = 0;         // (it / nstages) & 1
    bool ok = true;
    for (int64_t u = u0; u < u1 && ok; u++) {
        UnitInfo ui;
        pol.unit(u, ui);
        if (ssb) {
            const int64_t j = u - u0;
            constexpr int NS = sw_nslot(DT);
            const int slot = (int)(j % NS);
            if (j >= NS && !mbar_wait(&sh->sempty[slot], (uint32_t)(((j / NS) - 1) & 1))) {
                ok = false;
                break;
            }
            mbar_arrive_expect_tx(&sh->sfull[slot], pol.scale_bytes(ui));
            pol.issue_scales(ui, ss + (size_t)slot * ssb, &sh->sfull[slot]);
            nu = j + 1;
        }
        for (int64_t b = ui.b0; b < ui.b1; b += SW_SEGB, it++) {
            if (it >= nstages && !mbar_wait(&sh->empty[s], ph ^ 1u)) {
                ok = false;
                break;
            }
            mbar_arrive_expect_tx(&sh->full[s], SW_STAGE_BYTES);
            pol.issue(maps, ui, b, ring + (size_t)s * SW_STAGE_BYTES, &sh->full[s]);
            if (++s == nstages) { s = 0; ph ^= 1u; }
        }
    }
    if (!ok) atomicExch(err, SW_ERR_TIMEOUT);
    // every copy issued has landed before the CTA may exit (already true on
    // success: the consumers waited for all of them)
    for (int64_t k = it - 1; k >= 0 && k >= it - nstages; k--)
        if (!mbar_wait(&sh->full[k % nstages], (uint32_t)((k / nstages) & 1))) atomicExch(err, SW_ERR_TIMEOUT);
    constexpr int NS = sw_nslot(DT);
    for (int64_t j = nu - 1; j >= 0 && j >= nu - NS; j--)
        if (!mbar_wait(&sh->sfull[j % NS], (uint32_t)((j / NS) & 1))) atomicExch(err, SW_ERR_TIMEOUT);
}

// -------------------------------------------------------------- consumer
// Activation row stride (halves) of the streamed kernels, chosen so that the
// 16-byte activation loads of a quarter-warp (rows g, g+1, 4 lanes t each)
// fall in distinct bank groups: row stride = 64 B mod 128 for the 4-bit
// layout (lanes t at 16 t), 16 B mod 32 for int8 (lanes t at 32 t).
template <int DT>
__host__ __device__ __forceinline__ int sw_xs_stride(int64_t cols) {
    return (int)(((cols + 63) / 64) * 64 + (DT == MG_Q8R ? 8 : 32));
}

__device__ __forceinline__ void mma_16816_z(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}

// Per-lane constants of a consumer warp, fixed for the kernel: the byte
// offsets (within a stage) of the lane's two MMA rows ra = stage_row(w, g),
// rb = stage_row(w, g + 8), pre-XORed with their swizzle keys so that chunk c
// is at off ^ (c << 4) (4-bit: 16-byte chunks, lane word 4t) or off ^ (c << 6)
// (int8: 64-byte chunks, lane piece 4c + t); and the lane's activation byte
// offset (row g of the staged activations, column piece t).
struct SwLane {
    uint32_t offA, offB, xoff;
};

template <int DT, class P>
__device__ __forceinline__ SwLane sw_lane(const P &pol, int w, int xs_stride) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const int ra = pol.stage_row(w, g), rb = pol.stage_row(w, g + 8);
    SwLane L;
    if (DT == MG_Q8R) {
        L.offA = (uint32_t)(ra * 128 + (((t ^ (ra & 7))) << 4));
        L.offB = (uint32_t)(rb * 128 + (((t ^ (rb & 7))) << 4));
        L.xoff = (uint32_t)(g * xs_stride * 2 + 32 * t);
    } else {
        L.offA = (uint32_t)((ra * 128 + 4 * t) ^ ((ra & 7) << 4));
        L.offB = (uint32_t)((rb * 128 + 4 * t) ^ ((rb & 7) << 4));
        L.xoff = (uint32_t)(g * xs_stride * 2 + 16 * t);
    }
    return L;
}

// One warp's pass over one stage: its row group's 16 MMA rows times the
// stage's bytes [b, b + nbytes) of each row (all chunks when FULL), for the
// first NTA of the NT token groups.
//   st: the stage; xs8: staged activations (bytes); xo[nt]: the lane's byte
//   offset in xs8 of token group nt (its activation row, column piece t);
//   pa, pb: the lane's rows' scales in the unit's scale slot (4-bit, SS).
template <int DT, int SC, int NT, int NTA, bool FULL, bool SS, class P>
__device__ __forceinline__ void sw_stage(const P &pol, const UnitInfo &ui, const SwLane &ln, const uint8_t *st,
                                         int64_t b, int nbytes, const uint8_t *xs8, const uint32_t xo[NT],
                                         const uint8_t *pa, const uint8_t *pb, float acc[NT][4]) {
    using G = SwGeom<DT>;
    constexpr int CPS = SW_SEGB / G::CB;  // chunks per stage
    const int nch = FULL ? CPS : nbytes / G::CB;
    const int lane = threadIdx.x & 31, g = lane >> 2;
    if constexpr (DT == MG_Q8R) {
        const uint8_t *xb = xs8 + b * 2;  // column b (1 byte per column), 2 bytes per half
#pragma unroll
        for (int c = 0; c < CPS; c++) {
            if (!FULL && c >= nch) break;
            const uint4 wa = *reinterpret_cast<const uint4 *>(st + (ln.offA ^ (c << 6)));
            const uint4 wb = *reinterpret_cast<const uint4 *>(st + (ln.offB ^ (c << 6)));
            const uint32_t wav[4] = {wa.x, wa.y, wa.z, wa.w}, wbv[4] = {wb.x, wb.y, wb.z, wb.w};
            uint32_t fa[4][4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                s8x4_to_h2(wav[q], fa[q][0], fa[q][2]);
                s8x4_to_h2(wbv[q], fa[q][1], fa[q][3]);
            }
#pragma unroll
            for (int nt = 0; nt < NTA; nt++) {
                const uint8_t *xp = xb + xo[nt] + c * 128;
                const uint4 x0 = *reinterpret_cast<const uint4 *>(xp);
                const uint4 x1 = *reinterpret_cast<const uint4 *>(xp + 16);
                const uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int q = 0; q < 4; q++) mma_16816(acc[nt], fa[q], bx[2 * q], bx[2 * q + 1]);
            }
        }
    } else {
        constexpr int SB = SC == MG_SCALE_UE8M0 ? 1 : 2;
        const int64_t gchunk0 = b / G::CB;          // group index of the stage's first chunk
        const uint8_t *xb = xs8 + b * 4;   // column 2b, 2 bytes per half
        const uint8_t *psa = SS ? pa + gchunk0 * SB : nullptr, *psb = SS ? pb + gchunk0 * SB : nullptr;
#pragma unroll
        for (int c = 0; c < CPS; c++) {
            if (!FULL && c >= nch) break;
            const uint32_t wa = *reinterpret_cast<const uint32_t *>(st + (ln.offA ^ (c << 4)));
            const uint32_t wb = *reinterpret_cast<const uint32_t *>(st + (ln.offB ^ (c << 4)));
            const float sa = SS ? scale_at<SC>(psa + c * SB) : pol.scale(ui, g, gchunk0 + c);
            const float sb = SS ? scale_at<SC>(psb + c * SB) : pol.scale(ui, g + 8, gchunk0 + c);
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
            for (int nt = 0; nt < NTA; nt++) {
                const uint4 bx = *reinterpret_cast<const uint4 *>(xb + xo[nt] + c * 64);
                float d[4];
                mma_16816_z(d, a0, bx.x, bx.y);
                mma_16816(d, a1, bx.z, bx.w);
                acc[nt][0] = fmaf(sa, d[0], acc[nt][0]);
                acc[nt][1] = fmaf(sa, d[1], acc[nt][1]);
                acc[nt][2] = fmaf(sb, d[2], acc[nt][2]);
                acc[nt][3] = fmaf(sb, d[3], acc[nt][3]);
            }
        }
    }
}

// sw_stage with the unit's active token-group count and scale-slot use as
// compile-time constants (no per-chunk branches)
template <int DT, int SC, int NT, bool FULL, bool SS, class P>
__device__ __forceinline__ void sw_stage_nt(const P &pol, const UnitInfo &ui, const SwLane &ln, const uint8_t *st,
                                            int64_t b, int nbytes, const uint8_t *xs8, const uint32_t xo[NT],
                                            int nt_active, const uint8_t *pa, const uint8_t *pb, float acc[NT][4]) {
    if constexpr (NT >= 4)
        if (nt_active >= 4) return sw_stage<DT, SC, NT, 4, FULL, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, pa, pb, acc);
    if constexpr (NT >= 3)
        if (nt_active == 3) return sw_stage<DT, SC, NT, 3, FULL, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, pa, pb, acc);
    if constexpr (NT >= 2)
        if (nt_active == 2) return sw_stage<DT, SC, NT, 2, FULL, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, pa, pb, acc);
    sw_stage<DT, SC, NT, 1, FULL, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, pa, pb, acc);
}

template <int DT, int SC, int NT, bool SS, class P>
__device__ __forceinline__ void sw_stage_any(const P &pol, const UnitInfo &ui, const SwLane &ln, const uint8_t *st,
                                             int64_t b, int nbytes, const uint8_t *xs8, const uint32_t xo[NT],
                                             int nt_active, const uint8_t *pa, const uint8_t *pb, float acc[NT][4]) {
    if (nbytes == SW_SEGB)
        sw_stage_nt<DT, SC, NT, true, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, nt_active, pa, pb, acc);
    else
        sw_stage_nt<DT, SC, NT, false, SS>(pol, ui, ln, st, b, nbytes, xs8, xo, nt_active, pa, pb, acc);
}

// Default activation rows of the consumers: token group nt is staged rows
// 8 nt .. 8 nt + 7 (token 4 nt + r/2, half r%2)
template <int NT>
__device__ __forceinline__ void sw_x_rows(const SwLane &ln, uint32_t xs8_nt, uint32_t xo[NT]) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) xo[nt] = ln.xoff + nt * xs8_nt;
}

// Consumer warps.  The two warps of a row group take a unit's stages in
// turn (warp kh takes the stages whose running index has parity kh), each
// accumulating its row group's sums; at the end of the unit the second warp
// hands its sums to the first, which runs the policy epilogue.
template <int DT, int SC, int NT, class P>
__device__ __forceinline__ void sw_consumers(P &pol, int64_t u0, int64_t u1, uint8_t *ring, int nstages,
                                             uint8_t *ss_base, int ssb, float *red, SwShared *sh, __half *xs,
                                             int xs_stride, int *err) {
    const int lane = threadIdx.x & 31, w = sw_rg(), kh = (threadIdx.x >> 5) / SW_RG;
    const int g = lane >> 2;
    const SwLane ln = sw_lane<DT>(pol, w, xs_stride);
    const uint8_t *xs8 = reinterpret_cast<const uint8_t *>(xs);
    const uint32_t xs8_nt = (uint32_t)(8 * xs_stride * 2);
    uint32_t it = 0;  // running stage index (its parity picks the warp)
    int s = 0;        // it % nstages
    uint32_t ph = 0;  // (it / nstages) & 1
    // After a timed-out wait a warp stops waiting and computing but keeps
    // taking part in the named barriers, so no other warp is left waiting.
    bool failed = false;
    for (int64_t u = u0; u < u1; u++) {
        if (pol.restage(u, u0)) {
            named_bar_sync(1, SW_CONS * 32);  // everyone is done with the old activations
            pol.stage_x(u, xs, xs_stride);
            named_bar_sync(1, SW_CONS * 32);
        }
        UnitInfo ui;
        pol.unit(u, ui);
        uint32_t xo[NT];
        const int nt_active = pol.template x_rows<NT>(ui, ln, xs8_nt, xs_stride, xo);
        float acc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
        const bool live = pol.warp_live(ui, w);
        const uint8_t *pa = nullptr, *pb = nullptr;
        constexpr int NS = sw_nslot(DT);
        const int slot = (int)((u - u0) % NS);
        if (ssb && !failed) {
            bool ok = true;
            if (lane == 0) ok = mbar_wait(&sh->sfull[slot], (uint32_t)(((u - u0) / NS) & 1));
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) atomicExch(err, SW_ERR_TIMEOUT);
                failed = true;
            }
            const uint8_t *ss = ss_base + (size_t)slot * ssb;
            pa = pol.scale_sm(ui, ss, g);
            pb = pol.scale_sm(ui, ss, g + 8);
        }
        for (int64_t b = ui.b0; b < ui.b1; b += SW_SEGB, it++) {
            const int sc = s;
            const uint32_t phc = ph;
            if (++s == nstages) { s = 0; ph ^= 1u; }
            if ((int)(it & 1u) != kh) continue;  // the other warp of the row group takes this stage
            if (!failed) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&sh->full[sc], phc);
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) {
                    if (lane == 0) atomicExch(err, SW_ERR_TIMEOUT);
                    failed = true;
                }
            }
            if (live && !failed) {
                const uint8_t *st = ring + (size_t)sc * SW_STAGE_BYTES;
                const int nbytes = (int)min((int64_t)SW_SEGB, ui.b1 - b);
                if (DT == MG_Q8R || pa)
                    sw_stage_any<DT, SC, NT, true>(pol, ui, ln, st, b, nbytes, xs8, xo, nt_active, pa, pb, acc);
                else
                    sw_stage_any<DT, SC, NT, false>(pol, ui, ln, st, b, nbytes, xs8, xo, nt_active, pa, pb, acc);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->empty[sc]);
        }
        if (live) {  // both warps of the row group agree on `live`
            float *rp = red + ((size_t)w * 32 + lane) * (NT * 4);
            if (kh == 1) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) rp[nt * 4 + i] = acc[nt][i];
            }
            named_bar_sync(SW_BAR_PAIR0 + w, 64);
            if (kh == 0) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                    for (int i = 0; i < 4; i++) acc[nt][i] += rp[nt * 4 + i];
                if (!failed) pol.template epilogue<NT>(ui, w, acc, ssb ? ss_base + (size_t)slot * ssb : nullptr);
            }
            named_bar_sync(SW_BAR_PAIR0 + w, 64);  // the sums are read before the next unit's overwrite them
        }
        if (ssb) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->sempty[slot]);
        }
    }
    pol.finish();  // all consumer threads
}

// The kernel shell: barrier setup, block's unit range, role split.
template <int DT, int SC, int NT, class P>
__global__ void __launch_bounds__(SW_THREADS, 1) k_stream(const __grid_constant__ SwMaps maps, P pol, int nstages,
                                                          int ssb, int *err) {
    extern __shared__ __align__(1024) uint8_t sw_smem_raw[];
    uint8_t *sw_smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(sw_smem_raw) + 1023) & ~(uintptr_t)1023);
    SwShared *sh = reinterpret_cast<SwShared *>(sw_smem);
    pdl_trigger();  // a programmatically launched next kernel may start its setup
    uint8_t *ring = sw_smem + 1024;  // stages 1024-aligned for the 128-byte swizzle
    uint8_t *ss = ring + (size_t)nstages * SW_STAGE_BYTES;  // sw_nslot scale slots of ssb bytes (ssb % 128 == 0)
    float *red = reinterpret_cast<float *>(ss + sw_nslot(DT) * (size_t)ssb);  // SW_RG x 32 lanes x NT*4 partial sums
    __half *xs = reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(red) + SW_RED_BYTES);
    const int xs_stride = pol.xs_stride();
    pol.init_shared();  // all threads; ends with __syncthreads
    const int64_t nunits = pol.units();
    const int64_t per = (nunits + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = (int64_t)blockIdx.x * per, u1 = min(nunits, u0 + per);
    if (threadIdx.x == 0) {
        for (int s = 0; s < nstages; s++) {
            mbar_init(&sh->full[s], 1);
            mbar_init(&sh->empty[s], SW_RG);  // the row-group warps that took the stage
        }
        for (int s = 0; s < sw_nslot(DT); s++) {
            mbar_init(&sh->sfull[s], 1);
            mbar_init(&sh->sempty[s], SW_CONS);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (u0 >= u1) return;
    const int w = threadIdx.x >> 5;
    if (w == SW_CONS) {
        sw_producer<DT>(pol, maps, u0, u1, ring, nstages, ss, ssb, sh, err);
    } else {
        pol.stage_x_units(u0, u1, xs, xs_stride);
        named_bar_sync(1, SW_CONS * 32);
        sw_consumers<DT, SC, NT>(pol, u0, u1, ring, nstages, ss, ssb, red, sh, xs, xs_stride, err);
    }
}

__device__ __forceinline__ void tma_box_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_box_4d(void *dst, const CUtensorMap *map, int x, int y, int z, int w,
                                           uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------- policies
// Plain GEMV over up to 3 row-concatenated matrices sharing cols and the
// activations; K split ks_count ways.  Unit = (tile of 128 rows of one
// matrix, K split).  maps.m[i] is matrix i as a 2-D byte tensor
// {row bytes, rows}.  Output: ks_count == 1 -> y = W x (+bias), stored or
// accumulated; else y + ks*part_stride holds split ks's partial sums (bias in
// split 0) for a later reduction.
struct GemvMat {
    const uint8_t *sc;
    const float *bias;
    int64_t rows;
    float *y;
    int64_t ldy;
    int64_t tile0;  // first tile index of this matrix
};

template <int DT, int SC>
struct PolGemv {
    GemvMat m[3];
    int nmat;
    int cols;
    int ks_count;
    int64_t kbytes_per_split;  // multiple of SW_SEGB
    int64_t ntiles;
    const float *x;
    int64_t ldx;
    int n_tok;
    int accumulate;
    int64_t part_stride;
    unsigned long long *amax;  // optional: per-token packed (value, -index) maximum of the outputs
    float bv[2];               // this lane's best output for tokens t and 4+t
    int bi[2];

    __device__ int64_t rowbytes() const { return DT == MG_Q8R ? cols : cols / 2; }
    __device__ int xs_stride() const { return sw_xs_stride<DT>(cols); }
    __device__ void init_shared() {
        bv[0] = bv[1] = -INFINITY;
        bi[0] = bi[1] = 0x7fffffff;
        __syncthreads();
    }
    // first maximum per token over everything this CTA produced, then one
    // 64-bit atomic max per token: key = ordered value << 32 | ~index
    __device__ void finish() {
        if (!amax) return;
        __shared__ float sv[SW_CONS][8];
        __shared__ int si[SW_CONS][8];
        const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, t = lane & 3;
#pragma unroll
        for (int nt = 0; nt < 2; nt++) {
            float v = bv[nt];
            int i = bi[nt];
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, i, o);
                if (ov > v || (ov == v && oi < i)) { v = ov; i = oi; }
            }
            if (lane < 4) { sv[w][nt * 4 + t] = v; si[w][nt * 4 + t] = i; }
        }
        named_bar_sync(1, SW_CONS * 32);
        if (threadIdx.x < n_tok && threadIdx.x < 8) {
            const int tok = threadIdx.x;
            float v = -INFINITY;
            int i = 0x7fffffff;
            for (int ww = 0; ww < SW_CONS; ww++)
                if (sv[ww][tok] > v || (sv[ww][tok] == v && si[ww][tok] < i)) { v = sv[ww][tok]; i = si[ww][tok]; }
            if (i != 0x7fffffff) {
                uint32_t u = __float_as_uint(v);
                u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
                atomicMax(&amax[tok], ((unsigned long long)u << 32) | (unsigned long long)(0xffffffffu - (uint32_t)i));
            }
        }
    }
    __device__ int64_t units() const { return ntiles * ks_count; }
    __device__ int mat_of(int64_t tile) const {
        int k = 0;
        if (nmat > 1 && tile >= m[1].tile0) k = 1;
        if (nmat > 2 && tile >= m[2].tile0) k = 2;
        return k;
    }
    __device__ void unit(int64_t u, UnitInfo &ui) const {
        // K-split-major: a CTA's consecutive units share a K split (and so the
        // activation columns it stages)
        ui.ks = (int)(u / ntiles);
        ui.tile = u - (int64_t)ui.ks * ntiles;
        ui.b0 = (int64_t)ui.ks * kbytes_per_split;
        ui.b1 = min(rowbytes(), ui.b0 + kbytes_per_split);
        ui.aux = mat_of(ui.tile);
    }
    // field of matrix i without dynamic indexing of the parameter array (which
    // would copy the policy to local memory)
#define MG_SEL(i, f) ((i) == 0 ? m[0].f : ((i) == 1 ? m[1].f : m[2].f))
    __device__ int64_t row0(const UnitInfo &ui) const { return (ui.tile - MG_SEL(ui.aux, tile0)) * SW_ROWS; }
    __device__ void issue(const SwMaps &maps, const UnitInfo &ui, int64_t b, void *dst, uint64_t *bar) const {
        tma_box_2d(dst, &maps.m[ui.aux], (int)b, (int)row0(ui), bar);
    }
    __device__ int stage_row(int w, int r16) const { return 16 * w + r16; }
    __device__ bool warp_live(const UnitInfo &ui, int w) const { return row0(ui) + 16 * w < MG_SEL(ui.aux, rows); }
    __device__ float scale(const UnitInfo &ui, int r16, int64_t grp) const {
        const int w = sw_rg();
        const int64_t row = row0(ui) + 16 * w + r16;
        if (row >= MG_SEL(ui.aux, rows)) return 0.f;
        const int64_t gpr = cols / 32;
        const uint8_t *sc = MG_SEL(ui.aux, sc);
        if (SC == MG_SCALE_UE8M0) return ue8m0_to_f32(__ldg(sc + row * gpr + grp));
        return h2f(__ldg(reinterpret_cast<const uint16_t *>(sc) + row * gpr + grp));
    }
    // Unit scales.  4-bit: the tile's rows' group scales, whole rows (every K
    // split reads all of them).  int8: the rows' f32 scales at +0 and, in K
    // split 0 of a matrix with a bias, the rows' biases at +SW_ROWS*4, read by
    // the epilogue from shared memory (the launch gives int8 slots only when
    // both arrays are 16-byte aligned and every matrix has rows % 4 == 0).
    static constexpr int SB = SC == MG_SCALE_UE8M0 ? 1 : 2;
    __device__ bool slot_bias(const UnitInfo &ui) const { return MG_SEL(ui.aux, bias) != nullptr && ui.ks == 0; }
    __device__ uint32_t scale_bytes(const UnitInfo &ui) const {
        const int64_t nr = min((int64_t)SW_ROWS, MG_SEL(ui.aux, rows) - row0(ui));
        if (DT == MG_Q8R) return (uint32_t)(nr * 4) * (slot_bias(ui) ? 2u : 1u);
        return round16((uint32_t)(nr * (cols / 32) * SB));
    }
    __device__ void issue_scales(const UnitInfo &ui, uint8_t *dst, uint64_t *bar) const {
        if (DT == MG_Q8R) {
            const int64_t nr = min((int64_t)SW_ROWS, MG_SEL(ui.aux, rows) - row0(ui));
            bulk_g2s(dst, reinterpret_cast<const float *>(MG_SEL(ui.aux, sc)) + row0(ui), (uint32_t)(nr * 4), bar);
            if (slot_bias(ui)) bulk_g2s(dst + SW_ROWS * 4, MG_SEL(ui.aux, bias) + row0(ui), (uint32_t)(nr * 4), bar);
            return;
        }
        bulk_g2s(dst, MG_SEL(ui.aux, sc) + row0(ui) * (cols / 32) * SB, scale_bytes(ui), bar);
    }
    __device__ const uint8_t *scale_sm(const UnitInfo &, const uint8_t *ss, int r16) const {
        const int w = sw_rg();
        return ss + (int64_t)(16 * w + r16) * (cols / 32) * SB;
    }
    template <int NT>
    __device__ int x_rows(const UnitInfo &, const SwLane &ln, uint32_t xs8_nt, int, uint32_t xo[NT]) const {
        sw_x_rows<NT>(ln, xs8_nt, xo);
        return (n_tok + 3) >> 2;
    }
    __device__ bool restage(int64_t, int64_t) const { return false; }
    __device__ void stage_x(int64_t, __half *xs, int xs_stride) const {
        stage_x_n<DT>(x, ldx, n_tok, cols, xs, xs_stride, threadIdx.x, SW_CONS * 32);
    }
    // only the columns of the K splits of units [u0, u1) (consecutive splits:
    // the units are K-split-major); split starts are multiples of 128 bytes
    __device__ void stage_x_units(int64_t u0, int64_t u1, __half *xs, int xs_stride) const {
        const int64_t b0 = (u0 / ntiles) * kbytes_per_split;
        const int64_t b1 = min(rowbytes(), ((u1 - 1) / ntiles + 1) * kbytes_per_split);
        const int c0 = (int)(DT == MG_Q8R ? b0 : 2 * b0), c1 = (int)(DT == MG_Q8R ? b1 : 2 * b1);
        stage_x_n<DT>(x + c0, ldx, n_tok, c1 - c0, xs + c0, xs_stride, threadIdx.x, SW_CONS * 32);
    }
    template <int NT>
    __device__ void epilogue(const UnitInfo &ui, int w, const float acc[NT][4], const uint8_t *ss) {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        const int64_t mrows = MG_SEL(ui.aux, rows), mldy = MG_SEL(ui.aux, ldy);
        const uint8_t *msc = MG_SEL(ui.aux, sc);
        const float *mbias = MG_SEL(ui.aux, bias);
        float *my = MG_SEL(ui.aux, y);
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int64_t row = row0(ui) + 16 * w + g + 8 * half;
            if (row >= mrows) continue;
            const int r = 16 * w + g + 8 * half;  // row within the tile
            float rs = 1.f, bias;
            if (DT == MG_Q8R && ss) {
                rs = reinterpret_cast<const float *>(ss)[r];
                bias = slot_bias(ui) ? reinterpret_cast<const float *>(ss + SW_ROWS * 4)[r] : 0.f;
            } else {
                if (DT == MG_Q8R) rs = reinterpret_cast<const float *>(msc)[row];
                bias = (mbias && ui.ks == 0) ? mbias[row] : 0.f;
            }
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int tok = nt * 4 + t;
                if (tok >= n_tok) continue;
                float v = acc[nt][2 * half] + acc[nt][2 * half + 1];
                if (DT == MG_Q8R) v *= rs;
                v += bias;
                if (ks_count == 1) {
                    float *yp = my + (int64_t)tok * mldy + row;
                    *yp = accumulate ? *yp + v : v;
                    if (amax && nt < 2 && (v > bv[nt] || (v == bv[nt] && (int)row < bi[nt]))) {  // NaN never wins
                        bv[nt] = v;
                        bi[nt] = (int)row;
                    }
                    // the reference's scan starts from element 0 and never replaces a NaN there
                    // (engine/midge.c:657-660): that token's argmax is 0
                    if (amax && row == 0 && v != v) atomicMax(&amax[tok], ~0ull);
                } else {
                    my[(int64_t)ui.ks * part_stride + (int64_t)tok * mldy + row] = v;
                }
            }
        }
    }
};
#undef MG_SEL

// ------------------------------------------------------ routed experts
// Decode MoE over the distinct experts of n_tok tokens' top-k selection.
// maps.m[0..2] = gate, up, down of every expert of every layer as 4-D byte
// tensors {row bytes, rows, expert, layer}.
constexpr int SW_MAX_SLOTS = 128;  // n_tok * top_k
constexpr int SW_MAX_TOK = 8;      // tokens per launch (a token picks an expert at most once)
struct MoeShared {
    int nd;                                    // distinct local experts routed to
    uint16_t list[SW_MAX_SLOTS];               // their local ids, ascending
    int ecount[SW_MAX_SLOTS];                  // routing slots of list[d]
    uint8_t eslot[SW_MAX_SLOTS][SW_MAX_TOK];   // those slots (any fixed order)
};

struct MoeCommon {
    mg_expert_layout L;
    const uint8_t *experts_layer;
    int layer;
    int e0;  // sel holds global expert ids; this blob holds experts [e0, e0 + n_experts)
    int n_experts, n_tok, top_k;
    const int32_t *sel;
    MoeShared *ms;

    __device__ const uint8_t *expert(int e) const { return experts_layer + (int64_t)e * L.expert_stride; }
    // the j-th routing slot of listed expert d, or -1
    __device__ int nth_slot(int d, int j) const { return j < ms->ecount[d] ? (int)ms->eslot[d][j] : -1; }
    // Experts routed to (ascending local ids) and, per expert, its routing
    // slots; the order of an expert's slots is immaterial (each is an
    // independent MMA column and output row).
    // All threads; needs blockDim.x >= SW_MAX_SLOTS and n_tok * top_k <= SW_MAX_SLOTS
    // (one routing slot per thread, read once).
    __device__ void build_list() {
        __shared__ uint32_t bm[64];
        __shared__ int wpre[65];
        const int n = n_tok * top_k, t = threadIdx.x;
        int e = -1;
        if (t < n) {
            e = sel[t] - e0;  // local index; other ranks' experts fall outside
            if (e < 0 || e >= n_experts) e = -1;
        }
        if (t < 64) bm[t] = 0;
        if (t < SW_MAX_SLOTS) ms->ecount[t] = 0;
        __syncthreads();
        if (e >= 0) atomicOr(&bm[e >> 5], 1u << (e & 31));
        __syncthreads();
        if (t < 32) {  // exclusive prefix of the words' popcounts, two words per lane
            const int c0 = __popc(bm[2 * t]), c1 = __popc(bm[2 * t + 1]);
            int incl = c0 + c1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (t >= o) incl += v;
            }
            wpre[2 * t] = incl - c0 - c1;
            wpre[2 * t + 1] = incl - c1;
            if (t == 31) {
                wpre[64] = incl;
                ms->nd = incl;
            }
        }
        __syncthreads();
        for (int x = t; x < n_experts; x += blockDim.x) {
            const uint32_t word = bm[x >> 5], bit = 1u << (x & 31);
            if (word & bit) ms->list[wpre[x >> 5] + __popc(word & (bit - 1))] = (uint16_t)x;
        }
        if (e >= 0) {
            const int d = wpre[e >> 5] + __popc(bm[e >> 5] & ((1u << (e & 31)) - 1u));
            const int k = atomicAdd(&ms->ecount[d], 1);
            if (k < SW_MAX_TOK) ms->eslot[d][k] = (uint8_t)t;
        }
        __syncthreads();
        // ascending slot order: every CTA sees the same per-expert lists (the
        // token groups of the block-scaled kernels split them)
        if (t < wpre[64]) {
            const int c = min(ms->ecount[t], SW_MAX_TOK);
            uint8_t *v = ms->eslot[t];
            for (int i = 1; i < c; i++)
                for (int j = i; j > 0 && v[j - 1] > v[j]; j--) {
                    const uint8_t x = v[j];
                    v[j] = v[j - 1];
                    v[j - 1] = x;
                }
        }
        __syncthreads();
    }
};

// gate/up: a unit is 64 output rows of one expert.  Stage rows 0..63 hold the
// gate rows and 64..127 the up rows; warp w's MMA rows 0..7 are gate rows
// 8w..8w+7 and 8..15 the up rows of the same outputs, so each lane holds gate
// (c0,c1) and up (c2,c3) of one row and applies the activation in registers.
template <int DT, int SC>
struct PolMoeGateUp : MoeCommon {
    const float *xb;
    int bias_ss;  // the scale slot carries the unit's biases
    int act_plain;
    float alpha, limit;
    float *h;

    __device__ int64_t rowbytes() const { return DT == MG_Q8R ? L.hidden : L.hidden / 2; }
    __device__ int xs_stride() const { return sw_xs_stride<DT>(L.hidden); }
    __device__ int64_t tpe() const { return (L.ffn + 63) / 64; }
    __device__ void init_shared() {
        __shared__ MoeShared s;
        ms = &s;
        build_list();
    }
    __device__ void finish() {}
    __device__ int64_t units() const { return (int64_t)ms->nd * tpe(); }
    __device__ void unit(int64_t u, UnitInfo &ui) const {
        const int tp = (int)tpe();
        ui.aux = (int)u / tp;
        ui.tile = (int)u - ui.aux * tp;
        ui.ks = 0;
        ui.b0 = 0;
        ui.b1 = rowbytes();
    }
    __device__ void issue(const SwMaps &maps, const UnitInfo &ui, int64_t b, void *dst, uint64_t *bar) const {
        const int e = ms->list[ui.aux];
        tma_box_4d(dst, &maps.m[0], (int)b, (int)(ui.tile * 64), e, layer, bar);
        tma_box_4d(static_cast<uint8_t *>(dst) + 64 * 128, &maps.m[1], (int)b, (int)(ui.tile * 64), e, layer, bar);
    }
    __device__ int stage_row(int w, int r16) const { return r16 < 8 ? 8 * w + r16 : 64 + 8 * w + (r16 - 8); }
    __device__ bool warp_live(const UnitInfo &ui, int w) const { return ui.tile * 64 + 8 * w < L.ffn; }
    __device__ float scale(const UnitInfo &ui, int r16, int64_t grp) const {
        const int w = sw_rg();
        const int64_t row = ui.tile * 64 + 8 * w + (r16 & 7);
        if (row >= L.ffn) return 0.f;
        const uint8_t *sc = expert(ms->list[ui.aux]) + ((r16 & 8) ? L.off[1][1] : L.off[0][1]);
        const int64_t gpr = L.hidden / 32;
        if (SC == MG_SCALE_UE8M0) return ue8m0_to_f32(__ldg(sc + row * gpr + grp));
        return h2f(__ldg(reinterpret_cast<const uint16_t *>(sc) + row * gpr + grp));
    }
    // unit scales: [gate rows tile*64.. +64][up rows], each 64 x hidden/32 scales
    static constexpr int SB = SC == MG_SCALE_UE8M0 ? 1 : 2;
    __device__ uint32_t half_bytes(const UnitInfo &ui) const {
        const int64_t nr = min((int64_t)64, L.ffn - ui.tile * 64);
        return round16((uint32_t)(nr * (L.hidden / 32) * SB));
    }
    // then the tile's gate biases and up biases (64 floats each) when bias_ss
    // (ffn % 4 == 0: every tile's bias run is a multiple of 16 bytes)
    __device__ uint32_t bias_off() const { return (uint32_t)(2 * 64 * (L.hidden / 32) * SB); }
    __device__ uint32_t bias_bytes(const UnitInfo &ui) const {
        return bias_ss ? (uint32_t)(min((int64_t)64, L.ffn - ui.tile * 64) * 4) : 0u;
    }
    __device__ uint32_t scale_bytes(const UnitInfo &ui) const { return 2 * half_bytes(ui) + 2 * bias_bytes(ui); }
    __device__ void issue_scales(const UnitInfo &ui, uint8_t *dst, uint64_t *bar) const {
        const uint8_t *eb = expert(ms->list[ui.aux]);
        const int64_t off = ui.tile * 64 * (L.hidden / 32) * SB;
        const uint32_t n = half_bytes(ui);
        bulk_g2s(dst, eb + L.off[0][1] + off, n, bar);
        bulk_g2s(dst + 64 * (L.hidden / 32) * SB, eb + L.off[1][1] + off, n, bar);
        if (bias_ss) {
            const uint32_t nb = bias_bytes(ui);
            bulk_g2s(dst + bias_off(), eb + L.off[0][2] + ui.tile * 64 * 4, nb, bar);
            bulk_g2s(dst + bias_off() + 256, eb + L.off[1][2] + ui.tile * 64 * 4, nb, bar);
        }
    }
    __device__ const uint8_t *scale_sm(const UnitInfo &, const uint8_t *ss, int r16) const {
        const int w = sw_rg();
        return ss + (int64_t)((r16 & 8 ? 64 : 0) + 8 * w + (r16 & 7)) * (L.hidden / 32) * SB;
    }
    // All tokens are staged once; a unit multiplies only the expert's own
    // tokens: MMA column n of token group nt is the expert's token 4 nt + n/2
    // (its activation rows 2 tok + n%2), columns past the expert's count read
    // token 0 and are dropped by the epilogue.
    template <int NT>
    __device__ int x_rows(const UnitInfo &ui, const SwLane &ln, uint32_t, int xs_stride, uint32_t xo[NT]) const {
        const int g = (threadIdx.x & 31) >> 2;
        const int ne = min(ms->ecount[ui.aux], SW_MAX_TOK);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int slot = nth_slot(ui.aux, nt * 4 + (g >> 1));
            const int tok = slot >= 0 ? slot / top_k : 0;
            xo[nt] = (uint32_t)((2 * tok + (g & 1)) * xs_stride * 2) + (ln.xoff - (uint32_t)(g * xs_stride * 2));
        }
        return (ne + 3) >> 2;
    }
    __device__ bool restage(int64_t, int64_t) const { return false; }
    __device__ void stage_x_units(int64_t u0, int64_t, __half *xs, int xs_stride) const { stage_x(u0, xs, xs_stride); }
    __device__ void stage_x(int64_t, __half *xs, int xs_stride) const {
        stage_x_n<DT>(xb, L.hidden, n_tok, (int)L.hidden, xs, xs_stride, threadIdx.x, SW_CONS * 32);
    }
    template <int NT>
    __device__ void epilogue(const UnitInfo &ui, int w, const float acc[NT][4], const uint8_t *ss) const {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        const int e = ms->list[ui.aux];
        const int64_t row = ui.tile * 64 + 8 * w + g;
        if (row >= L.ffn) return;
        const uint8_t *eb = expert(e);
        float bg, bu;
        if (bias_ss && ss) {
            bg = reinterpret_cast<const float *>(ss + bias_off())[8 * w + g];
            bu = reinterpret_cast<const float *>(ss + bias_off())[64 + 8 * w + g];
        } else {
            bg = reinterpret_cast<const float *>(eb + L.off[0][2])[row];
            bu = reinterpret_cast<const float *>(eb + L.off[1][2])[row];
        }
        float sg = 1.f, su = 1.f;
        if (DT == MG_Q8R) {
            sg = reinterpret_cast<const float *>(eb + L.off[0][1])[row];
            su = reinterpret_cast<const float *>(eb + L.off[1][1])[row];
        }
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            const int slot = nth_slot(ui.aux, nt * 4 + t);  // MMA columns 2t, 2t+1: the expert's slot 4 nt + t
            if (slot < 0) continue;
            float gv = acc[nt][0] + acc[nt][1], uv = acc[nt][2] + acc[nt][3];
            if (DT == MG_Q8R) { gv = __fmul_rn(gv, sg); uv = __fmul_rn(uv, su); }
            gv = __fadd_rn(gv, bg);
            uv = __fadd_rn(uv, bu);
            float hv;
            if (act_plain) {
                hv = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
            } else {
                if (gv > limit) gv = limit;
                if (uv > limit) uv = limit;
                if (uv < -limit) uv = -limit;
                hv = __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(__fmul_rn(-alpha, gv)))), __fadd_rn(uv, 1.0f));
            }
            h[(int64_t)slot * L.ffn + row] = hv;
        }
    }
};

// down: a unit is 128 rows of one expert's down matrix times a K split; the
// activations are the expert's slots' h rows (re-staged when the expert
// changes).  Output: y[ks][slot][row] partial sums (+ bias in split 0).
template <int DT, int SC>
struct PolMoeDown : MoeCommon {
    const float *h;
    float *y;
    int bias_ss;  // the scale slot carries the unit's biases
    int ks_count;
    int64_t kbytes_per_split;

    __device__ int64_t rowbytes() const { return DT == MG_Q8R ? L.ffn : L.ffn / 2; }
    __device__ int xs_stride() const { return sw_xs_stride<DT>(L.ffn); }
    __device__ int64_t tpe() const { return ((L.hidden + SW_ROWS - 1) / SW_ROWS) * ks_count; }
    __device__ void init_shared() {
        __shared__ MoeShared s;
        ms = &s;
        build_list();
    }
    __device__ void finish() {}
    __device__ int64_t units() const { return (int64_t)ms->nd * tpe(); }
    __device__ void unit(int64_t u, UnitInfo &ui) const {
        const int tp = (int)tpe();
        ui.aux = (int)u / tp;
        const int r = (int)u - ui.aux * tp;
        ui.tile = r / ks_count;
        ui.ks = r - (r / ks_count) * ks_count;
        ui.b0 = (int64_t)ui.ks * kbytes_per_split;
        ui.b1 = min(rowbytes(), ui.b0 + kbytes_per_split);
    }
    __device__ void issue(const SwMaps &maps, const UnitInfo &ui, int64_t b, void *dst, uint64_t *bar) const {
        tma_box_4d(dst, &maps.m[2], (int)b, (int)(ui.tile * SW_ROWS), ms->list[ui.aux], layer, bar);
    }
    __device__ int stage_row(int w, int r16) const { return 16 * w + r16; }
    __device__ bool warp_live(const UnitInfo &ui, int w) const { return ui.tile * SW_ROWS + 16 * w < L.hidden; }
    __device__ float scale(const UnitInfo &ui, int r16, int64_t grp) const {
        const int w = sw_rg();
        const int64_t row = ui.tile * SW_ROWS + 16 * w + r16;
        if (row >= L.hidden) return 0.f;
        const uint8_t *sc = expert(ms->list[ui.aux]) + L.off[2][1];
        const int64_t gpr = L.ffn / 32;
        if (SC == MG_SCALE_UE8M0) return ue8m0_to_f32(__ldg(sc + row * gpr + grp));
        return h2f(__ldg(reinterpret_cast<const uint16_t *>(sc) + row * gpr + grp));
    }
    // unit scales: the tile's 128 rows, whole rows (both K splits read all of them)
    static constexpr int SB = SC == MG_SCALE_UE8M0 ? 1 : 2;
    // then the tile's biases (128 floats) when bias_ss (hidden % 4 == 0)
    __device__ uint32_t bias_off() const { return (uint32_t)(SW_ROWS * (L.ffn / 32) * SB); }
    __device__ uint32_t scale_part(const UnitInfo &ui) const {
        const int64_t nr = min((int64_t)SW_ROWS, L.hidden - ui.tile * SW_ROWS);
        return round16((uint32_t)(nr * (L.ffn / 32) * SB));
    }
    __device__ uint32_t bias_bytes(const UnitInfo &ui) const {
        return bias_ss ? (uint32_t)(min((int64_t)SW_ROWS, L.hidden - ui.tile * SW_ROWS) * 4) : 0u;
    }
    __device__ uint32_t scale_bytes(const UnitInfo &ui) const { return scale_part(ui) + bias_bytes(ui); }
    __device__ void issue_scales(const UnitInfo &ui, uint8_t *dst, uint64_t *bar) const {
        const uint8_t *eb = expert(ms->list[ui.aux]);
        bulk_g2s(dst, eb + L.off[2][1] + ui.tile * SW_ROWS * (L.ffn / 32) * SB, scale_part(ui), bar);
        if (bias_ss) bulk_g2s(dst + bias_off(), eb + L.off[2][2] + ui.tile * SW_ROWS * 4, bias_bytes(ui), bar);
    }
    __device__ const uint8_t *scale_sm(const UnitInfo &, const uint8_t *ss, int r16) const {
        const int w = sw_rg();
        return ss + (int64_t)(16 * w + r16) * (L.ffn / 32) * SB;
    }
    template <int NT>
    __device__ int x_rows(const UnitInfo &ui, const SwLane &ln, uint32_t xs8_nt, int, uint32_t xo[NT]) const {
        sw_x_rows<NT>(ln, xs8_nt, xo);
        return (min(ms->ecount[ui.aux], SW_MAX_TOK) + 3) >> 2;
    }
    __device__ bool restage(int64_t u, int64_t u0) const { return u != u0 && unit_expert(u) != unit_expert(u - 1); }
    __device__ void stage_x_units(int64_t u0, int64_t, __half *xs, int xs_stride) const { stage_x(u0, xs, xs_stride); }
    __device__ int unit_expert(int64_t u) const { return (int)u / (int)tpe(); }
    // the expert's slots' h rows: slot j at activation rows 2j, 2j + 1
    __device__ void stage_x(int64_t u, __half *xs, int xs_stride) const {
        const int d = unit_expert(u), ne = min(ms->ecount[d], SW_MAX_TOK);
        for (int j = 0; j < ne; j++)
            stage_x_n<DT>(h + (int64_t)ms->eslot[d][j] * L.ffn, L.ffn, 1, (int)L.ffn, xs + 2 * j * xs_stride,
                          xs_stride, threadIdx.x, SW_CONS * 32);
    }
    template <int NT>
    __device__ void epilogue(const UnitInfo &ui, int w, const float acc[NT][4], const uint8_t *ss) const {
        const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
        const uint8_t *eb = expert(ms->list[ui.aux]);
#pragma unroll
        for (int half = 0; half < 2; half++) {
            const int64_t row = ui.tile * SW_ROWS + 16 * w + g + 8 * half;
            if (row >= L.hidden) continue;
            float rs = 1.f;
            if (DT == MG_Q8R) rs = reinterpret_cast<const float *>(eb + L.off[2][1])[row];
            const float bd = ui.ks != 0 ? 0.f
                             : (bias_ss && ss) ? reinterpret_cast<const float *>(ss + bias_off())[16 * w + g + 8 * half]
                                               : reinterpret_cast<const float *>(eb + L.off[2][2])[row];
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
                const int slot = nth_slot(ui.aux, nt * 4 + t);
                if (slot < 0) continue;
                float v = acc[nt][2 * half] + acc[nt][2 * half + 1];
                if (DT == MG_Q8R) v = __fmul_rn(v, rs);
                v = __fadd_rn(v, bd);
                y[((int64_t)ui.ks * n_tok * top_k + slot) * L.hidden + row] = v;
            }
        }
    }
};

}  // namespace mg

// mg_bsmoe.cu -- decode-time routed experts (MXFP4, ue8m0 group scales) on
// block-scaled tcgen05 MMAs: tcgen05.mma.kind::mxf4.block_scale.block32.
//
// The tensor core reads the e2m1 weights and their ue8m0 group scales as
// they are stored (engine/mten.h:136 expert layout; the scale of 32 weights
// is 2^(code - 127), the reference's dequant), so no SM instruction is spent
// per weight:
//   * A (weights): TMA copies each K-stage of 128 bytes (256 packed e2m1
//     values) of 128 rows from HBM into shared memory (128-byte swizzle,
//     K-major); gate/up stages hold 64 gate rows then the 64 up rows of the
//     same outputs, down stages 128 rows.  The ragged end of a row is
//     zero-filled by the TMA bounds.
//   * B (activations): each activation row x is written as 12 e2m1 limbs,
//     x = sum_l q_l 2^(c_l,b - 127), with one ue8m0 code per limb and block of
//     32 values: limb l quantises the residual of limbs < l at a scale 4x
//     below limb l-1's (round-to-nearest leaves less than half a step, so the
//     scaled residual stays below 4 and never saturates), i.e. 2 bits per
//     limb, 24 bits below the block maximum.  A token owns 16 B rows (MMA
//     columns); rows 12..15 stay zero.
//   * scale factors: per stage the 128 A rows x 8 blocks and the B rows x 8
//     blocks are laid out as 32 x 16-byte atoms (4 blocks each) and copied
//     into TMEM with tcgen05.cp.32x128b.warpx4; an MMA (K = 64) reads two
//     blocks, selected by its scale-factor id (0 or 2).  The A atoms are
//     written once, when the model is made ready (k_bs_atoms: 1 KB per
//     (expert, tile, stage)), and streamed beside the A tile; the B atoms of
//     a token group stay in TMEM for all its units, so a stage costs two
//     atom copies and four MMAs (the MMA issuer's loop sets the kernel's
//     pace: measured per-stage marks showed the data ready ~3 us after issue
//     and the issuer never waiting for it).
//   * D (fp32, TMEM): 128 output rows x 16 columns per token; the epilogue
//     sums each token's 16 limb columns.
// Each unit multiplies one expert's weight tile by up to 2 of its routed
// tokens (the MMA cost does not depend on N at these widths); an expert
// with more routed tokens takes further token groups.
//
// Warp roles (320 threads, one CTA per SM, persistent over the units):
//   warp 0     producer: per stage the A box(es) by TMA and the stage's A
//              atoms by bulk copy into a ring; per token group its B rows
//              (resident for all K stages) and its B scale words
//   warp 1     MMA issuer (one thread): per token group the B scale atoms of
//              every K stage into one of two resident TMEM buffers; per stage
//              the 2 A scale atoms into the stage's TMEM columns (tcgen05.cp,
//              ordered before the MMAs that read them), 4 MMAs of K = 64,
//              commit -> the stage is free; per unit commit -> accumulator
//              buffer ready (2 buffers)
//   warp 2     B atoms: per token group, the B atoms of every K stage from
//              the group's words (lane = B row) into shared memory
//   warps 3-5  idle after setup
//   warps 6-9  epilogue (TMEM lane quadrant = warp % 4): limb sums; gate/up:
//              bias, clamped SwiGLU (engine/midge.c:386-392) and the h values
//              re-encoded as 12 limbs for the down pass; down: bias in split
//              0 and the per-slot partial sums y[ks][slot][row]
// Every wait is bounded: a timed-out wait sets the error word and the role
// stops; the producer waits for its copies in flight and the MMA issuer for
// its MMAs before the CTA exits.
#include <cstdlib>

#include "mg_bsmoe.h"
#include "mg_stream.cuh"
#include "mg_tc.cuh"

namespace mg {

#define BS_TRY(expr)                  \
    do {                              \
        int _rc = (expr);             \
        if (_rc != MG_OK) return _rc; \
    } while (0)

constexpr int BS_LIMBS = 16;                           // B rows (MMA columns) per token
constexpr int BS_LQ = 12;                              // of which encoded limbs
constexpr int BS_KE = 256;                             // K values per stage (128 packed bytes)
constexpr int BS_TOKG = 2;                             // tokens per unit
constexpr int BS_A_BYTES = 128 * 128;                  // A stage: 128 rows x 128 B
constexpr int BS_B_TOK = BS_LIMBS * 128;               // B rows of one token per K stage: 16 x 128 B
constexpr int BS_B_STAGE = BS_TOKG * BS_B_TOK;         // resident B: per K stage, the group's tokens
constexpr int BS_MAX_NK = 16;                          // K stages of a row (K <= 4096)
constexpr int BS_CH = 2;                               // K chunks (of 256 values) per ring stage
constexpr int BS_STAGE = BS_CH * BS_A_BYTES;           // ring stage: the A tiles of its chunks (1024-aligned)
constexpr int BS_ATOMS = 1024;                         // the 2 A scale atoms of a chunk
constexpr int BS_BATOMS = 1024;                        // the 2 B scale atoms of a K stage (resident per token group)
constexpr int BS_MAX_STAGES = 6;
constexpr int BS_THREADS = 320;
constexpr int BS_ACC_COLS = BS_TOKG * BS_LIMBS;        // accumulator columns of a unit (N)
// accumulators: 2 units in flight x 2 independent halves (the MMAs of a stage
// alternate between them, so consecutive MMAs do not wait for each other)
constexpr int BS_SFA_COL0 = 4 * BS_ACC_COLS;           // A scale columns: 8 per ring stage after the accumulators
constexpr int BS_SFB_COL0 = BS_SFA_COL0 + 8 * BS_CH * BS_MAX_STAGES;  // B scale columns: 2 buffers x 8 per K chunk
constexpr int BS_TMEM_COLS = 512;
static_assert(BS_SFB_COL0 + 2 * 8 * BS_MAX_NK <= BS_TMEM_COLS, "TMEM columns");
constexpr int BS_MAX_V = 4 * SW_MAX_SLOTS;             // token groups (experts x up to 4)
// error word codes of a timed-out wait, by role (beside the streamed kernels' 1)
constexpr int BS_ERR_PRODUCER = 11, BS_ERR_MMA = 12, BS_ERR_ATOMS = 13, BS_ERR_EPILOGUE = 14, BS_ERR_DRAIN = 15;
// the first failure is kept (21.. name the wait that gave up: producer 22 ring stage; MMA 24 B ready,
// 25 accumulator buffer, 26 stage; stager 27 the buffer's previous group's MMAs, 28 the previous
// group's atom copies, 30 a down group's gate/up tiles)
__device__ __forceinline__ void bs_fail(int *err, int code) { atomicCAS(err, 0, code); }

struct BsBars {
    uint64_t full[BS_MAX_STAGES], empty[BS_MAX_STAGES];
    uint64_t accfull[2], accempty[2];
    uint64_t bready[2];  // B buffer b holds a token group's rows, and the shared B atoms its atoms
    uint64_t bfree[2];   // the MMAs of buffer b's group are done: its rows may be replaced
    uint64_t batfree;    // the MMA issuer's copies of the shared B atoms into TMEM have completed
    uint64_t done;    // the MMA issuer's last commit: no MMA is in flight when TMEM is released
    uint32_t tmem;
};

struct BsMapsK {
    CUtensorMap a[3];  // A boxes: gate, up (64 rows each), down (128 rows)
};

// 16-byte global -> shared copy (L2 only), completed by cp.async.wait_all
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// shared-memory matrix descriptor, no swizzle (the scale atoms: 8-row core
// matrices of 16-byte rows, 128 B apart; one core matrix along K)
__device__ __forceinline__ uint64_t umma_desc_plain(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// instruction descriptor, kind::mxf4 block-scaled: A and B e2m1 (1), ue8m0
// scales (bit 23), K-major A and B, K = 64, D f32; scale-factor ids in bits
// 4-5 (B) and 29-30 (A)
__device__ __forceinline__ uint32_t bs_idesc(int N, uint32_t sf_id) {
    return (sf_id << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(128 >> 4) << 24) | (sf_id << 29);
}
__device__ __forceinline__ void bs_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa, uint32_t sfb,
                                       uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
}
__device__ __forceinline__ void bs_cp_atom(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// ---------------------------------------------------------- limb encoding
// e2m1 nibble of v (|v| < 4 here: no saturation) and its exact value
__device__ __forceinline__ uint32_t e2m1_rn(float v, float &back) {
    uint32_t byte;
    asm("{\n .reg .b8 t;\n cvt.rn.satfinite.e2m1x2.f32 t, %1, %1;\n mov.b32 %0, {t, t, t, t};\n}"
        : "=r"(byte)
        : "f"(v));
    uint32_t h2;
    asm("{\n .reg .b8 b0, b1, b2, b3;\n mov.b32 {b0, b1, b2, b3}, %1;\n cvt.rn.f16x2.e2m1x2 %0, b0;\n}"
        : "=r"(h2)
        : "r"(byte));
    back = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFF)));
    return byte & 0xF;
}

__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }  // -126..127

// Warp-collective: the 32 lanes hold one block of 32 values (lane = column).
// Writes the packed limb bytes of the block (lane pair 2i, 2i+1 -> byte i:
// low nibble the even column) at dst[l * ld + i] from the even lanes, and from
// lane 0 limb l's scale code at codes[4 l], for l < BS_LQ.  Limb 0's scale is
// 2^(E - 1), E the exponent of the block maximum (so the scaled values lie
// below 4, e2m1 max 6); limb l's is 4^-l times that (never below 2^-126).  An
// all-zero or non-finite block gets code 127 throughout (NaN passes on).
__device__ __forceinline__ void bs_limbs(float v, uint8_t *dst, int64_t ld, uint8_t *codes) {
    const int lane = threadIdx.x & 31;
    const float m = warp_max(fabsf(v));
    int e = 0;
    bool scaled = false;
    if (m > 0.f && m <= 3.4e38f) {
        e = (int)((__float_as_uint(m) >> 23) & 0xFF) - 128;  // E - 1
        if (e < -126) e = -126;
        scaled = true;
    }
    float r = v;
#pragma unroll
    for (int l = 0; l < BS_LQ; l++) {
        float back;
        const uint32_t q = e2m1_rn(r * pow2f(-e), back);
        r = fmaf(-back, pow2f(e), r);
        const uint32_t hi = __shfl_down_sync(0xffffffffu, q, 1);
        if (!(lane & 1)) dst[(int64_t)l * ld + (lane >> 1)] = (uint8_t)(q | (hi << 4));
        if (lane == 0) codes[4 * l] = (uint8_t)(scaled ? e + 127 : 127);
        if (scaled && e - 2 >= -126) e -= 2;
    }
}

// rows x K floats -> packed limbs [row*16 + l][kpad/2] and scale words
// [row][kpad/128][16] (byte kb % 4 of word (row, kb / 4, l) = limb l's code of
// block kb).  Blocks past K encode zeros.  One warp per (row, block of 32).
__global__ void k_bs_limbs(const float *x, int64_t ldx, int rows, int K, int kpad, uint8_t *limbs, uint8_t *sfw) {
    asm volatile("griddepcontrol.launch_dependents;");  // the gate/up grid may start its setup
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = kpad / 32;
    if (warp >= rows * nb) return;
    const int row = warp / nb, kb = warp - row * nb, k = kb * 32 + lane;
    const float v = k < K ? x[(int64_t)row * ldx + k] : 0.f;
    bs_limbs(v, limbs + (int64_t)row * BS_LIMBS * (kpad / 2) + kb * 16, kpad / 2,
             sfw + (((int64_t)row * (kpad / 128) + kb / 4) * BS_LIMBS) * 4 + (kb & 3));
}

// Expert scales -> the A scale atoms of every unit stage (once per model).
// Unit u of an expert: gate/up tile u / nk_h, stage u % nk_h for u < atoms_dn
// (rows 0-63 the tile's gate rows, 64-127 the up rows of the same outputs),
// else down tile (u - atoms_dn) / nk_f (128 rows).  Its 1024 bytes are two
// atoms (blocks 8k..8k+3, 8k+4..8k+7): block kb of row r at byte
// 512 (kb / 4 % 2) + (r % 32) 16 + (r / 32) 4 + kb % 4.  Rows past the matrix
// and blocks past K get code 127 (their weights are zero-filled by the TMA).
// Block (256 threads) = one unit; thread = (atom h, row r).
__global__ void k_bs_atoms(const uint8_t *experts, mg_expert_layout L, int64_t n_le, int n_local, int nk_h, int nk_f,
                           int atoms_dn, uint8_t *atoms, int64_t atoms_expert) {
    const int u = blockIdx.x, h = threadIdx.x >> 7, r = threadIdx.x & 127;
    for (int64_t le = blockIdx.y; le < n_le; le += gridDim.y) {
        const uint8_t *eb = experts + (le / n_local) * L.layer_stride + (le % n_local) * L.expert_stride;
        const uint8_t *src = nullptr;
        int G, k;
        if (u < atoms_dn) {
            const int tile = u / nk_h;
            k = u - tile * nk_h;
            G = (int)(L.hidden / 32);
            const int64_t row = (int64_t)tile * 64 + (r & 63);
            if (row < L.ffn) src = eb + L.off[r < 64 ? 0 : 1][1] + row * G;
        } else {
            const int v = u - atoms_dn, tile = v / nk_f;
            k = v - tile * nk_f;
            G = (int)(L.ffn / 32);
            const int64_t row = (int64_t)tile * 128 + r;
            if (row < L.hidden) src = eb + L.off[2][1] + row * G;
        }
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int kb = 8 * k + 4 * h + i;
            const uint32_t c = (src && kb < G) ? src[kb] : 127u;
            w |= c << (8 * i);
        }
        *reinterpret_cast<uint32_t *>(atoms + le * atoms_expert + (int64_t)u * 1024 + 512 * h + (r & 31) * 16 +
                                      (r >> 5) * 4) = w;
    }
}

// ---------------------------------------------------------- routed experts
// the parameters of one pass (0 gate/up, 1 down)
struct BsPass {
    const uint8_t *limbs; // B limb rows [src * 16 + l][ld] (src: token for gate/up, slot for down)
    int64_t ld;           // bytes per limb row
    const uint32_t *bsf;  // B scale words [src][g4][16]
    int g4;               // scale words per B row and limb
    int nk;               // K chunks of an A row
    int atoms_u0;         // first atom of the pass within an expert (0 gate/up, atoms_dn down)
};
// one unit of a CTA's sequence: 128 A rows of expert list[d] times token group tg
struct BsUnit {
    int mode, v, d, tg, tile, ks, k0, k1;
};
struct BsPol : MoeCommon {
    BsPass ps[2];
    int act_plain;
    float alpha, limit;
    uint8_t *hl;          // gate/up: h limbs out [slot*16 + l][hl_ld]
    uint8_t *hsf;         // gate/up: their scale words (bytes) [slot][hg4][16][4]
    int64_t hl_ld;        // bytes per limb row
    int hg4;
    float *y;             // down: [ks][n_tok*top_k][hidden]
    int ks_count, kst;    // down: K splits and K chunks per split
    int *err;
    uint32_t *sync;       // [0] CTAs finished, [1 + v] gate/up tiles done of token group v
    const int *vl;        // token groups: (list index) | (group << 16)
    const uint8_t *atoms; // this layer's expert scale atoms
    int64_t atoms_expert; // bytes per expert
    int g_all, g_per, d_all, d_per;  // units of each pass, and per CTA (set in the kernel)

    // (selected, not indexed: a run-time index into the parameter array would
    // copy it to local memory)
    __device__ BsPass pass(int mode) const { return mode ? ps[1] : ps[0]; }
    __device__ int tpe(int mode) const {
        return mode == 0 ? (int)((L.ffn + 63) / 64) : (int)((L.hidden + 127) / 128) * ks_count;
    }
    // CTA c runs gate/up units [c g_per, (c+1) g_per), then down units [c d_per, (c+1) d_per)
    __device__ int seq_gate(int c) const { return max(0, min(g_all, (c + 1) * g_per) - c * g_per); }
    __device__ int seq_len(int c) const { return seq_gate(c) + max(0, min(d_all, (c + 1) * d_per) - c * d_per); }
    __device__ void seq_unit(int c, int j, BsUnit &x) const {
        const int gn = seq_gate(c);
        int u;
        if (j < gn) {
            x.mode = 0;
            u = c * g_per + j;
        } else {
            x.mode = 1;
            u = c * d_per + (j - gn);
        }
        const int t = tpe(x.mode), v = u / t, r = u - v * t;
        x.v = v;
        x.d = vl[v] & 0xFFFF;
        x.tg = vl[v] >> 16;
        if (x.mode == 0) {
            x.tile = r; x.ks = 0; x.k0 = 0; x.k1 = ps[0].nk;
        } else {
            x.tile = r / ks_count; x.ks = r - x.tile * ks_count;
            x.k0 = x.ks * kst; x.k1 = min(ps[1].nk, x.k0 + kst);
        }
    }
    // Chunk order of a unit: its K chunks [k0, k1) from a start that depends
    // on the tile and split only, so that the CTAs working on one expert
    // read different parts of the shared activation limb rows at any time
    // (the same rows read in lockstep by many SMs contend in L2); the order
    // is fixed per (tile, split), so results do not depend on the grid.
    __device__ int stage_k(int k0, int k1, int i, int tile, int ks) const {
        const int n = k1 - k0;
        int r = (tile * 5 + ks * 3) % n;
        r += i;
        if (r >= n) r -= n;
        return k0 + r;
    }
    // routing slots of (expert d, group tg) and their B source rows
    __device__ int ntok(int d, int tg) const { return min(BS_TOKG, min(ms->ecount[d], SW_MAX_TOK) - BS_TOKG * tg); }
    __device__ int slot_of(int d, int tg, int j) const { return ms->eslot[d][BS_TOKG * tg + j]; }
    __device__ int src_of(int mode, int d, int tg, int j) const {
        const int s = slot_of(d, tg, j);
        return mode == 0 ? s / top_k : s;
    }
    // the A atoms of local expert e, tile, K chunk k (1024 bytes)
    __device__ const uint8_t *atoms_of(int mode, int e, int tile, int k) const {
        return atoms + e * atoms_expert + ((int64_t)pass(mode).atoms_u0 + (int64_t)tile * pass(mode).nk + k) * 1024;
    }
    // the group's B scale words [token j][g4][16]
    __device__ uint32_t bw_bytes(int mode) const { return (uint32_t)pass(mode).g4 * BS_LIMBS * 4; }
};

// a down group's gate/up tiles: the count the epilogues raise (release) reaches
// need; generic-proxy writes then feed async-proxy (TMA, bulk) reads
constexpr uint32_t BS_TILE_POLLS = 1u << 22;
__device__ __forceinline__ bool bs_tiles_done(const uint32_t *cnt, uint32_t need, bool block) {
    for (uint32_t i = 0;; i++) {
        uint32_t v;
        asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(cnt) : "memory");
        if (v >= need) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            return true;
        }
        if (!block || i >= BS_TILE_POLLS) return false;
        __nanosleep(64);
    }
}

__device__ __forceinline__ float bs_act(float gv, float uv, const BsPol &p) {
    if (p.act_plain) return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
    if (gv > p.limit) gv = p.limit;
    if (uv > p.limit) uv = p.limit;
    if (uv < -p.limit) uv = -p.limit;
    return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(__fmul_rn(-p.alpha, gv)))), __fadd_rn(uv, 1.0f));
}

__global__ void __launch_bounds__(BS_THREADS, 1) k_bsmoe(const __grid_constant__ BsMapsK maps, BsPol pol, int nst,
                                                         int ssb) {
    extern __shared__ __align__(1024) uint8_t bs_raw[];
    uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(bs_raw) + 1023) & ~(uintptr_t)1023);
    const int nk_max = max(pol.ps[0].nk, pol.ps[1].nk);
    uint8_t *stages = sm;
    uint8_t *atoms = stages + (size_t)nst * BS_STAGE;  // per ring stage and chunk: its 2 A atoms (bulk copy) +0, +512
    // two B row buffers [K chunk][token j][16 rows x 128 B] (1024-aligned), one
    // per token group in flight; the group's B atoms pass through one shared
    // buffer on their way to TMEM (whose two buffers hold them for the MMAs)
    uint8_t *bres = atoms + (size_t)nst * BS_CH * BS_ATOMS;
    const size_t bbuf = (size_t)nk_max * BS_B_STAGE;
    uint8_t *batoms = bres + 2 * bbuf;  // [K chunk][2 B atoms of 512 B]
    uint8_t *bwreg = batoms + (size_t)nk_max * BS_BATOMS;  // the token group's B scale words [token j][g4][16]
    float *ex = reinterpret_cast<float *>(bwreg + (size_t)ssb);  // 64 rows x 2 tokens (up values)
    BsBars *bb = reinterpret_cast<BsBars *>(ex + 64 * BS_TOKG);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    __shared__ int vlist[BS_MAX_V];
    __shared__ int nv_sh, last_cta, stage_ok, atoms_ok;
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 3; i++) tma_prefetch_map(&maps.a[i]);
    }
    // barriers and TMEM first: they overlap the routing-slot loads of build_list
    if (warp == 2) {
        if (lane < nst) {
            mbar_init(&bb->full[lane], 1);  // the producer's expect-tx arrival: A tiles + A atoms
            mbar_init(&bb->empty[lane], 1);
        } else if (lane >= 18 && lane < 20) {
            mbar_init(&bb->accfull[lane - 18], 1);
            mbar_init(&bb->accempty[lane - 18], 4);
        } else if (lane == 20) {
            mbar_init(&bb->bready[0], 1);
            mbar_init(&bb->bready[1], 1);
            mbar_init(&bb->bfree[0], 1);
            mbar_init(&bb->bfree[1], 1);
            mbar_init(&bb->batfree, 1);
        } else if (lane == 21) {
            mbar_init(&bb->done, 1);
        }
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(&bb->tmem, BS_TMEM_COLS);
    {
        __shared__ MoeShared s;
        pol.ms = &s;
        pol.build_list();  // all threads; ends with __syncthreads
    }
    if (warp == 0) {  // token groups in expert order: up to 4 experts per lane, prefix over the warp
        int c[4], sum = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int d = 4 * lane + i;
            c[i] = d < pol.ms->nd ? (min(pol.ms->ecount[d], SW_MAX_TOK) + BS_TOKG - 1) / BS_TOKG : 0;
            sum += c[i];
        }
        int incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int pos = incl - sum;
#pragma unroll
        for (int i = 0; i < 4; i++)
            for (int g = 0; g < c[i]; g++) vlist[pos++] = (4 * lane + i) | (g << 16);
        if (lane == 31) nv_sh = incl;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // the next kernel may start its setup on SMs this grid leaves; it waits
    // for this grid before it reads what this one writes
    if (tid == 0) asm volatile("griddepcontrol.launch_dependents;");
    // Every role but the producer needs the previous grid's outputs (the x
    // limbs) before its first wait can complete: it waits for that grid here,
    // so that its bounded waits count from then on.
    if (warp != 0) asm volatile("griddepcontrol.wait;" ::: "memory");
    pol.vl = vlist;
    const uint32_t tb = bb->tmem;
    const int nv = nv_sh, c = (int)blockIdx.x;
    pol.g_all = nv * pol.tpe(0);
    pol.d_all = nv * pol.tpe(1);
    pol.g_per = (pol.g_all + (int)gridDim.x - 1) / (int)gridDim.x;
    pol.d_per = (pol.d_all + (int)gridDim.x - 1) / (int)gridDim.x;
    const int nseq = pol.seq_len(c);
    const uint32_t tiles_need = (uint32_t)pol.tpe(0);

    if (warp == 0) {
        // ------------------------------------------------------ producer
        // the A stages of the CTA's units, back to back through the ring
        if (lane == 0 && nseq > 0) {
            bool ok = true;
            int s = 0;
            uint32_t ph = 0, it = 0;
            for (int q = 0; q < nseq && ok; q++) {
                BsUnit x;
                pol.seq_unit(c, q, x);
                const int e = pol.ms->list[x.d];
                const int nchk = x.k1 - x.k0;
                for (int i = 0; i < nchk; i += BS_CH) {
                    const int nch = min(BS_CH, nchk - i);
                    if (it >= (uint32_t)nst && !mbar_wait(&bb->empty[s], ph ^ 1u)) { bs_fail(pol.err, 22); ok = false; break; }
                    mbar_arrive_expect_tx(&bb->full[s], (uint32_t)nch * (BS_A_BYTES + BS_ATOMS));
                    for (int h = 0; h < nch; h++) {
                        const int k = pol.stage_k(x.k0, x.k1, i + h, x.tile, x.ks);
                        uint8_t *st = stages + (size_t)s * BS_STAGE + (size_t)h * BS_A_BYTES;
                        if (x.mode == 0) {
                            tma_box_4d(st, &maps.a[0], k * 128, x.tile * 64, e, pol.layer, &bb->full[s]);
                            tma_box_4d(st + BS_A_BYTES / 2, &maps.a[1], k * 128, x.tile * 64, e, pol.layer, &bb->full[s]);
                        } else {
                            tma_box_4d(st, &maps.a[2], k * 128, x.tile * 128, e, pol.layer, &bb->full[s]);
                        }
                        bulk_g2s(atoms + ((size_t)s * BS_CH + h) * BS_ATOMS, pol.atoms_of(x.mode, e, x.tile, k), BS_ATOMS,
                                 &bb->full[s]);
                    }
                    it++;
                    if (++s == nst) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) bs_fail(pol.err, BS_ERR_PRODUCER);
            // every copy issued has landed before the CTA may exit (a failed wait is recorded)
            for (int64_t k = (int64_t)it - 1; k >= 0 && k >= (int64_t)it - nst; k--)
                if (!mbar_wait(&bb->full[k % nst], (uint32_t)((k / nst) & 1))) bs_fail(pol.err, BS_ERR_DRAIN);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0 && nseq > 0) {
            bool ok = true;
            int s = 0;
            uint32_t ph = 0;
            const uint64_t da0 = umma_desc_sw128(smem_u32(stages)), db0 = umma_desc_sw128(smem_u32(bres));
            const uint64_t dat0 = umma_desc_plain(smem_u32(atoms), 512, 128);
            const uint64_t dbt0 = umma_desc_plain(smem_u32(batoms), 512, 128);
            int key = -1, ng = 0, gb = 0;
            uint32_t tbb = tb + BS_SFB_COL0;  // the current token group's B scale columns
            uint64_t dbg = db0;               // and its B row buffer
            for (int q = 0; q < nseq && ok; q++) {
                BsUnit x;
                pol.seq_unit(c, q, x);
                const int N = BS_LIMBS * pol.ntok(x.d, x.tg);
                const int b = q & 1;
                // unit q - 2's accumulator handed back: its MMAs, and all before, are done
                if (q >= 2 && !mbar_wait(&bb->accempty[b], (uint32_t)(((q >> 1) - 1) & 1))) { bs_fail(pol.err, 25); ok = false; break; }
                const int gkey = x.d | (x.tg << 16) | (x.mode << 30);
                if (gkey != key) {
                    // a new token group: its B rows are in buffer ng % 2; its B scale atoms of
                    // every K chunk go into TMEM buffer ng % 2 (the MMAs of group ng - 2, the
                    // last to read it, have completed: the stager saw bfree before staging)
                    key = gkey;
                    gb = ng & 1;
                    if (!mbar_wait(&bb->bready[gb], (uint32_t)((ng >> 1) & 1))) { bs_fail(pol.err, 24); ok = false; break; }
                    tc_fence_after();
                    tbb = tb + BS_SFB_COL0 + (uint32_t)(gb * 8 * BS_MAX_NK);
                    dbg = db0 + (uint64_t)((gb * bbuf) >> 4);
                    for (int kk = 0, nk = pol.pass(x.mode).nk; kk < nk; kk++) {
                        const uint64_t dk = dbt0 + (uint64_t)((kk * BS_BATOMS) >> 4);
                        bs_cp_atom(tbb + 8u * (uint32_t)kk, dk);
                        bs_cp_atom(tbb + 8u * (uint32_t)kk + 4u, dk + 32);
                    }
                    tc_commit(&bb->batfree);  // the shared atoms may be rebuilt once these copies are done
                    ng++;
                }
                tc_fence_after();
                const uint32_t tacc = tb + (uint32_t)(b * BS_ACC_COLS);  // half 1 at + 2 * BS_ACC_COLS
                const uint32_t id0 = bs_idesc(N, 0), id2 = bs_idesc(N, 2);
                const int nchk = x.k1 - x.k0;
                for (int i = 0; i < nchk; i += BS_CH) {
                    const int nch = min(BS_CH, nchk - i);
                    if (!mbar_wait(&bb->full[s], ph)) { bs_fail(pol.err, 26); ok = false; break; }
                    tc_fence_after();
                    // the stage's A scale atoms into its TMEM columns (+0, +4 per chunk),
                    // executed in order before the MMAs below; the B atoms of every K chunk
                    // are resident
                    for (int h = 0; h < nch; h++) {
                        const uint64_t dat = dat0 + (uint64_t)((((size_t)s * BS_CH + h) * BS_ATOMS) >> 4);
                        const uint32_t tsa = tb + BS_SFA_COL0 + 8u * (uint32_t)(s * BS_CH + h);
                        bs_cp_atom(tsa, dat);
                        bs_cp_atom(tsa + 4u, dat + 32);
                    }
                    for (int h = 0; h < nch; h++) {
                        const int k = pol.stage_k(x.k0, x.k1, i + h, x.tile, x.ks);
                        const uint32_t tsa = tb + BS_SFA_COL0 + 8u * (uint32_t)(s * BS_CH + h), tsb = tbb + 8u * (uint32_t)k;
                        // descriptors: the start-address field is the low 14 bits (address >> 4)
                        const uint64_t da = da0 + (uint64_t)(((size_t)s * BS_STAGE + (size_t)h * BS_A_BYTES) >> 4);
                        const uint64_t db = dbg + (uint64_t)((k * BS_B_STAGE) >> 4);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const uint32_t sid = 2u * (uint32_t)(j & 1), g = 4u * (uint32_t)(j >> 1);
                            bs_mma(tacc + (uint32_t)((j & 1) * 2 * BS_ACC_COLS), da + 2 * j, db + 2 * j,
                                   (j & 1) ? id2 : id0, (tsa + g) | (sid << 30), (tsb + g) | (sid << 30),
                                   (i > 0 || h > 0 || j > 1) ? 1u : 0u);
                        }
                    }
                    tc_commit(&bb->empty[s]);
                    if (++s == nst) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                tc_commit(&bb->accfull[b]);
                // the group's last unit: its B rows are free once these MMAs are done (one
                // phase per group and buffer, so the stager's parity waits cannot alias)
                bool last = q + 1 == nseq;
                if (!last) {
                    BsUnit y;
                    pol.seq_unit(c, q + 1, y);
                    last = (y.d | (y.tg << 16) | (y.mode << 30)) != gkey;
                }
                if (last) tc_commit(&bb->bfree[gb]);
            }
            if (!ok) bs_fail(pol.err, BS_ERR_MMA);
            tc_commit(&bb->done);
            if (!mbar_wait(&bb->done, 0)) bs_fail(pol.err, BS_ERR_MMA);
        }
    } else if (warp < 6) {
        // ------------------------------------------------------ B stager
        // warps 2-5, once per token group g, into B buffer g % 2: after the MMAs of
        // group g - 2 (the buffer's last user) and, for a down group, its gate/up
        // tiles are done, the group's B rows (12 limbs per token and K chunk, 16-byte
        // async copies from L2 into the 128-byte-swizzled layout) and B scale words;
        // then, once the MMA issuer has copied group g - 1's atoms into TMEM, the B
        // atoms of every K chunk from the words (lane = B row).  After a timed-out
        // wait all four warps stop.
        const int t = tid - 64;
        const uint32_t *bw = reinterpret_cast<const uint32_t *>(bwreg);
        // limb rows 12..15 of both token slots of both buffers stay zero (never copied)
        for (int i = t; i < 2 * nk_max * BS_TOKG * (BS_LIMBS - BS_LQ) * 8; i += 128) {
            const int r = BS_LQ + (i >> 3) % (BS_LIMBS - BS_LQ), jk = (i >> 3) / (BS_LIMBS - BS_LQ);
            *reinterpret_cast<uint4 *>(bres + (size_t)(jk >> 1) * BS_B_STAGE + (jk & 1) * BS_B_TOK + r * 128 +
                                       (i & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        bool failed = false;
        int key = -1, ng = 0;
        for (int q = 0; q < nseq && !failed; q++) {
            BsUnit x;
            pol.seq_unit(c, q, x);
            const int gkey = x.d | (x.tg << 16) | (x.mode << 30);
            if (gkey == key) continue;
            key = gkey;
            const int gb = ng & 1;
            uint8_t *bdst = bres + gb * bbuf;
            if (t == 0) {
                bool okw = true;
                if (ng >= 2 && !mbar_wait(&bb->bfree[gb], (uint32_t)(((ng - 2) >> 1) & 1))) {
                    okw = false;
                    bs_fail(pol.err, 27);
                }
                if (okw && x.mode == 1 && !bs_tiles_done(pol.sync + 1 + x.v, tiles_need, true)) {
                    okw = false;
                    bs_fail(pol.err, 30);
                }
                stage_ok = okw;
            }
            named_bar_sync(2, 128);
            if (!stage_ok) {
                failed = true;
                break;
            }
            const BsPass P = pol.pass(x.mode);
            const int nt = pol.ntok(x.d, x.tg);
            const int src0 = pol.src_of(x.mode, x.d, x.tg, 0), src1 = nt > 1 ? pol.src_of(x.mode, x.d, x.tg, 1) : src0;
            for (int i = t, n = P.nk * nt * BS_LQ * 8; i < n; i += 128) {
                const int c16 = i & 7, l = (i >> 3) % BS_LQ, r = (i >> 3) / BS_LQ, j = r % nt, kk = r / nt;
                const int row = BS_LIMBS * (j ? src1 : src0) + l;
                cp_async16(bdst + (size_t)kk * BS_B_STAGE + (j * BS_LIMBS + l) * 128 + ((c16 ^ (l & 7)) << 4),
                           P.limbs + row * P.ld + kk * 128 + c16 * 16);
            }
            const int wv = P.g4 * BS_LIMBS / 4;  // 16-byte vectors of a token's words
            for (int i = t; i < nt * wv; i += 128) {
                const int j = i / wv, o = i - j * wv;
                cp_async16(bwreg + (size_t)i * 16, P.bsf + ((int64_t)(j ? src1 : src0) * P.g4 * BS_LIMBS + o * 4));
            }
            cp_async_wait_all();
            if (t == 0) {  // the shared atoms of group ng - 1 are in TMEM
                atoms_ok = ng == 0 || mbar_wait(&bb->batfree, (uint32_t)((ng - 1) & 1));
                if (!atoms_ok) bs_fail(pol.err, 28);
            }
            named_bar_sync(2, 128);  // every thread's words have landed
            if (!atoms_ok) {
                failed = true;
                break;
            }
            const int nrows = BS_LIMBS * nt;
            if (lane < nrows)
                for (int kk = warp - 2; kk < P.nk; kk += 4)
#pragma unroll
                    for (int h = 0; h < 2; h++)
                        *reinterpret_cast<uint32_t *>(batoms + (size_t)kk * BS_BATOMS + 512 * h + lane * 16) =
                            bw[((lane >> 4) * P.g4 + 2 * kk + h) * BS_LIMBS + (lane & 15)];
            fence_proxy_async_smem();  // the rows and atoms, for the tensor core's reads
            named_bar_sync(2, 128);
            if (t == 0) mbar_arrive(&bb->bready[gb]);
            ng++;
        }
        if (failed && t == 0) bs_fail(pol.err, BS_ERR_ATOMS);
    } else {
        // ------------------------------------------------------ epilogue
        const int ew = warp & 3, r = 32 * ew + lane;  // TMEM lane quadrant = warp % 4
        // after a timed-out wait a warp stops waiting and computing but keeps
        // taking part in the named barriers, so no other warp is left waiting
        bool failed = false;
        for (int q = 0; q < nseq; q++) {
            BsUnit x;
            pol.seq_unit(c, q, x);
            const int e = pol.ms->list[x.d];
            const uint8_t *eb = pol.expert(e);
            const int nt = pol.ntok(x.d, x.tg), b = q & 1;
            float bias = 0.f;
            if (x.mode == 0) {
                const int64_t f = (int64_t)x.tile * 64 + (r & 63);
                if (f < pol.L.ffn) bias = reinterpret_cast<const float *>(eb + pol.L.off[r < 64 ? 0 : 1][2])[f];
            } else {
                const int64_t row = (int64_t)x.tile * 128 + r;
                if (x.ks == 0 && row < pol.L.hidden) bias = reinterpret_cast<const float *>(eb + pol.L.off[2][2])[row];
            }
            if (!failed && !mbar_wait(&bb->accfull[b], (uint32_t)((q >> 1) & 1))) {
                failed = true;
                if (lane == 0) bs_fail(pol.err, BS_ERR_EPILOGUE);
            }
            tc_fence_after();
            float v[BS_TOKG];
#pragma unroll
            for (int j = 0; j < BS_TOKG; j++) {
                v[j] = 0.f;
                if (j < nt && !failed) {
                    float t[16], t2[16];
                    const uint32_t ta = tb + (uint32_t)(b * BS_ACC_COLS + BS_LIMBS * j) + ((uint32_t)(32 * ew) << 16);
                    tmem_ld16(ta, t);
                    tmem_ld16(ta + 2 * BS_ACC_COLS, t2);
                    float acc = t[0];
#pragma unroll
                    for (int i = 1; i < 16; i++) acc += t[i];
#pragma unroll
                    for (int i = 0; i < 16; i++) acc += t2[i];
                    v[j] = acc;
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0 && !failed) mbar_arrive(&bb->accempty[b]);
            if (x.mode == 0) {
                if (r >= 64)  // up values + up bias
#pragma unroll
                    for (int j = 0; j < BS_TOKG; j++) ex[(r - 64) * BS_TOKG + j] = __fadd_rn(v[j], bias);
                named_bar_sync(1, 128);
                if (r < 64 && !failed) {
                    const int64_t f = (int64_t)x.tile * 64 + r;
                    const bool valid = f < pol.L.ffn;
                    const int64_t fb = (int64_t)x.tile * 64 + 32 * ew;  // this warp's block of 32 features
#pragma unroll
                    for (int j = 0; j < BS_TOKG; j++) {
                        if (j >= nt) break;  // warp-uniform
                        const int slot = pol.slot_of(x.d, x.tg, j);
                        const float hv = valid ? bs_act(__fadd_rn(v[j], bias), ex[r * BS_TOKG + j], pol) : 0.f;
                        bs_limbs(hv, pol.hl + (int64_t)slot * BS_LIMBS * pol.hl_ld + fb / 2, pol.hl_ld,
                                 pol.hsf + (((int64_t)slot * pol.hg4 + fb / 128) * BS_LIMBS) * 4 + ((fb / 32) & 3));
                    }
                }
                named_bar_sync(1, 128);  // ex is read, and this tile's h limbs written, before what follows
                // the tile is done (also after a failed wait: the error word is set,
                // and the down units waiting for it end at once)
                if (r == 0) {
                    __threadfence();
                    atomicAdd(pol.sync + 1 + x.v, 1u);
                }
            } else if (!failed) {
                const int64_t row = (int64_t)x.tile * 128 + r;
                if (row < pol.L.hidden)
#pragma unroll
                    for (int j = 0; j < BS_TOKG; j++)
                        if (j < nt)
                            pol.y[((int64_t)x.ks * pol.n_tok * pol.top_k + pol.slot_of(x.d, x.tg, j)) * pol.L.hidden + row] =
                                __fadd_rn(v[j], bias);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tb, BS_TMEM_COLS);
    }
    // the last CTA to finish clears the tile counters for the next launch
    // (which starts after this grid has completed)
    if (tid == 0) {
        __threadfence();
        last_cta = atomicAdd(pol.sync, 1u) == gridDim.x - 1;
        __threadfence();
    }
    __syncthreads();
    if (last_cta) {
        for (int i = tid; i < nv; i += BS_THREADS) pol.sync[1 + i] = 0;
        if (tid == 0) pol.sync[0] = 0;
    }
}

// ---------------------------------------------------------- host side
static int bs_launch(const BsMapsK &maps, BsPol &pol, size_t ssb, cudaStream_t st) {
    cudaFuncAttributes fa{};
    MG_CUDA(cudaFuncGetAttributes(&fa, reinterpret_cast<const void *>(k_bsmoe)));
    ssb = (ssb + 127) & ~(size_t)127;
    const int nk_max = pol.ps[0].nk > pol.ps[1].nk ? pol.ps[0].nk : pol.ps[1].nk;
    for (int m = 0; m < 2; m++)
        MG_REQUIRE(pol.ps[m].nk >= 1 && pol.ps[m].nk <= BS_MAX_NK, MG_ERR_ARG,
                   "block-scaled MoE: K of %d chunks unsupported", pol.ps[m].nk);
    const size_t fixed = 1024 + (size_t)nk_max * (2 * BS_B_STAGE + BS_BATOMS) + ssb + 64 * BS_TOKG * 4 + sizeof(BsBars);
    const size_t budget = 227 * 1024 - fa.sharedSizeBytes;
    MG_REQUIRE(budget > fixed + 2 * (BS_STAGE + BS_CH * BS_ATOMS), MG_ERR_ARG, "block-scaled MoE: no room for a ring");
    int nst = (int)((budget - fixed) / (BS_STAGE + BS_CH * BS_ATOMS));
    if (nst > BS_MAX_STAGES) nst = BS_MAX_STAGES;
    const size_t smem = fixed + (size_t)nst * (BS_STAGE + BS_CH * BS_ATOMS);
    BS_TRY(ensure_smem_attr(reinterpret_cast<const void *>(k_bsmoe), smem));
    // programmatic dependent launch: this grid may start while the previous
    // kernel on the stream finishes; its producer waits for that grid
    // (griddepcontrol.wait) before reading its outputs
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)num_sms());
    cfg.blockDim = dim3(BS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    static const bool pdl = [] {
        const char *v = getenv("MIDGE_BS_PDL");
        return !(v && *v == '0');
    }();
    cfg.numAttrs = pdl ? 1 : 0;
    MG_CUDA(cudaLaunchKernelEx(&cfg, k_bsmoe, maps, pol, nst, (int)ssb));
    return MG_OK;
}

bool bsmoe_supported(const mg_expert_layout &L) {
    return L.dt == MG_MXFP4 && L.scale_fmt == MG_SCALE_UE8M0 && L.hidden % 64 == 0 && L.ffn % 64 == 0;
}

int bs_kpad(int64_t k) { return (int)((k + BS_KE - 1) / BS_KE * BS_KE); }
size_t bs_limb_bytes(int rows, int kpad) { return (size_t)rows * BS_LIMBS * (kpad / 2); }
size_t bs_word_bytes(int rows, int kpad) { return (size_t)rows * (kpad / 128) * BS_LIMBS * 4; }

size_t bs_atoms_bytes(const mg_expert_layout &L, int kpad_h, int kpad_f) {
    const int64_t units = (L.ffn / 64) * (kpad_h / BS_KE) + ((L.hidden + 127) / 128) * (kpad_f / BS_KE);
    return (size_t)units * 1024;
}

int bs_atoms_build(BsBuffers &b, const mg_expert_layout &L, const uint8_t *experts, int n_layers, int n_local,
                   cudaStream_t st) {
    MG_REQUIRE(bsmoe_supported(L) && b.atoms && n_layers > 0 && n_local > 0, MG_ERR_ARG,
               "block-scaled MoE: scale atoms need MXFP4 experts with ue8m0 scales");
    const int nk_h = b.kpad_h / BS_KE, nk_f = b.kpad_f / BS_KE;
    b.atoms_dn = (int)(L.ffn / 64) * nk_h;
    b.atoms_expert = (int64_t)bs_atoms_bytes(L, b.kpad_h, b.kpad_f);
    const int units = (int)(b.atoms_expert / 1024);
    const int64_t n_le = (int64_t)n_layers * n_local;
    dim3 g((unsigned)units, (unsigned)(n_le < 65535 ? n_le : 65535));
    k_bs_atoms<<<g, 256, 0, st>>>(experts, L, n_le, n_local, nk_h, nk_f, b.atoms_dn, b.atoms, b.atoms_expert);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int bs_buffers_init(BsBuffers &b) {
    // limbs zero everywhere and scale codes 127: the K pad and the unencoded
    // rows BS_LQ..BS_LIMBS-1 of every token keep them
    MG_CUDA(cudaMemset(b.xl, 0, bs_limb_bytes(8, b.kpad_h)));
    MG_CUDA(cudaMemset(b.xsf, 0x7F, bs_word_bytes(8, b.kpad_h)));
    MG_CUDA(cudaMemset(b.hl, 0, bs_limb_bytes(b.slots_max, b.kpad_f)));
    MG_CUDA(cudaMemset(b.hsf, 0x7F, bs_word_bytes(b.slots_max, b.kpad_f)));
    MG_CUDA(cudaMemset(b.sync, 0, bs_sync_bytes()));
    return MG_OK;
}

size_t bs_sync_bytes() { return (size_t)(1 + BS_MAX_V) * 4; }

int moe_bs(const MoeStreamArgs &a, cudaStream_t st) {
    const BsBuffers &B = *a.bs;
    const mg_expert_layout &L = a.L;
    MG_REQUIRE(bsmoe_supported(L) && a.maps && a.n_tok >= 1 && a.n_tok <= 8 && a.n_tok * a.top_k <= B.slots_max,
               MG_ERR_ARG, "block-scaled MoE: unsupported call");
    MG_REQUIRE(B.atoms && B.atoms_expert > 0, MG_ERR_STATE, "block-scaled MoE: expert scale atoms not built");
    MG_REQUIRE(B.sync, MG_ERR_STATE, "block-scaled MoE: no tile counters");
    int *err = stream_error_word();
    MG_REQUIRE(err, MG_ERR_OOM, "block-scaled MoE: no error word");
    {  // activations -> limbs
        const int warps = a.n_tok * (B.kpad_h / 32);
        k_bs_limbs<<<(warps * 32 + 255) / 256, 256, 0, st>>>(a.xb, L.hidden, a.n_tok, (int)L.hidden, B.kpad_h, B.xl,
                                                             reinterpret_cast<uint8_t *>(B.xsf));
        MG_CHECK_LAUNCH();
    }
    BsPol p{};
    p.L = L;
    p.experts_layer = a.experts_layer;
    p.layer = a.layer;
    p.e0 = a.e0;
    p.n_experts = a.n_experts;
    p.n_tok = a.n_tok;
    p.top_k = a.top_k;
    p.sel = a.sel;
    p.act_plain = a.act_plain;
    p.alpha = a.alpha;
    p.limit = a.limit;
    p.err = err;
    p.atoms = B.atoms + (int64_t)a.layer * a.n_experts * B.atoms_expert;
    p.atoms_expert = B.atoms_expert;
    p.sync = B.sync;
    // one launch, both passes.  gate/up: B = the expert's tokens' x limbs,
    // output: their h limbs; down: B = the expert's slots' h limbs
    BsMapsK mk{};
    for (int i = 0; i < 3; i++) mk.a[i] = a.maps[i];
    p.ps[0].limbs = B.xl;
    p.ps[0].ld = B.kpad_h / 2;
    p.ps[0].bsf = B.xsf;
    p.ps[0].g4 = B.kpad_h / 128;
    p.ps[0].nk = B.kpad_h / BS_KE;
    p.ps[0].atoms_u0 = 0;
    p.ps[1].limbs = B.hl;
    p.ps[1].ld = B.kpad_f / 2;
    p.ps[1].bsf = B.hsf;
    p.ps[1].g4 = B.kpad_f / 128;
    p.ps[1].nk = B.kpad_f / BS_KE;
    p.ps[1].atoms_u0 = B.atoms_dn;
    p.hl = B.hl;
    p.hsf = reinterpret_cast<uint8_t *>(B.hsf);
    p.hl_ld = B.kpad_f / 2;
    p.hg4 = B.kpad_f / 128;
    p.y = a.y;
    p.ks_count = a.down_ksplit_out;
    p.kst = (p.ps[1].nk + p.ks_count - 1) / p.ks_count;
    const int g4_max = p.ps[0].g4 > p.ps[1].g4 ? p.ps[0].g4 : p.ps[1].g4;
    return bs_launch(mk, p, (size_t)BS_TOKG * g4_max * BS_LIMBS * 4, st);
}

}  // namespace mg

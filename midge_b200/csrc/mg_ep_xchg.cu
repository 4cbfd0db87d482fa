// mg_ep_xchg.cu -- expert-parallel token exchange: the device side of the
// dispatch (tokens to the ranks that hold their routed experts) and of the
// combine (per-slot expert outputs back to the token's owner).  Data moves
// through buffers every rank maps into every other (CUDA IPC over NVLink).
//
// Prefill (variable sizes, one host agreement per layer and chunk):
//   plan     per destination rank d: the owner's tokens routed to any expert of
//            d (each token once per destination, in token order) and its slots
//            routed to d (in token order, then top-k rank order); counts,
//            send rows and the return row of every slot
//   pack     [normed row | top-k expert ids] per (token, destination)
//   -- copy-engine puts into each destination's receive buffer, a barrier --
//   retplan  on the expert side: the received tokens' local slots numbered in
//            received order (= per source, the source's own slot order), which
//            is where the DOWN GEMM writes each slot's output
//   -- puts of the outputs into each owner's return buffer, a barrier; the
//      owner adds them to the residual in ascending expert order
//      (k_pf_combine through ret_pos) --
// Decode (<= 8 tokens per step over all ranks; graph-captured): every rank
// stores its [row | ids] rows (fixed count per rank, pads carry id -1) into
// every rank's gather buffer, runs its experts over all gathered tokens, and
// stores each slot output of its experts into the owner's slot buffer; flags
// hand the data over (k_ep_dec_dispatch, k_ep_dec_return).
#include "mg_common.cuh"
#include "mg_ep.h"
#include "mg_ep_xchg.h"

namespace mg {

// ---------------------------------------------------------------- decode
__global__ void k_ep_dec_unpack(const float *__restrict__ recv, int64_t H, int k, int rowf, float *__restrict__ xb_all,
                                int32_t *__restrict__ sel_all) {
    const int r = blockIdx.x;
    const float *src = recv + (int64_t)r * rowf;
    for (int64_t c = threadIdx.x; c < H + k; c += blockDim.x) {
        if (c < H) xb_all[(int64_t)r * H + c] = src[c];
        else sel_all[(int64_t)r * k + (c - H)] = __float_as_int(src[c]);
    }
}

int ep_dec_unpack(const float *recv, int n_all, int64_t H, int k, int rowf, float *xb_all, int32_t *sel_all,
                  cudaStream_t st) {
    if (n_all <= 0) return MG_OK;
    k_ep_dec_unpack<<<n_all, 256, 0, st>>>(recv, H, k, rowf, xb_all, sel_all);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// ------------------------------------------------- decode over peer memory
// A rank's data reaches a peer by plain stores to the peer's mapped buffer;
// the hand-over is a flag the writer stores with release semantics at system
// scope after a system fence, and the reader polls with acquire semantics.
// The flag value is an epoch: a per-site counter in device memory that every
// rank advances identically (the last CTA of each exchange kernel), so the
// kernels replay correctly inside CUDA graphs.  Every poll is bounded (about a
// second); a wait that runs out sets the error word and the CTA moves on.
constexpr uint32_t EP_SPIN = 1u << 23;
constexpr int EP_ERR_SPIN = 41;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// thread 0: publish to rank d, wait for source d, and (last CTA) advance the epoch
__device__ void ep_handover(const EpDecPeers &p, int site, uint32_t ep, int me, int d, int G) {
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(p.flag[d] + site * EP_MAX_WORLD + me, ep);
        bool ok = false;
        for (uint32_t i = 0; i < EP_SPIN; i++) {
            if (ld_acquire_sys(p.flag[me] + site * EP_MAX_WORLD + d) == ep) { ok = true; break; }
            __nanosleep(64);
        }
        if (!ok) atomicCAS(p.err, 0, EP_ERR_SPIN);
        __threadfence();
        if (atomicAdd(p.seq + 2 + site, 1u) == (unsigned)G - 1) {
            p.seq[2 + site] = 0;
            p.seq[site] = ep;
        }
    }
    __syncthreads();
}

// CTA d: this rank's n_max rows [normed row | ids | pad] into rank d's buffer
__global__ void k_ep_dec_dispatch(EpDecPeers p, const float *__restrict__ xb, const int32_t *__restrict__ sel, int n,
                                  int nmax, int64_t H, int k, int rowf, int me, int G) {
    const int d = blockIdx.x;
    const uint32_t ep = *reinterpret_cast<volatile uint32_t *>(p.seq) + 1;
    float *dst = p.recv[d] + (int64_t)me * nmax * rowf;
    for (int r = 0; r < nmax; r++) {
        const bool real = r < n;
        for (int64_t c = threadIdx.x; c < rowf; c += blockDim.x) {
            float v;
            if (c < H) v = real ? xb[(int64_t)r * H + c] : 0.f;
            else if (c < H + k) v = __int_as_float(real ? sel[(int64_t)r * k + (c - H)] : -1);
            else v = 0.f;
            dst[(int64_t)r * rowf + c] = v;
        }
    }
    ep_handover(p, 0, ep, me, d, G);
}

// CTA d: the outputs of this rank's experts for owner d's tokens into d's moe_y
__global__ void k_ep_dec_return(EpDecPeers p, const float *__restrict__ y_all, const int32_t *__restrict__ sel_all,
                                int nmax, int64_t H, int k, int ks, int64_t plane_all, int64_t plane_loc, int e0,
                                int n_local, int me, int G) {
    const int d = blockIdx.x;
    const uint32_t ep = *reinterpret_cast<volatile uint32_t *>(p.seq + 1) + 1;
    for (int j = 0; j < nmax; j++) {
        const int r = d * nmax + j;
        for (int i = 0; i < k; i++) {
            const int e = sel_all[(int64_t)r * k + i] - e0;
            if (e < 0 || e >= n_local) continue;  // uniform over the block
            for (int q = 0; q < ks; q++) {
                const float4 *src = reinterpret_cast<const float4 *>(y_all + q * plane_all + ((int64_t)r * k + i) * H);
                float4 *dst = reinterpret_cast<float4 *>(p.y[d] + q * plane_loc + ((int64_t)j * k + i) * H);
                for (int64_t c = threadIdx.x; c < H / 4; c += blockDim.x) dst[c] = src[c];
            }
        }
    }
    ep_handover(p, 1, ep, me, d, G);
}

int ep_dec_dispatch(const EpDecPeers &p, const float *xb, const int32_t *sel, int n, int n_max, int64_t H, int k,
                    int rowf, int me, int G, cudaStream_t st) {
    MG_REQUIRE(G >= 2 && G <= EP_MAX_WORLD && n_max >= 1, MG_ERR_ARG, "ep_dec_dispatch: bad arguments");
    k_ep_dec_dispatch<<<G, 256, 0, st>>>(p, xb, sel, n, n_max, H, k, rowf, me, G);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

int ep_dec_return(const EpDecPeers &p, const float *y_all, const int32_t *sel_all, int n_max, int64_t H, int k, int ks,
                  int64_t plane_all, int64_t plane_loc, int e0, int n_local, int me, int G, cudaStream_t st) {
    MG_REQUIRE(G >= 2 && G <= EP_MAX_WORLD && n_max >= 1 && H % 4 == 0, MG_ERR_ARG, "ep_dec_return: bad arguments");
    k_ep_dec_return<<<G, 256, 0, st>>>(p, y_all, sel_all, n_max, H, k, ks, plane_all, plane_loc, e0, n_local, me, G);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// --------------------------------------------------------------- prefill
constexpr int XG_PLAN_THREADS = 1024;

// Inclusive scan over the block of NQ ints per thread; `tot` receives the
// exclusive prefix of this thread's warp (per quantity); warp totals go
// through shared memory.  Returns nothing; v[] becomes the inclusive scan
// within the warp.
template <int NQ>
__device__ __forceinline__ void plan_block_scan(int (&v)[NQ], int (&wofs)[NQ], int (*s_warp)[NQ]) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const int a = __shfl_up_sync(0xffffffffu, v[q], off);
            if (lane >= off) v[q] += a;
        }
    }
    if (lane == 31)
#pragma unroll
        for (int q = 0; q < NQ; q++) s_warp[wid][q] = v[q];
    __syncthreads();
    if (wid == 0) {
#pragma unroll
        for (int q = 0; q < NQ; q++) {
            const int orig = lane < nw ? s_warp[lane][q] : 0;
            int x = orig;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, x, off);
                if (lane >= off) x += a;
            }
            if (lane < nw) s_warp[lane][q] = x - orig;  // exclusive warp offsets
        }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < NQ; q++) wofs[q] = s_warp[wid][q];
}

// One block.  counts[0..G) tokens and counts[G..2G) slots per destination;
// send_row[t*G + d]: row of (t, d) in the destination-major send buffer or -1;
// ret_pos[t*k + i]: row of slot (t, i) in the destination-major return buffer
// or -1 (expert id out of range).
__global__ void __launch_bounds__(XG_PLAN_THREADS)
    k_ep_pf_plan(const int32_t *__restrict__ sel, int n, int k, int G, int per, int n_experts, int *counts,
                 int *send_row, int *ret_pos) {
    constexpr int MG_ = EP_MAX_WORLD, NQ = 2 * EP_MAX_WORLD;
    __shared__ int s_tot[NQ], s_off[NQ], s_run[NQ];
    __shared__ int s_warp[32][NQ];
    const int tid = threadIdx.x;
    if (tid < NQ) { s_tot[tid] = 0; s_run[tid] = 0; }
    __syncthreads();
    for (int t = tid; t < n; t += blockDim.x) {
        int c[MG_] = {};
        for (int i = 0; i < k; i++) {
            const int e = sel[(int64_t)t * k + i];
            if (e >= 0 && e < n_experts) c[e / per]++;
        }
#pragma unroll
        for (int d = 0; d < MG_; d++)
            if (c[d]) { atomicAdd(&s_tot[d], 1); atomicAdd(&s_tot[MG_ + d], c[d]); }
    }
    __syncthreads();
    if (tid == 0) {
        int a = 0, b = 0;
        for (int d = 0; d < G; d++) {
            s_off[d] = a; a += s_tot[d];
            s_off[MG_ + d] = b; b += s_tot[MG_ + d];
            counts[d] = s_tot[d];
            counts[G + d] = s_tot[MG_ + d];
        }
    }
    __syncthreads();
    for (int base = 0; base < n; base += blockDim.x) {
        const int t = base + tid;
        int c[MG_] = {};
        if (t < n)
            for (int i = 0; i < k; i++) {
                const int e = sel[(int64_t)t * k + i];
                if (e >= 0 && e < n_experts) c[e / per]++;
            }
        int v[NQ], wofs[NQ];
#pragma unroll
        for (int d = 0; d < MG_; d++) { v[d] = c[d] > 0; v[MG_ + d] = c[d]; }
        plan_block_scan<NQ>(v, wofs, s_warp);
        if (t < n) {
            for (int d = 0; d < G; d++)
                send_row[(int64_t)t * G + d] = c[d] ? s_off[d] + s_run[d] + wofs[d] + v[d] - 1 : -1;
            int seen[MG_] = {};
            for (int i = 0; i < k; i++) {
                const int e = sel[(int64_t)t * k + i];
                int r = -1;
                if (e >= 0 && e < n_experts) {
                    const int d = e / per;
                    r = s_off[MG_ + d] + s_run[MG_ + d] + wofs[MG_ + d] + (v[MG_ + d] - c[d]) + seen[d]++;
                }
                ret_pos[(int64_t)t * k + i] = r;
            }
        }
        __syncthreads();
        if (tid == blockDim.x - 1)  // chunk totals: the last thread's inclusive values
#pragma unroll
            for (int q = 0; q < NQ; q++) s_run[q] += wofs[q] + v[q];
        __syncthreads();
    }
}

int ep_pf_plan(const int32_t *sel, int n, int k, int G, int per, int n_experts, int *counts, int *send_row,
               int *ret_pos, cudaStream_t st) {
    MG_REQUIRE(G >= 1 && G <= EP_MAX_WORLD && per >= 1 && k >= 1 && k <= 16, MG_ERR_ARG, "ep_pf_plan: bad arguments");
    k_ep_pf_plan<<<1, XG_PLAN_THREADS, 0, st>>>(sel, n, k, G, per, n_experts, counts, send_row, ret_pos);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// one block per token: [normed row | expert ids | zero pad] to every destination it has
__global__ void k_ep_pf_pack(const float *__restrict__ xb, const int32_t *__restrict__ sel, int k, int G, int64_t H,
                             int rowf, const int *__restrict__ send_row, float *__restrict__ send) {
    const int t = blockIdx.x;
    for (int d = 0; d < G; d++) {
        const int r = send_row[(int64_t)t * G + d];
        if (r < 0) continue;
        float4 *dst = reinterpret_cast<float4 *>(send + (int64_t)r * rowf);
        const float4 *src = reinterpret_cast<const float4 *>(xb + (int64_t)t * H);
        for (int64_t c = threadIdx.x; c < H / 4; c += blockDim.x) dst[c] = src[c];
        for (int64_t c = H + threadIdx.x; c < rowf; c += blockDim.x)
            send[(int64_t)r * rowf + c] = c < H + k ? __int_as_float(sel[(int64_t)t * k + (c - H)]) : 0.f;
    }
}

int ep_pf_pack(const float *xb, const int32_t *sel, int n, int k, int G, int64_t H, int rowf, const int *send_row,
               float *send, cudaStream_t st) {
    if (n <= 0) return MG_OK;
    MG_REQUIRE(H % 4 == 0 && rowf % 4 == 0, MG_ERR_ARG, "ep_pf_pack: rows must be multiples of 4 floats");
    k_ep_pf_pack<<<n, 256, 0, st>>>(xb, sel, k, G, H, rowf, send_row, send);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

__global__ void k_ep_pf_unpack_sel(const float *__restrict__ recv, int64_t total, int k, int64_t H, int rowf,
                                   int32_t *__restrict__ sel_recv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t j = i / k, q = i - j * k;
        sel_recv[i] = __float_as_int(recv[j * rowf + H + q]);
    }
}

int ep_pf_unpack_sel(const float *recv, int n_recv, int k, int64_t H, int rowf, int32_t *sel_recv, cudaStream_t st) {
    if (n_recv <= 0) return MG_OK;
    const int64_t total = (int64_t)n_recv * k;
    int g = ceil_div(total, 256);
    if (g > 148 * 8) g = 148 * 8;
    k_ep_pf_unpack_sel<<<g, 256, 0, st>>>(recv, total, k, H, rowf, sel_recv);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// One block: the received slots whose expert is local, numbered in received
// order (slot order within a token); -1 for the others.
__global__ void __launch_bounds__(XG_PLAN_THREADS)
    k_ep_pf_retplan(const int32_t *__restrict__ sel_recv, int n_recv, int k, int e0, int n_local, int *ret_row) {
    __shared__ int s_warp[32][1];
    __shared__ int s_run;
    if (threadIdx.x == 0) s_run = 0;
    __syncthreads();
    for (int base = 0; base < n_recv; base += blockDim.x) {
        const int j = base + threadIdx.x;
        int c = 0;
        if (j < n_recv)
            for (int i = 0; i < k; i++) {
                const int e = sel_recv[(int64_t)j * k + i] - e0;
                c += e >= 0 && e < n_local;
            }
        int v[1] = {c}, wofs[1];
        plan_block_scan<1>(v, wofs, s_warp);
        if (j < n_recv) {
            int r = s_run + wofs[0] + v[0] - c;
            for (int i = 0; i < k; i++) {
                const int e = sel_recv[(int64_t)j * k + i] - e0;
                ret_row[(int64_t)j * k + i] = (e >= 0 && e < n_local) ? r++ : -1;
            }
        }
        __syncthreads();
        if (threadIdx.x == blockDim.x - 1) s_run += wofs[0] + v[0];
        __syncthreads();
    }
}

int ep_pf_retplan(const int32_t *sel_recv, int n_recv, int k, int e0, int n_local, int *ret_row, cudaStream_t st) {
    if (n_recv <= 0) return MG_OK;
    k_ep_pf_retplan<<<1, XG_PLAN_THREADS, 0, st>>>(sel_recv, n_recv, k, e0, n_local, ret_row);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

// DOWN output row of every expert-major position: the return row of its slot
__global__ void k_ep_pf_remap(const int *__restrict__ slot_of_pos, const int *__restrict__ offs_end,
                              const int *__restrict__ ret_row, int max_p, int *__restrict__ slot2) {
    const int P = min(*offs_end, max_p);
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < P; p += gridDim.x * blockDim.x)
        slot2[p] = ret_row[slot_of_pos[p]];
}

int ep_pf_remap(const int *slot_of_pos, const int *offs_end, const int *ret_row, int max_p, int *slot2,
                cudaStream_t st) {
    if (max_p <= 0) return MG_OK;
    int g = ceil_div(max_p, 256);
    if (g > 148 * 8) g = 148 * 8;
    k_ep_pf_remap<<<g, 256, 0, st>>>(slot_of_pos, offs_end, ret_row, max_p, slot2);
    MG_CHECK_LAUNCH();
    return MG_OK;
}

}  // namespace mg

// mg_ep_xchg.h -- launchers of the expert-parallel token exchange kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

// decode: gathered rows [normed row (H) | top-k ids (k, as int bits) | pad] -> rows and ids
int ep_dec_unpack(const float *recv, int n_all, int64_t H, int k, int rowf, float *xb_all, int32_t *sel_all,
                  cudaStream_t st);

// prefill: see mg_ep_xchg.cu
int ep_pf_plan(const int32_t *sel, int n, int k, int G, int per, int n_experts, int *counts, int *send_row,
               int *ret_pos, cudaStream_t st);
int ep_pf_pack(const float *xb, const int32_t *sel, int n, int k, int G, int64_t H, int rowf, const int *send_row,
               float *send, cudaStream_t st);
int ep_pf_unpack_sel(const float *recv, int n_recv, int k, int64_t H, int rowf, int32_t *sel_recv, cudaStream_t st);
int ep_pf_retplan(const int32_t *sel_recv, int n_recv, int k, int e0, int n_local, int *ret_row, cudaStream_t st);
int ep_pf_remap(const int *slot_of_pos, const int *offs_end, const int *ret_row, int max_p, int *slot2,
                cudaStream_t st);

// Decode over peer memory (NVLink): every rank's buffers mapped into every
// rank (CUDA IPC).  flag[d] = rank d's hand-over flags [2 sites][EP_MAX_WORLD
// sources]; seq = this rank's epoch counters [2] and CTA tickets [2].
struct EpDecPeers {
    float *recv[8];      // rank d's gather buffer: rows [source * n_max + j][rowf]
    float *y[8];         // rank d's MoE slot outputs (moe_y)
    uint32_t *flag[8];
    uint32_t *seq;
    int *err;
};
// rows of this rank's n tokens (pads to n_max) into every rank's gather
// buffer, then the hand-over; returns when every rank's rows are here
int ep_dec_dispatch(const EpDecPeers &p, const float *xb, const int32_t *sel, int n, int n_max, int64_t H, int k,
                    int rowf, int me, int G, cudaStream_t st);
// the slot outputs of this rank's experts (y_all, gathered-token layout) into
// each owner's moe_y; returns when every rank's outputs for this rank's tokens are here
int ep_dec_return(const EpDecPeers &p, const float *y_all, const int32_t *sel_all, int n_max, int64_t H, int k, int ks,
                  int64_t plane_all, int64_t plane_loc, int e0, int n_local, int me, int G, cudaStream_t st);

// floats per packed row: hidden + top-k ids, rounded up to 16 bytes
inline int ep_rowf(int64_t H, int k) { return (int)((H + k + 3) / 4 * 4); }

}  // namespace mg

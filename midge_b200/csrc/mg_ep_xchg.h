// mg_ep_xchg.h -- launchers of the expert-parallel token exchange kernels.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

// decode: fixed-size rows [normed row (H) | top-k ids (k, as int bits) | pad] per token
int ep_dec_pack(const float *xb, const int32_t *sel, int n, int n_max, int64_t H, int k, int rowf, float *send,
                cudaStream_t st);
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

// floats per packed row: hidden + top-k ids, rounded up to 16 bytes
inline int ep_rowf(int64_t H, int k) { return (int)((H + k + 3) / 4 * 4); }

}  // namespace mg

// mg_prefill.h -- launchers of the tensor-core prefill path.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "mg_ep.h"
#include "mg_gemm.h"
#include "midgecuda.h"

namespace mg {

struct MoePrefill {
    mg_expert_layout L;
    const uint8_t *experts_layer;
    const int *rebase;  // this layer's [E x 3] rebase exponents
    int n, top_k, n_experts;  // n_experts: all experts (sel holds global ids)
    int e0, n_local;          // this rank's experts [e0, e0 + n_local), the ones in experts_layer
    const int32_t *sel;
    const float *w;
    const float *xb;    // [n x hidden] normed inputs
    float *x;           // [n x hidden] residual, accumulated into
    int act_plain;
    float alpha, limit;
    // scratch
    int *counts, *offs, *cursor, *ntiles, *pos_of_slot, *slot_of_pos;
    XgTile *tiles;
    __half *x_hi, *x_lo;  // [n*top_k x hidden]
    __half *h_hi, *h_lo;  // [n*top_k x ffn]
    float *y;             // [n*top_k x hidden], slot-major
    int *err;
    // expert-parallel form (moe_prefill_experts): xb rows at stride ldx
    // (0: hidden), and the DOWN output of slot s at row out_row[s] of y
    // (null: slot-major); slot2 is scratch for the remapped positions
    int64_t ldx;
    const int *out_row;
    int *slot2;
};
// the whole MoE block of a prefill chunk on one rank (experts + combine)
int moe_prefill(const MoePrefill &a, cudaStream_t st);
// only the routed experts: count, tile, gather, GATEUP, DOWN (no combine)
int moe_prefill_experts(const MoePrefill &a, cudaStream_t st);
// x[t] += w * Y[row(t, i)] per routed expert in ascending expert id;
// row(t, i) = slot_row ? slot_row[t*top_k + i] : t*top_k + i
int pf_combine(float *x, int64_t H, const int32_t *sel, const float *w, int n, int top_k, int n_experts, const float *Y,
               const int *slot_row, cudaStream_t st);

struct DenseGemm {
    const void *w, *scales;  // q8r matrix [rows x cols], f32 row scales
    const float *bias;
    int64_t rows, cols;
    const __half *x_hi, *x_lo;  // [n x cols]
    int n;
    float *y;
    int64_t ldy;
    int accumulate;
    int *err;
};
int dense_gemm(const DenseGemm &d, cudaStream_t st);

int split_rows(const float *x, int64_t ldx, int n, int64_t K, __half *hi, __half *lo, cudaStream_t st);
int pf_rebase(const uint8_t *experts, const mg_expert_layout &L, int n_layers, int n_experts, int *rebase, int *inexact,
              cudaStream_t st);

}  // namespace mg

// mg_kernels.h -- host-side launchers shared by the C ABI and the model.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "midgecuda.h"

namespace mg {

void set_error(const char *fmt, ...);

int gemv(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols, const float *x,
         int64_t ldx, int n_tok, const float *bias, int accumulate, float *y, int64_t ldy, cudaStream_t st);
size_t gemv_smem_bytes(int cols, int mt, int nt);
int dequant_rows(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols,
                 const int32_t *ids, int n, float *out, cudaStream_t st);
int scales_to_ue8m0(const uint16_t *f16, uint8_t *ue8m0, int64_t n, int *n_inexact, cudaStream_t st);
int rmsnorm(const float *x, const float *w, float *out, int64_t n, int n_rows, float eps, cudaStream_t st);
int to_f16_ftz(const float *x, uint16_t *out, int64_t n, cudaStream_t st);

// streamed (bulk-copy ring) GEMV over up to 3 row-concatenated matrices
// TMA tensor maps of weight matrices (row bytes x rows [x experts x layers])
int map_weights_2d(CUtensorMap *map, const void *base, int64_t rowbytes, int64_t rows, int box_rows);
int map_weights_4d(CUtensorMap *map, const void *base, int64_t rowbytes, int64_t rows, int64_t n_experts,
                   int64_t n_layers, int64_t expert_stride, int64_t layer_stride, int box_rows);
void *encode_tiled_fn();

struct StreamMat {
    const CUtensorMap *map;  // 2-D map of w (box 128 B x 128 rows); built here when null
    const void *w, *scales;
    const float *bias;
    int64_t rows;
    float *y;      // outputs (ksplit == 1) or partial planes (ksplit > 1)
    int64_t ldy;
};
struct StreamGemvArgs {
    int dt, scale_fmt;
    StreamMat mat[3];
    int nmat;
    int64_t cols;
    const float *x;
    int64_t ldx;
    int n_tok;            // <= 8
    int accumulate;       // ksplit == 1 only
    int ksplit;           // K splits (partials written to y + ks*part_stride)
    int64_t part_stride;
    unsigned long long *amax;  // optional (ksplit == 1): per-token packed first-maximum of the outputs
};
int stream_gemv(const StreamGemvArgs &a, cudaStream_t st);

struct BsBuffers;
struct MoeStreamArgs {
    mg_expert_layout L;
    const CUtensorMap *maps;  // gate (box 64 rows), up (64), down (128): 4-D over all experts and layers
    int layer;
    const uint8_t *experts_layer;
    int e0;  // global id of local expert 0 (sel holds global ids)
    int n_experts, n_tok, top_k;
    const int32_t *sel;
    const float *xb;      // [n_tok x hidden]
    int act_plain;
    float alpha, limit;
    float *h;             // [n_tok*top_k x ffn]
    float *y;             // [down_ksplit x n_tok*top_k x hidden]
    int down_ksplit;      // requested
    int down_ksplit_out;  // what moe_down_ksplit() returned for it
    const BsBuffers *bs;  // block-scaled tensor-core kernels (MXFP4, ue8m0), or null
};
int moe_stream(const MoeStreamArgs &a, cudaStream_t st);
int moe_down_ksplit(const mg_expert_layout &L, int want);

struct CombineNormArgs {
    const float *x_in;     // residual before the MoE (null: x itself)
    float *x;              // [n_tok x hidden] residual out (x_in + MoE when y != null)
    const float *y;        // MoE partials [ksplit x n_tok*top_k x hidden] or null
    int ksplit;
    const int32_t *sel;
    const float *w;
    int n_tok, top_k, n_experts;
    int64_t hidden;
    const float *nw;       // norm weight
    float eps;
    float *xb;             // normed output (may be null)
    int64_t plane;         // floats between the K-split planes of y (0: n_tok*top_k*hidden)
    int pdl;               // launched dependent on the MoE grid: slots, weights, residual and norm weight
                           // are read before its wait (they must not come from the grid just before)
};
int combine_norm(const CombineNormArgs &a, cudaStream_t st);
int sum_parts(const float *part, int ks, int64_t plane, int n_tok, int64_t rows, int64_t ldp, float *out, int64_t ldo,
              int accumulate, cudaStream_t st);
// temperature / top-p sampling of n_rows logits rows (mg_sample.cu)
int sample_topp(const float *logits, int64_t ldl, int64_t V, int n_rows, float temp, float topp, uint64_t *rng,
                int32_t *out, float *probs, cudaStream_t st);
int stream_error_check();
int stream_prepare();
int *stream_error_word();
int stream_ksplit(int dt, int64_t cols, int want);  // effective K split for a row of `cols`

// router: norm (optional) + AVX2-order f32 logits + top-k + weights + usage
struct RouterArgs {
    const float *x;        // [n_tok x hidden] residual rows (normed here if norm_w != null)
    const float *norm_w;   // mlp norm weight or null (then x is already normed)
    float eps;
    float *xb_out;         // normed rows out (may be null when norm_w == null)
    const float *rw, *rb;  // router weight [E x hidden] f32, bias [E]
    int n_experts, top_k, router_norm, variant;
    int64_t hidden;
    int n_tok;
    float *logits;         // [n_tok x E] (may be null)
    int32_t *sel;          // [n_tok x top_k]
    float *weights;        // [n_tok x top_k]
    uint32_t *usage;       // [E] counters of this layer, or null
    const float *x_parts;  // if set: the residual is x + sum_ks x_parts[ks]; written to x_out
    float *x_out;
    int x_parts_ks;
    int64_t x_parts_stride;
    int *err;              // decode router: error word set when a bounded wait gives up (may be null)
    int pdl;               // decode router: logits launched dependent on the norm kernel (weights
                           // staged before the wait)
};
int router(const RouterArgs &a, cudaStream_t st);
int router_split(const RouterArgs &a, float *logits_scratch, unsigned *ticket, cudaStream_t st);  // decode
int router_batch(const RouterArgs &a, float *logits_scratch, cudaStream_t st);                     // prefill

// decode MoE FFN (gate/up + activation, then down + rank-order combine)
struct MoeArgs {
    mg_expert_layout L;            // by value: read on the device
    const uint8_t *experts_layer;  // this layer's first expert
    int n_experts;
    const float *xb;  // [n_tok x hidden] normed inputs
    int n_tok, top_k;
    const int32_t *sel;
    const float *weights;
    int act_plain;
    float alpha, limit;
    float *h;  // [n_tok*top_k x ffn] scratch
    float *x;  // [n_tok x hidden] residual, accumulated into
    int64_t ldx;
};
int moe_decode(const MoeArgs &a, cudaStream_t st);

}  // namespace mg

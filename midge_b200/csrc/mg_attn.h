// mg_attn.h -- argument blocks of the attention launchers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace mg {

struct QkvPostArgs {
    float *q, *k;          // [n_tok x ldq], [n_tok x ldk], modified in place
    const float *v;        // [n_tok x ldk]
    int64_t ldq, ldk;
    int n_heads, n_kv_heads, head_dim;
    const float *qn, *kn;  // qk-norm weights or null
    float eps;
    const float *rope_cos, *rope_sin;  // [ctx x head_dim/2]
    const int32_t *tok_pos;            // [n_tok] positions
    const int32_t *tok_seq;            // [n_tok] sequence ids (null = 0)
    int write_cache;
    uint16_t *kc, *vc;                 // layer cache [max_seqs x cap x kv_dim]
    int cap;
    uint16_t *tmp_k, *tmp_v;           // optional [n_tok x kv_dim] f16 copies
    // optional: q, k, v are the sums of ks K-split planes (plane stride
    // `plane`, rows as q/k/v) and written to q, k and v_out (qkv_post_parts)
    int pdl;  // launched dependent on the q/k/v GEMV: positions, sequences and RoPE values read before the wait
    const float *parts;
    int ks;
    int64_t plane;
    float *v_out;
};
int qkv_post(const QkvPostArgs &a, int n_tok, cudaStream_t st);
int qkv_post_parts(const QkvPostArgs &a, int n_tok, cudaStream_t st);

struct AttnDecodeArgs {
    const float *q;  // [n_seqs x ldq]
    int64_t ldq;
    const int32_t *seq_ids, *pos;  // per decode row: sequence, position of the token
    const uint16_t *kc, *vc;
    int cap, n_heads, n_kv_heads, head_dim;
    float scale;
    const float *sinks;  // [n_heads] or null
    int split_len, max_splits;
    float *partial;      // [n_seqs x n_heads x max_splits x (hd+2)]
    float *out;          // [n_seqs x ldo]
    int64_t ldo;
    int use_tc;          // head_dim 64, split_len 64: the tensor-core kernel
    int pdl;             // the combine launched dependent on the attention grid
};
int attn_decode(const AttnDecodeArgs &a, int n_seqs, cudaStream_t st);

struct AttnPrefillArgs {
    const float *q;  // [n x ldq] after rope
    int64_t ldq;
    const uint16_t *tmp_k, *tmp_v;  // [n x kv_dim] this chunk's f16 K/V
    const uint16_t *kc, *vc;        // layer cache
    int seq, pos0, n, cap, n_heads, n_kv_heads, head_dim;
    float scale;
    const float *sinks;
    float *out;
    int64_t ldo;
    int use_tc;  // head_dim 64: the tensor-core kernel
};
int attn_prefill(const AttnPrefillArgs &a, cudaStream_t st);

}  // namespace mg

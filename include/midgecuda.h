/* midgecuda.h -- C ABI of libmidgecuda.so, the sm_100a quantized-MoE hot path.
 *
 * The reference engine (drmihirbrahme/midge) calls its kernels directly as
 * static C functions; this header is the seam a C host binds instead.  Each
 * entry point names the reference interface it replaces (file:line within the
 * reference project).  Conventions:
 *   - every function returns MG_OK (0) or a negative MG_ERR_* code and never
 *     exits the process; mg_last_error() gives the message of the calling
 *     thread's last failure;
 *   - "kernel level" functions take DEVICE pointers and a cudaStream_t passed
 *     as void* (NULL = legacy default stream); they are asynchronous;
 *   - "model level" functions take HOST pointers and synchronise before they
 *     return; one host thread drives one mg_model.
 * Weight dtypes and byte layouts are exactly the midge container's
 * (engine/mten.h:24-31): q8r = int8 rows + f32 row scales; q4g32 / mxfp4 =
 * packed nibbles (low nibble = even column) + one scale per 32 columns.
 */
#ifndef MIDGECUDA_H
#define MIDGECUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* weight dtypes: same codes as engine/mten.h:42, plus MG_MXFP4_E8, the
 * opt-in "mxfp4e8" expert container dtype (no counterpart in the reference,
 * whose converter writes f16 group scales, tools/convert.py:37-53): MXFP4
 * nibbles with one ue8m0 byte (2^(u-127), 0 = zero) per 32 columns, written
 * by midge_b200/convert_ue8m0.py and uploaded without re-expression.  An
 * mg_expert_layout of that dtype reports dt MG_MXFP4, scale_fmt
 * MG_SCALE_UE8M0. */
enum { MG_F32 = 0, MG_Q8R = 1, MG_Q4G32 = 2, MG_MXFP4 = 3, MG_MXFP4_E8 = 4 };
/* encoding of the per-32-column scales of q4g32/mxfp4 */
enum { MG_SCALE_F16 = 0, MG_SCALE_UE8M0 = 1 };

enum {
    MG_OK = 0,
    MG_ERR_ARG = -1,     /* bad argument */
    MG_ERR_CUDA = -2,    /* CUDA runtime error */
    MG_ERR_OOM = -3,     /* device allocation failed */
    MG_ERR_STATE = -4,   /* call out of order (e.g. forward before ready) */
    MG_ERR_RANGE = -5,   /* context full or token out of range: the reference exits 4 (engine/midge.c:554-555) */
    MG_ERR_SPEC = -6,    /* bad spec / missing tensor: the reference exits 3 (engine/midge.c:136,195-201) */
    MG_ERR_TIMEOUT = -8, /* a bounded device wait gave up */
    MG_ERR_COMM = -9     /* expert-parallel communication failed */
};

const char *mg_last_error(void);
int mg_version(void);

/* ===================================================== kernel level ==== */

/* y[t][r] = sum_c W[r][c] * x[t][c] (+ bias[r]) for t < n_tok; y may also be
 * accumulated into (accumulate != 0: y += result).  fp32 accumulation.
 * Replaces wk_matvec (engine/mkern.h:180) followed by wk_addbias
 * (engine/mkern.h:245), batched over n_tok <= 256 input vectors (one weight
 * pass per group of up to 16 vectors).
 * q4g32/mxfp4 need cols % 32 == 0; q8r needs cols % 64 == 0 or falls back to
 * the generic path; x rows have stride ldx floats, y rows stride ldy. */
int mg_gemv(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows, int64_t cols,
            const float *x, int64_t ldx, int n_tok, const float *bias, int accumulate, float *y,
            int64_t ldy, void *stream);

/* out[i][:] = dequantised row ids[i] of W; replaces wk_row (engine/mkern.h:201). */
int mg_dequant_rows(int dt, int scale_fmt, const void *w, const void *scales, int64_t rows,
                    int64_t cols, const int32_t *ids, int n, float *out, void *stream);

/* Re-express power-of-two f16 group scales as ue8m0 bytes (2^(u-127); u = 0
 * for a zero scale).  *n_inexact (device int, accumulated) counts scales that
 * are not a positive power of two or zero; those bytes are left 0.  Exact for
 * every scale the midge converter writes (tools/convert.py:37-53). */
int mg_scales_to_ue8m0(const uint16_t *f16, uint8_t *ue8m0, int64_t n, int *n_inexact, void *stream);

/* out = x * (1/sqrt(mean(x^2)+eps)) * w per row of n; replaces wk_rmsnorm
 * (engine/mkern.h:238).  Parallel sum: equal to the reference within fp32
 * rounding of the sum of squares. */
int mg_rmsnorm(const float *x, const float *w, float *out, int64_t n, int n_rows, float eps, void *stream);

/* float -> f16 with the reference's subnormal flush (engine/mkern.h:261). */
int mg_to_f16_ftz(const float *x, uint16_t *out, int64_t n, void *stream);

/* Router for n_tok normed rows xb: logits = Wr * xb + b with the f32 weight
 * reduced in the reference's AVX2 lane order (engine/mkern.h:85-99), so the
 * logits and the selected experts are bit-identical to the reference for the
 * same xb; then top-k and routing weights.  variant 0 = decode top-k
 * (engine/midge.c:476-486), 1 = batched-prefill top-k (engine/midge.c:410-422);
 * router_norm as engine/midge.c:423-433.  Outputs: logits [n_tok x E],
 * sel [n_tok x k] (int32), weights [n_tok x k].  Replaces route_topk
 * (engine/midge.c:404). */
int mg_router_topk(const float *xb, int n_tok, const float *rw, const float *rb, int n_experts,
                   int64_t hidden, int top_k, int router_norm, int variant, float *logits, int32_t *sel,
                   float *weights, void *stream);

/* Expert geometry of experts.midge (engine/mten.h:136-150). */
typedef struct {
    int dt;          /* MG_* dtype of every expert matrix */
    int scale_fmt;   /* MG_SCALE_* of the 4-bit scales as stored on the device */
    int64_t hidden, ffn;
    int64_t off[3][3];   /* [gate,up,down][data,scales,bias] byte offsets within an expert */
    int64_t expert_stride, layer_stride;
} mg_expert_layout;

/* Fill an mg_expert_layout exactly as wt_expert_layout (engine/mten.h:136). */
int mg_expert_layout_init(mg_expert_layout *L, int dt, int64_t hidden, int64_t ffn, int64_t n_experts);

/* Routed-expert FFN for n_tok tokens of one layer (decode form):
 *   x[t] += sum_i w[t][i] * (down_e(act(gate_e(xb[t]) + bg, up_e(xb[t]) + bu)) + bd),
 *   e = sel[t][i], summed in top-k rank order as engine/midge.c:514-548.
 * experts_layer points at layer 0 of the experts blob; layer selects the layer.
 * act_plain / alpha / limit as engine/midge.c:525-539.  n_tok <= 16.
 * h_scratch: device buffer of n_tok*top_k*ffn floats. */
int mg_moe_ffn(const mg_expert_layout *L, const uint8_t *experts, int layer, int n_experts,
               const float *xb, int n_tok, int top_k, const int32_t *sel, const float *weights,
               int act_plain, float alpha, float limit, float *h_scratch, float *x, void *stream);

/* No counterpart in the reference.  mg_moe_ffn for callers that may not
 * allocate device memory on the call path (a fixed start-up memory budget,
 * an allocator owned by another component, a plain C or cgo host without a
 * device allocator): the gate/up activations live in a fixed device array
 * inside this library instead of a caller's h_scratch.  Limits: n_tok <=
 * MG_NOALLOC_MAX_TOK (16, as for mg_moe_ffn), else MG_ERR_ARG; and
 * n_tok * top_k * ffn <= MG_NOALLOC_MAX_H floats, else MG_ERR_RANGE.  The
 * first call on a device (with that device current) looks up the array and
 * should come before any stream capture.  Calls that overlap in time on one
 * device share the array and race; serialise them.  The array needs no
 * zeroing. */
#define MG_NOALLOC_MAX_H (1 << 20)
#define MG_NOALLOC_MAX_TOK 16
int mg_moe_ffn_noalloc(const mg_expert_layout *L, const uint8_t *experts, int layer, int n_experts,
                       const float *xb, int n_tok, int top_k, const int32_t *sel, const float *weights,
                       int act_plain, float alpha, float limit, float *x, void *stream);

/* Sampling of the next token from n_rows logits rows (row i at
 * logits + i*ldl, V entries): sample (engine/midge.c:650-678).  temp <= 0:
 * the first maximum (greedy).  Otherwise softmax with the temperature, the
 * shortest descending-probability prefix whose mass reaches top_p, and a draw
 * from it with the reference's xorshift64* generator, whose per-row state
 * rng[i] (device) advances by one draw.  Entries of exactly equal
 * probability are ordered by index.  probs: device scratch of n_rows*V
 * floats (may be NULL when temp <= 0).  out: device int32 [n_rows]. */
int mg_sample_topp(const float *logits, int64_t ldl, int64_t V, int n_rows, float temp, float top_p, uint64_t *rng,
                   int32_t *out, float *probs, void *stream);

/* Failure-path self-test of a bounded device wait (no counterpart in the
 * reference): a one-CTA kernel waits `polls` times (1..2^20) on an mbarrier
 * that nothing arrives on, records the timeout in the library's error word,
 * waits for the bulk copy it issued to land (*drained = 43 when it did),
 * frees its tensor memory and exits -- the sequence every pipelined kernel of
 * the library follows when a wait runs out.  Returns MG_ERR_TIMEOUT; the
 * context stays usable. */
int mg_wait_selftest(int polls, int *drained);

/* ====================================================== model level ==== */

/* The model spec (engine/midge.c:46-63, parsed from the container's embedded
 * JSON by the host). */
typedef struct {
    int64_t hidden, vocab, ffn;
    int n_layers, n_heads, n_kv_heads, head_dim;
    int n_experts, top_k;
    float alpha, limit;
    int act_plain, router_norm, qk_norm;
    int sliding_window, sinks;
    float norm_eps, rope_theta;
    int yarn;
    float yarn_factor, yarn_beta_fast, yarn_beta_slow;
    int yarn_orig_ctx, yarn_truncate;
    float attn_scale;
    const int *layer_sliding; /* n_layers entries, copied at create */
} mg_spec;

typedef struct mg_model mg_model;

/* Create a model for `max_seqs` concurrent sequences of up to `ctx` tokens on
 * CUDA device `device`.  Replaces the allocation half of model_load
 * (engine/midge.c:204-294). */
int mg_model_create(const mg_spec *spec, int ctx, int max_seqs, int device, mg_model **out);

/* Expert parallelism over the GPUs of one box (no counterpart in the
 * reference, which is one process; its expert-swarm proposal,
 * docs/SPEED.md:94-99, shards experts the same way).  Rank r of `world`
 * (<= 8) holds experts [r E/world, (r+1) E/world) and owns its own sequences
 * (their attention, KV cache, router and lm_head; the trunk weights are
 * replicated).  Each MoE layer sends every routed token to the ranks that hold
 * its experts and the per-slot outputs back to the token's owner, which adds
 * them in the reference's order: results equal the one-GPU results bit for
 * bit.  NCCL is loaded at run time.  mg_ep_unique_id fills MG_EP_ID_BYTES
 * bytes on one rank, which the host hands to every rank; mg_model_set_ep goes
 * between mg_model_create and the experts upload (which then takes the full
 * blob and keeps this rank's shard).
 * With world > 1, mg_forward_batch, mg_decode_step, mg_decode_greedy and
 * mg_forward are collective: every rank calls them together, each with its
 * own sequences (a rank with nothing to do passes n = 0 / n_seqs = 0 and
 * still serves its experts); decode serves at most 8 tokens per step over all
 * ranks.  Blocking waits are watched: when the other ranks do not answer
 * within MIDGE_EP_TIMEOUT_S seconds (default 600) or the communicator reports
 * an error, the communicator is aborted (ncclCommAbort) and the call returns
 * MG_ERR_COMM; the model then only accepts mg_model_free. */
#define MG_EP_ID_BYTES 128
int mg_ep_unique_id(void *id);
int mg_model_set_ep(mg_model *m, int rank, int world, const void *id);

/* Expert-parallel prefill timing, with MIDGE_EP_STATS=1 at model creation:
 * milliseconds summed over every MoE layer of every prefill chunk so far,
 * per phase [plan + count agreement, dispatch, expert GEMMs, return +
 * combine] (CUDA events on the model's stream); zeros otherwise. */
int mg_model_ep_stats(mg_model *m, double *ms4);

/* Self-test of the expert-parallel watchdog loop against fakes (no GPU, no
 * NCCL): scenario 0 = the wait completes, 1 = it never completes (timeout),
 * 2 = the communicator reports an asynchronous error, 3 = a device error.
 * Returns what the watchdog returns (MG_OK, MG_ERR_COMM, MG_ERR_CUDA);
 * *aborted = how many times it aborted the (fake) communicator. */
int mg_ep_watchdog_selftest(int scenario, double timeout_s, int *aborted);

/* Upload one dense tensor named as in dense.midge (embed, lm_head,
 * final_norm, L<i>.attn.q ...; docs/ADDING_MODELS.md naming); host pointers,
 * copied into HBM.  Vectors: rows = n, cols = 0, dt = MG_F32.  Replaces the
 * view resolution of model_load (engine/midge.c:229-260). */
int mg_model_set_dense(mg_model *m, const char *name, int dt, int64_t rows, int64_t cols,
                       const void *data, const void *scales);

/* Upload the experts.midge data region (all layers, layout of
 * mg_expert_layout_init) from host memory with pinned staging and
 * cudaMemcpyAsync; power-of-two f16 scales are re-expressed as ue8m0 in HBM.
 * Replaces the mmap of experts.midge (engine/midge.c:210-227). */
int mg_model_set_experts(mg_model *m, int dt, const void *data, uint64_t bytes);

/* Fill the expert blob with seeded synthetic weights directly in HBM (for
 * benchmarks of shapes whose files would not fit a disk): MXFP4 nibbles
 * uniform over 0..15, scales 2^k with k uniform in [-8,-4], biases N(0,0.1);
 * q8r bytes uniform in [-127,127] with power-of-two row scales. */
int mg_model_synth_experts(mg_model *m, int dt, uint64_t seed);

/* Finish loading (rope tables, KV caches, work buffers).  After this the
 * model accepts forward calls. */
int mg_model_ready(mg_model *m);

/* Forget sequence `seq`'s context (position 0). */
int mg_model_reset(mg_model *m, int seq);
int mg_model_pos(const mg_model *m, int seq);

/* One token of sequence `seq` through the model: forward
 * (engine/midge.c:552-566).  logits (host, vocab floats) and/or argmax (host
 * int32, first maximum wins as engine/midge.c:657-660) may be NULL. */
int mg_forward(mg_model *m, int seq, int32_t token, float *logits, int32_t *argmax);

/* Expert-major batched prefill of n tokens of sequence `seq`: forward_batch
 * (engine/midge.c:576-622).  logits_mode 0 = none, 1 = last position,
 * 2 = every position ([n x vocab]). */
int mg_forward_batch(mg_model *m, int seq, const int32_t *toks, int n, int logits_mode, float *logits);

/* One decode step for n_seqs sequences at once (one token each): the
 * concurrent-sequence form of forward.  logits [n_seqs x vocab] and argmax
 * [n_seqs] (host) may be NULL. */
int mg_decode_step(mg_model *m, int n_seqs, const int32_t *seq_ids, const int32_t *toks, float *logits,
                   int32_t *argmax);

/* Greedy decode of n_steps tokens for n_seqs sequences without host round
 * trips: the concurrent-sequence form of midged's gen: loop
 * (engine/midge.c:812-826, argmax as engine/midge.c:657-660).  Step k's
 * input is step k-1's argmax, fed on the device; out_toks (host,
 * [n_steps x n_seqs]) receives every step's argmax, exactly what n_steps
 * calls of mg_decode_step with argmax feedback return.  n_steps <= 4096. */
int mg_decode_greedy(mg_model *m, int n_seqs, const int32_t *seq_ids, const int32_t *toks, int n_steps,
                     int32_t *out_toks);

/* Kernels launched so far by the decode entry points of this model (graph
 * replays counted by their kernel nodes). */
uint64_t mg_model_kernel_launches(const mg_model *m);

/* Measurement hook, no counterpart in the reference: the routed-expert FFN
 * kernels of the streamed decode (gate/up + clamped SwiGLU, then down) for
 * n_tok tokens routed by sel (device, [n_tok x top_k]) on the model's
 * resident experts of `layer`, reading the model's current normed rows and
 * writing its scratch.  Asynchronous on mg_model_stream(m), unlike the other
 * model-level calls, so that a caller can time it with stream events. */
int mg_model_moe_stream(mg_model *m, int layer, int n_tok, const int32_t *sel);

/* Sample the next token of the first n_rows rows of the model's last
 * logits on the device (mg_sample_topp): the rows of the last decode step's
 * sequences, or row 0 = the last prompt position after mg_forward_batch.
 * rng: HOST array of n_rows generator states, advanced in place (midged's
 * one state for one sequence); out: host int32 [n_rows]. */
int mg_model_sample(mg_model *m, int n_rows, float temp, float top_p, uint64_t *rng, int32_t *out);

/* Copy row `row` of the logits the last forward / decode step / prefill
 * computed (host, vocab floats); the device-resident copy of the reference's
 * m->logits (engine/midge.c:82). */
int mg_model_logits(mg_model *m, int row, float *out);

/* Put a host logits row (vocab floats) into row `row` (< 16) of the model's
 * device logits, where mg_model_sample reads it: a host serving several
 * sequences keeps a sequence's pending logits while another one runs. */
int mg_model_put_logits(mg_model *m, int row, const float *logits);

/* usage histogram u32[n_layers x n_experts] (engine/midge.c:283-303) */
int mg_model_get_usage(mg_model *m, uint32_t *usage);
int mg_model_set_usage(mg_model *m, const uint32_t *usage);
uint64_t mg_model_expert_loads(const mg_model *m);

/* Device pointers for benches/tests that drive kernel-level calls on the
 * model's resident weights. */
const uint8_t *mg_model_experts_device(const mg_model *m, mg_expert_layout *layout);
void *mg_model_stream(const mg_model *m);

int mg_model_free(mg_model *m);

/* Weight-streaming microbench of one dequant-GEMV on device `device`: a
 * [rows x cols] matrix of dtype dt (seeded data, f16 scales re-expressed as
 * ue8m0 for mxfp4) times n_tok <= 256 vectors, repeated over enough copies to exceed
 * L2, for at least `seconds`.  *gbps = (weight + scale bytes) per call / time,
 * in GiB/s like run_bench (engine/midge.c:687-720), the device replacement of
 * midged --bench. */
int mg_bench_gemv(int dt, int64_t rows, int64_t cols, int n_tok, double seconds, int device, double *gbps);

#ifdef __cplusplus
}
#endif
#endif /* MIDGECUDA_H */

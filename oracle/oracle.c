/* oracle.c -- CPU restatement of midge's quantized-MoE forward path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the shipped library or the midged host
 * links, loads or calls this file; only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py use it, and only as the checker.
 *
 * Every function restates one piece of the reference engine (drmihirbrahme/midge,
 * engine/mkern.h, engine/mten.h, engine/midge.c) and cites the lines it follows.
 * The matvecs follow the AVX2+FMA code path (the one midged runs on any x86 host
 * with AVX2), including its 8-lane accumulation order and the hsum256 tree, so
 * that this file reproduces the reference bit for bit.  Build with
 * -std=c11 -ffp-contract=off: the reference is compiled with -std=c11 (ISO
 * mode, so GCC does not contract a*b+c into an FMA) and the only fused
 * multiply-adds it executes are the explicit _mm256_fmadd_ps calls, which are
 * restated here with fmaf().
 *
 * Speed (so that full-width model slices check in seconds): the matvecs keep
 * each output row's operation order exactly and only (1) let the compiler
 * vectorise the eight independent lane chains (an AVX2+FMA clone is selected
 * at load time where the CPU has it; fmaf is exact either way) and (2) split
 * the rows over OpenMP threads.  Neither changes a single rounding.
 *
 * Parity pin: tests/test_oracle_cpu.py compares this file against the reference
 * itself (oracle/_ref, compiled from the reference sources by oracle/Makefile)
 * and against golden outputs of the reference midged stored in tests/golden/.
 */
#include <math.h>
#include <stdio.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* rows x cols above which a matvec splits its rows over threads */
#define OR_PAR_WORK (1 << 18)
#if defined(__x86_64__) && defined(__GNUC__) && !defined(__clang__)
#define OR_CLONES __attribute__((target_clones("arch=x86-64-v3", "default")))
#else
#define OR_CLONES
#endif

#define OR_F32 0
#define OR_Q8R 1
#define OR_Q4G32 2
#define OR_MXFP4 3
#define OR_MAX_TOPK 16 /* engine/midge.c:44 */
#define OR_BATCH_MAX 64 /* engine/midge.c:43 */

/* e2m1 code -> value; engine/mten.h:44-47 */
static const float OR_FP4[16] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f,
                                 -0.0f, -0.5f, -1.0f, -1.5f, -2.0f, -3.0f, -4.0f, -6.0f};
/* signed doubled magnitudes used by the AVX2 kernel; engine/mkern.h:128-129 */
static const int OR_FP4X2[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* IEEE half bits -> float, exact including subnormals; engine/mten.h:49-57 */
float or_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) & 1u, ex = (h >> 10) & 31u, man = h & 1023u, bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign << 31;
        } else { /* normalise the subnormal */
            uint32_t e = 113;
            while (!(man & 1024u)) { man <<= 1; e--; }
            man &= 1023u;
            bits = (sign << 31) | (e << 23) | (man << 13);
        }
    } else if (ex == 31) {
        bits = (sign << 31) | 0x7f800000u | (man << 13);
    } else {
        bits = (sign << 31) | ((ex + 112u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* float -> half, round-to-nearest-even, subnormal results flushed to signed
 * zero, overflow to inf; engine/mkern.h:261-273 */
uint16_t or_f32_to_f16_ftz(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    int32_t e = (int32_t)((x >> 23) & 0xff) - 112;
    uint32_t man = x & 0x7fffffu;
    if (e <= 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    uint32_t m = man >> 13, rem = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (m & 1u))) {
        m++;
        if (m == 0x400u) {
            m = 0;
            e++;
            if (e >= 31) return (uint16_t)(sign | 0x7c00u);
        }
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | m);
}

/* blob sizes of a [rows x cols] matrix; engine/mten.h:101-109 */
void or_blob_sizes(int dt, int64_t rows, int64_t cols, int64_t *db, int64_t *sb) {
    switch (dt) {
    case OR_F32: *db = rows * cols * 4; *sb = 0; break;
    case OR_Q8R: *db = rows * cols; *sb = rows * 4; break;
    case OR_Q4G32:
    case OR_MXFP4: *db = rows * cols / 2; *sb = rows * (cols / 32) * 2; break;
    default: *db = 0; *sb = 0;
    }
}

/* one dequantised row (embedding lookup); engine/mkern.h:201-236 */
void or_dequant_row(int dt, const void *data, const void *scales, int64_t cols, int64_t r, float *out) {
    if (dt == OR_F32) {
        memcpy(out, (const float *)data + r * cols, (size_t)cols * 4);
    } else if (dt == OR_Q8R) {
        const int8_t *w = (const int8_t *)data + r * cols;
        float s = ((const float *)scales)[r];
        for (int64_t c = 0; c < cols; c++) out[c] = (float)w[c] * s;
    } else {
        const uint8_t *w = (const uint8_t *)data + r * (cols / 2);
        const uint16_t *s = (const uint16_t *)scales + r * (cols / 32);
        for (int64_t g = 0; g < cols / 32; g++) {
            float sc = or_f16_to_f32(s[g]);
            for (int j = 0; j < 16; j++) {
                uint8_t b = w[g * 16 + j];
                float lo, hi;
                if (dt == OR_MXFP4) { lo = OR_FP4[b & 15]; hi = OR_FP4[b >> 4]; }
                else { lo = (float)((int)(b & 15) - 8); hi = (float)((int)(b >> 4) - 8); }
                out[g * 32 + 2 * j] = lo * sc;
                out[g * 32 + 2 * j + 1] = hi * sc;
            }
        }
    }
}

/* horizontal sum of 8 lanes in the order of hsum256; engine/mkern.h:76-82 */
static float or_hsum8(const float a[8]) {
    float l0 = a[0] + a[4], l1 = a[1] + a[5], l2 = a[2] + a[6], l3 = a[3] + a[7];
    l0 = l0 + l2;
    l1 = l1 + l3;
    return l0 + l1;
}

/* f32 matvec, AVX2 order; engine/mkern.h:85-99 */
OR_CLONES static void or_mv_f32(const float *W, const float *x, float *y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static) if (rows * cols >= OR_PAR_WORK)
    for (int64_t r = 0; r < rows; r++) {
        const float *w = W + r * cols;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int64_t c = 0;
        for (; c + 8 <= cols; c += 8)
            for (int l = 0; l < 8; l++) acc[l] = fmaf(w[c + l], x[c + l], acc[l]);
        float a = or_hsum8(acc);
        for (; c < cols; c++) a += w[c] * x[c];
        y[r] = a;
    }
}

/* int8 per-row-scale matvec, AVX2 order, scale applied after the sum;
 * engine/mkern.h:102-118 */
OR_CLONES static void or_mv_q8r(const int8_t *W, const float *S, const float *x, float *y, int64_t rows, int64_t cols) {
#pragma omp parallel for schedule(static) if (rows * cols >= OR_PAR_WORK)
    for (int64_t r = 0; r < rows; r++) {
        const int8_t *w = W + r * cols;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        int64_t c = 0;
        for (; c + 8 <= cols; c += 8)
            for (int l = 0; l < 8; l++) acc[l] = fmaf((float)w[c + l], x[c + l], acc[l]);
        float a = or_hsum8(acc);
        for (; c < cols; c++) a += (float)w[c] * x[c];
        y[r] = a * S[r];
    }
}

/* 4-bit group-32 matvec (MXFP4 or q4g32), AVX2 order: per group the 16 bytes
 * give low-nibble (even column) and high-nibble (odd column) codes, four
 * 8-lane products are chained, then the group scale (halved for FP4, whose
 * codes are doubled) is fused into the 8-lane accumulator; engine/mkern.h:121-166 */
OR_CLONES static void or_mv_g32(const uint8_t *W, const uint16_t *S, const float *x, float *y, int64_t rows,
                                int64_t cols, int is_fp4) {
    int64_t gpr = cols / 32, half = cols / 2;
    float *xe = (float *)malloc((size_t)half * 4), *xo = (float *)malloc((size_t)half * 4);
    for (int64_t k = 0; k < half; k++) { xe[k] = x[2 * k]; xo[k] = x[2 * k + 1]; }
    /* per byte: the low (even column) and high (odd column) code as the float
     * the AVX2 kernel multiplies (doubled FP4 magnitude, or code - 8) */
    float tlo[256], thi[256];
    for (int b = 0; b < 256; b++) {
        tlo[b] = is_fp4 ? (float)OR_FP4X2[b & 15] : (float)((b & 15) - 8);
        thi[b] = is_fp4 ? (float)OR_FP4X2[b >> 4] : (float)((b >> 4) - 8);
    }
#pragma omp parallel for schedule(static) if (rows * cols >= OR_PAR_WORK)
    for (int64_t r = 0; r < rows; r++) {
        const uint8_t *w = W + r * half;
        const uint16_t *s = S + r * gpr;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t g = 0; g < gpr; g++) {
            float lo[16], hi[16];
            for (int j = 0; j < 16; j++) {
                lo[j] = tlo[w[g * 16 + j]];
                hi[j] = thi[w[g * 16 + j]];
            }
            const float *pe = xe + g * 16, *po = xo + g * 16;
            float g0[8];
            for (int i = 0; i < 8; i++) g0[i] = lo[i] * pe[i];
            for (int i = 0; i < 8; i++) g0[i] = fmaf(lo[8 + i], pe[8 + i], g0[i]);
            for (int i = 0; i < 8; i++) g0[i] = fmaf(hi[i], po[i], g0[i]);
            for (int i = 0; i < 8; i++) g0[i] = fmaf(hi[8 + i], po[8 + i], g0[i]);
            float sc = or_f16_to_f32(s[g]) * (is_fp4 ? 0.5f : 1.0f);
            for (int i = 0; i < 8; i++) acc[i] = fmaf(sc, g0[i], acc[i]);
        }
        y[r] = or_hsum8(acc);
    }
    free(xe);
    free(xo);
}

/* dtype dispatch; engine/mkern.h:180-198 (AVX2 branch) */
void or_matvec(int dt, const void *data, const void *scales, int64_t rows, int64_t cols, const float *x,
               float *y) {
    switch (dt) {
    case OR_F32: or_mv_f32((const float *)data, x, y, rows, cols); break;
    case OR_Q8R: or_mv_q8r((const int8_t *)data, (const float *)scales, x, y, rows, cols); break;
    case OR_Q4G32: or_mv_g32((const uint8_t *)data, (const uint16_t *)scales, x, y, rows, cols, 0); break;
    case OR_MXFP4: or_mv_g32((const uint8_t *)data, (const uint16_t *)scales, x, y, rows, cols, 1); break;
    }
}

/* Sum of |w|*|x| per row: the magnitude against which tests bound the
 * accumulation-order difference of a matvec (not a reference function). */
void or_matvec_abs(int dt, const void *data, const void *scales, int64_t rows, int64_t cols, const float *x,
                   double *y) {
#pragma omp parallel if (rows * cols >= OR_PAR_WORK)
    {
        float *row = (float *)malloc((size_t)cols * 4);
#pragma omp for schedule(static)
        for (int64_t r = 0; r < rows; r++) {
            or_dequant_row(dt, data, scales, cols, r, row);
            double a = 0;
            for (int64_t c = 0; c < cols; c++) a += fabs((double)row[c]) * fabs((double)x[c]);
            y[r] = a;
        }
        free(row);
    }
}

/* sequential-sum RMSNorm; engine/mkern.h:238-243 */
void or_rmsnorm(const float *x, const float *w, float *out, int64_t n, float eps) {
    float ss = 0.f;
    for (int64_t i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int64_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

static void or_addbias(float *y, const float *b, int64_t n) { /* engine/mkern.h:245 */
    for (int64_t i = 0; i < n; i++) y[i] += b[i];
}

/* top-k as in the decode path: bottom insertion, a later equal logit never
 * displaces an earlier one, slots start at (-1, -1e30); engine/midge.c:476-486 */
void or_topk_decode(const float *rl, int n_experts, int k, int *sel, float *val) {
    for (int i = 0; i < k; i++) { sel[i] = -1; val[i] = -1e30f; }
    for (int e = 0; e < n_experts; e++) {
        float v = rl[e];
        if (v > val[k - 1]) {
            int j = k - 1;
            while (j > 0 && val[j - 1] < v) { val[j] = val[j - 1]; sel[j] = sel[j - 1]; j--; }
            val[j] = v;
            sel[j] = e;
        }
    }
}

/* top-k as in the batched-prefill path: first slot the logit beats wins,
 * slots start at (0, -1e30); engine/midge.c:410-422 */
void or_topk_prefill(const float *rl, int n_experts, int k, int *sel, float *val) {
    for (int j = 0; j < k; j++) { val[j] = -1e30f; sel[j] = 0; }
    for (int e = 0; e < n_experts; e++) {
        float v = rl[e];
        for (int j = 0; j < k; j++) {
            if (v > val[j]) {
                for (int q = k - 1; q > j; q--) { val[q] = val[q - 1]; sel[q] = sel[q - 1]; }
                val[j] = v;
                sel[j] = e;
                break;
            }
        }
    }
}

/* routing weights: softmax over the selected logits (router_norm=1) or the
 * full-softmax probabilities of the selected experts (router_norm=0);
 * engine/midge.c:423-433 and :502-512 (identical arithmetic) */
void or_route_weights(const float *rl, int n_experts, const float *val, int k, int router_norm, float *w) {
    float mx = val[0], den = 0.f;
    if (router_norm) {
        for (int i = 0; i < k; i++) { w[i] = expf(val[i] - mx); den += w[i]; }
        for (int i = 0; i < k; i++) w[i] /= den;
    } else {
        float fmx = rl[0];
        for (int e = 1; e < n_experts; e++) if (rl[e] > fmx) fmx = rl[e];
        float fden = 0.f;
        for (int e = 0; e < n_experts; e++) fden += expf(rl[e] - fmx);
        for (int i = 0; i < k; i++) w[i] = expf(val[i] - fmx) / fden;
    }
}

/* gated activation in place over hb (gate) with hb2 (up);
 * engine/midge.c:525-539 */
void or_swiglu(float *hb, const float *hb2, int64_t n, int act_plain, float alpha, float limit) {
    if (act_plain) {
        for (int64_t j = 0; j < n; j++) { float g = hb[j]; hb[j] = g / (1.0f + expf(-g)) * hb2[j]; }
    } else {
        for (int64_t j = 0; j < n; j++) {
            float g = hb[j], u = hb2[j];
            if (g > limit) g = limit;
            if (u > limit) u = limit;
            if (u < -limit) u = -limit;
            float act = g / (1.0f + expf(-alpha * g));
            hb[j] = act * (u + 1.0f);
        }
    }
}

/* ------------------------------------------------------------------ model */

typedef struct { /* engine/midge.c:46-63 */
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
    const int *layer_sliding;
} or_spec;

typedef struct { int dt; int64_t rows, cols; const void *data, *scales; } or_wt;

typedef struct {
    or_spec s;
    int ctx, pos, expert_dt;
    const uint8_t *experts; /* data region of experts.midge */
    int64_t eoff[3][3], expert_stride, layer_stride;
    or_wt embed, lm_head;
    const float *final_norm;
    or_wt *wq, *wk, *wv, *wo, *router_w;
    const float **bq, **bk, **bv, **bo, **router_b, **attn_norm, **mlp_norm, **sink, **qn, **kn;
    uint16_t **kc, **vc;
    float *x, *xb, *q, *k, *v, *ao, *att, *hb, *hb2, *moe, *rl, *logits;
    float *bx, *bxb, *bw;
    int *bsel;
    float *rope_cos, *rope_sin;
    uint32_t *usage;
    uint64_t expert_loads;
} or_model;

static int64_t or_align64(int64_t v) { return (v + 63) & ~(int64_t)63; }

/* deterministic expert layout; engine/mten.h:136-150 */
void or_expert_layout(int dt, int64_t hidden, int64_t ffn, int64_t n_experts, int64_t off[3][3],
                      int64_t *expert_stride, int64_t *layer_stride) {
    int64_t rows[3] = {ffn, ffn, hidden}, cols[3] = {hidden, hidden, ffn}, o = 0;
    for (int m = 0; m < 3; m++) {
        int64_t db, sb;
        or_blob_sizes(dt, rows[m], cols[m], &db, &sb);
        off[m][0] = o; o = or_align64(o + db);
        off[m][1] = o; o = or_align64(o + sb);
        off[m][2] = o; o = or_align64(o + rows[m] * 4);
    }
    *expert_stride = or_align64(o);
    *layer_stride = *expert_stride * n_experts;
}

/* YaRN rope tables in double precision; engine/midge.c:141-176 */
static void or_rope_init(or_model *m) {
    or_spec *s = &m->s;
    int hd = s->head_dim, half = hd / 2;
    m->rope_cos = (float *)malloc((size_t)m->ctx * half * 4);
    m->rope_sin = (float *)malloc((size_t)m->ctx * half * 4);
    double *inv = (double *)malloc(half * sizeof(double)), mscale = 1.0;
    for (int i = 0; i < half; i++) inv[i] = 1.0 / pow((double)s->rope_theta, (double)(2 * i) / hd);
    if (s->yarn) {
        double f = s->yarn_factor, base = s->rope_theta, orig = s->yarn_orig_ctx;
        double low = hd * log(orig / (s->yarn_beta_fast * 2.0 * M_PI)) / (2.0 * log(base));
        double high = hd * log(orig / (s->yarn_beta_slow * 2.0 * M_PI)) / (2.0 * log(base));
        if (s->yarn_truncate) { low = floor(low); high = ceil(high); }
        if (low < 0) low = 0;
        if (high > hd - 1) high = hd - 1;
        if (high == low) high = low + 0.001;
        for (int i = 0; i < half; i++) {
            double ramp = ((double)i - low) / (high - low);
            if (ramp < 0) ramp = 0;
            if (ramp > 1) ramp = 1;
            double keep = 1.0 - ramp;
            inv[i] = (inv[i] / f) * (1.0 - keep) + inv[i] * keep;
        }
        mscale = 0.1 * log(f) + 1.0;
    }
    for (int p = 0; p < m->ctx; p++)
        for (int i = 0; i < half; i++) {
            double a = (double)p * inv[i];
            m->rope_cos[(size_t)p * half + i] = (float)(cos(a) * mscale);
            m->rope_sin[(size_t)p * half + i] = (float)(sin(a) * mscale);
        }
    free(inv);
}

/* half-split rotation; engine/midge.c:178-190 */
static void or_rope_apply(or_model *m, float *vec, int nh, int pos) {
    int hd = m->s.head_dim, half = hd / 2;
    const float *co = m->rope_cos + (size_t)pos * half, *si = m->rope_sin + (size_t)pos * half;
    for (int h = 0; h < nh; h++) {
        float *v = vec + (size_t)h * hd;
        for (int i = 0; i < half; i++) {
            float a = v[i], b = v[i + half];
            v[i] = a * co[i] - b * si[i];
            v[i + half] = b * co[i] + a * si[i];
        }
    }
}

or_model *or_model_new(const or_spec *spec, int ctx, int expert_dt, const uint8_t *experts) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->s = *spec;
    m->ctx = ctx;
    m->expert_dt = expert_dt;
    m->experts = experts;
    or_expert_layout(expert_dt, spec->hidden, spec->ffn, spec->n_experts, m->eoff, &m->expert_stride,
                     &m->layer_stride);
    int L = spec->n_layers;
    m->wq = calloc(L, sizeof(or_wt)); m->wk = calloc(L, sizeof(or_wt));
    m->wv = calloc(L, sizeof(or_wt)); m->wo = calloc(L, sizeof(or_wt));
    m->router_w = calloc(L, sizeof(or_wt));
    const float ***vecs[] = {&m->bq, &m->bk, &m->bv, &m->bo, &m->router_b, &m->attn_norm,
                             &m->mlp_norm, &m->sink, &m->qn, &m->kn};
    for (size_t i = 0; i < sizeof(vecs) / sizeof(vecs[0]); i++) *vecs[i] = calloc(L, sizeof(void *));
    int kv_dim = spec->n_kv_heads * spec->head_dim, q_dim = spec->n_heads * spec->head_dim;
    m->kc = calloc(L, sizeof(void *));
    m->vc = calloc(L, sizeof(void *));
    for (int i = 0; i < L; i++) { /* engine/midge.c:268-273 */
        int cap = spec->layer_sliding[i] && spec->sliding_window > 0 && spec->sliding_window < ctx
                      ? spec->sliding_window : ctx;
        m->kc[i] = calloc((size_t)cap * kv_dim, 2);
        m->vc[i] = calloc((size_t)cap * kv_dim, 2);
    }
    int64_t h = spec->hidden;
    m->x = malloc(h * 4); m->xb = malloc(h * 4); m->moe = malloc(h * 4);
    m->q = malloc(q_dim * 4); m->k = malloc(kv_dim * 4); m->v = malloc(kv_dim * 4);
    m->ao = malloc(q_dim * 4);
    m->att = malloc((size_t)spec->n_heads * ctx * 4);
    m->hb = malloc(spec->ffn * 4); m->hb2 = malloc(spec->ffn * 4);
    m->rl = malloc(spec->n_experts * 4);
    m->logits = malloc(spec->vocab * 4);
    m->bx = malloc((size_t)OR_BATCH_MAX * h * 4);
    m->bxb = malloc((size_t)OR_BATCH_MAX * h * 4);
    m->bw = malloc((size_t)OR_BATCH_MAX * OR_MAX_TOPK * 4);
    m->bsel = malloc((size_t)OR_BATCH_MAX * OR_MAX_TOPK * sizeof(int));
    m->usage = calloc((size_t)L * spec->n_experts, 4);
    or_rope_init(m);
    return m;
}

/* Register one dense tensor by its container name (engine/midge.c:229-260). */
int or_model_set(or_model *m, const char *name, int dt, int64_t rows, int64_t cols, const void *data,
                 const void *scales) {
    or_wt t = {dt, rows, cols, data, scales};
    if (!strcmp(name, "embed")) { m->embed = t; return 0; }
    if (!strcmp(name, "lm_head")) { m->lm_head = t; return 0; }
    if (!strcmp(name, "final_norm")) { m->final_norm = (const float *)data; return 0; }
    int layer;
    char rest[64];
    if (sscanf(name, "L%d.%63s", &layer, rest) != 2 || layer < 0 || layer >= m->s.n_layers) return -1;
    struct { const char *n; or_wt *mat; const float **vec; } map[] = {
        {"attn.q", m->wq, 0}, {"attn.k", m->wk, 0}, {"attn.v", m->wv, 0}, {"attn.o", m->wo, 0},
        {"router.w", m->router_w, 0}, {"attn.q_b", 0, m->bq}, {"attn.k_b", 0, m->bk},
        {"attn.v_b", 0, m->bv}, {"attn.o_b", 0, m->bo}, {"router.b", 0, m->router_b},
        {"attn.norm", 0, m->attn_norm}, {"mlp.norm", 0, m->mlp_norm}, {"attn.sinks", 0, m->sink},
        {"attn.q_norm", 0, m->qn}, {"attn.k_norm", 0, m->kn}};
    for (size_t i = 0; i < sizeof(map) / sizeof(map[0]); i++) {
        if (strcmp(rest, map[i].n)) continue;
        if (map[i].mat) map[i].mat[layer] = t;
        else map[i].vec[layer] = (const float *)data;
        return 0;
    }
    return -1;
}

/* per-token attention block; engine/midge.c:341-400 */
static void or_attention(or_model *m, int layer, int pos) {
    or_spec *s = &m->s;
    int hd = s->head_dim, nh = s->n_heads, nkv = s->n_kv_heads, kv_dim = nkv * hd, gq = nh / nkv;
    int sliding = s->layer_sliding[layer] && s->sliding_window > 0 && s->sliding_window < m->ctx;
    int cap = sliding ? s->sliding_window : m->ctx;
    or_rmsnorm(m->x, m->attn_norm[layer], m->xb, s->hidden, s->norm_eps);
    or_wt *t = &m->wq[layer];
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, m->xb, m->q);
    or_addbias(m->q, m->bq[layer], (int64_t)nh * hd);
    t = &m->wk[layer];
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, m->xb, m->k);
    or_addbias(m->k, m->bk[layer], kv_dim);
    t = &m->wv[layer];
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, m->xb, m->v);
    or_addbias(m->v, m->bv[layer], kv_dim);
    if (s->qk_norm) {
        for (int h = 0; h < nh; h++)
            or_rmsnorm(m->q + (size_t)h * hd, m->qn[layer], m->q + (size_t)h * hd, hd, s->norm_eps);
        for (int h = 0; h < nkv; h++)
            or_rmsnorm(m->k + (size_t)h * hd, m->kn[layer], m->k + (size_t)h * hd, hd, s->norm_eps);
    }
    or_rope_apply(m, m->q, nh, pos);
    or_rope_apply(m, m->k, nkv, pos);
    int slot = pos % cap;
    uint16_t *kc = m->kc[layer], *vc = m->vc[layer];
    for (int i = 0; i < kv_dim; i++) {
        kc[(size_t)slot * kv_dim + i] = or_f32_to_f16_ftz(m->k[i]);
        vc[(size_t)slot * kv_dim + i] = or_f32_to_f16_ftz(m->v[i]);
    }
    int nctx = pos + 1 < cap ? pos + 1 : cap;
    for (int h = 0; h < nh; h++) {
        float *sc = m->att + (size_t)h * m->ctx;
        const float *qh = m->q + (size_t)h * hd;
        int kh = h / gq;
        float mx = -1e30f;
        for (int tt = 0; tt < nctx; tt++) {
            const uint16_t *kt = kc + (size_t)tt * kv_dim + (size_t)kh * hd;
            float d = 0.f;
            for (int i = 0; i < hd; i++) d += qh[i] * or_f16_to_f32(kt[i]);
            d = d * s->attn_scale;
            sc[tt] = d;
            if (d > mx) mx = d;
        }
        float sinkv = s->sinks ? m->sink[layer][h] : -1e30f;
        if (sinkv > mx) mx = sinkv;
        float denom = s->sinks ? expf(sinkv - mx) : 0.f;
        for (int tt = 0; tt < nctx; tt++) { sc[tt] = expf(sc[tt] - mx); denom += sc[tt]; }
        float inv = 1.0f / denom;
        float *out = m->ao + (size_t)h * hd;
        memset(out, 0, hd * 4);
        for (int tt = 0; tt < nctx; tt++) {
            float w = sc[tt] * inv;
            const uint16_t *vt = vc + (size_t)tt * kv_dim + (size_t)kh * hd;
            for (int i = 0; i < hd; i++) out[i] += w * or_f16_to_f32(vt[i]);
        }
    }
    t = &m->wo[layer];
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, m->ao, m->xb);
    or_addbias(m->xb, m->bo[layer], s->hidden);
    for (int64_t i = 0; i < s->hidden; i++) m->x[i] += m->xb[i];
}

/* view of one expert matrix; engine/mten.h:153-162 */
static or_wt or_expert(or_model *m, int layer, int e, int mat, const float **bias) {
    const uint8_t *b = m->experts + (size_t)layer * m->layer_stride + (size_t)e * m->expert_stride;
    or_wt t;
    t.dt = m->expert_dt;
    t.rows = mat == 2 ? m->s.hidden : m->s.ffn;
    t.cols = mat == 2 ? m->s.ffn : m->s.hidden;
    t.data = b + m->eoff[mat][0];
    t.scales = m->expert_dt == OR_F32 ? NULL : b + m->eoff[mat][1];
    *bias = (const float *)(b + m->eoff[mat][2]);
    return t;
}

/* gate/up -> activation -> down for one expert, leaving down(h)+bias in out;
 * the shared body of engine/midge.c:443-464 and :519-543 */
static void or_expert_ffn(or_model *m, int layer, int e, const float *xb, float *out) {
    or_spec *s = &m->s;
    const float *bg, *bu, *bd;
    or_wt g = or_expert(m, layer, e, 0, &bg), u = or_expert(m, layer, e, 1, &bu),
          d = or_expert(m, layer, e, 2, &bd);
    or_matvec(g.dt, g.data, g.scales, g.rows, g.cols, xb, m->hb);
    or_addbias(m->hb, bg, s->ffn);
    or_matvec(u.dt, u.data, u.scales, u.rows, u.cols, xb, m->hb2);
    or_addbias(m->hb2, bu, s->ffn);
    or_swiglu(m->hb, m->hb2, s->ffn, s->act_plain, s->alpha, s->limit);
    or_matvec(d.dt, d.data, d.scales, d.rows, d.cols, m->hb, out);
    or_addbias(out, bd, s->hidden);
}

/* router logits for normed input xb (engine/midge.c:472-473) */
static void or_router(or_model *m, int layer, const float *xb) {
    or_wt *t = &m->router_w[layer];
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, xb, m->rl);
    or_addbias(m->rl, m->router_b[layer], m->s.n_experts);
}

/* decode MoE block; engine/midge.c:469-549 (prefetch hints dropped) */
static void or_moe(or_model *m, int layer, int *sel_out, float *w_out) {
    or_spec *s = &m->s;
    or_rmsnorm(m->x, m->mlp_norm[layer], m->xb, s->hidden, s->norm_eps);
    or_router(m, layer, m->xb);
    int sel[OR_MAX_TOPK], k = s->top_k;
    float val[OR_MAX_TOPK], w[OR_MAX_TOPK];
    or_topk_decode(m->rl, s->n_experts, k, sel, val);
    or_route_weights(m->rl, s->n_experts, val, k, s->router_norm, w);
    if (sel_out) { memcpy(sel_out, sel, k * sizeof(int)); memcpy(w_out, w, k * 4); }
    memset(m->moe, 0, (size_t)s->hidden * 4);
    for (int i = 0; i < k; i++) {
        int e = sel[i];
        m->usage[(size_t)layer * s->n_experts + e]++;
        m->expert_loads++;
        or_expert_ffn(m, layer, e, m->xb, m->xb);
        for (int64_t j = 0; j < s->hidden; j++) m->moe[j] += w[i] * m->xb[j];
        if (i + 1 < k) or_rmsnorm(m->x, m->mlp_norm[layer], m->xb, s->hidden, s->norm_eps);
    }
    for (int64_t j = 0; j < s->hidden; j++) m->x[j] += m->moe[j];
}

/* final norm + lm_head into m->logits (engine/midge.c:563-564) */
static void or_logits(or_model *m, const float *x) {
    or_rmsnorm(x, m->final_norm, m->xb, m->s.hidden, m->s.norm_eps);
    or_wt *t = &m->lm_head;
    or_matvec(t->dt, t->data, t->scales, t->rows, t->cols, m->xb, m->logits);
}

/* one token through the model; engine/midge.c:552-566. Returns 4 when the
 * context is full or the token is out of range (the reference exits 4).
 * If sel_trace is non-NULL it receives the [n_layers x top_k] routing. */
int or_forward(or_model *m, int token, float *logits, int *sel_trace, float *w_trace) {
    or_spec *s = &m->s;
    if (m->pos >= m->ctx || token < 0 || token >= s->vocab) return 4;
    or_dequant_row(m->embed.dt, m->embed.data, m->embed.scales, m->embed.cols, token, m->x);
    for (int layer = 0; layer < s->n_layers; layer++) {
        or_attention(m, layer, m->pos);
        or_moe(m, layer, sel_trace ? sel_trace + layer * s->top_k : NULL,
               w_trace ? w_trace + layer * s->top_k : NULL);
    }
    m->pos++;
    if (logits) {
        or_logits(m, m->x);
        memcpy(logits, m->logits, (size_t)s->vocab * 4);
    }
    return 0;
}

/* route one token for the batched path; engine/midge.c:404-434 */
static void or_route_topk(or_model *m, int layer, const float *x, float *xb, int *sel, float *w) {
    or_spec *s = &m->s;
    or_rmsnorm(x, m->mlp_norm[layer], xb, s->hidden, s->norm_eps);
    or_router(m, layer, xb);
    float val[OR_MAX_TOPK];
    or_topk_prefill(m->rl, s->n_experts, s->top_k, sel, val);
    or_route_weights(m->rl, s->n_experts, val, s->top_k, s->router_norm, w);
}

/* Expert-major batched prefill of n <= 64 tokens; engine/midge.c:576-622.
 * logits_out gets every position's logits when tfall, else the last one's
 * when want_last.  Returns 4 on context overflow / bad token. */
int or_forward_batch(or_model *m, const int *toks, int n, int tfall, int want_last, float *logits_out) {
    or_spec *s = &m->s;
    int64_t h = s->hidden;
    if (n > OR_BATCH_MAX) return 3;
    for (int t = 0; t < n; t++) {
        if (m->pos + t >= m->ctx || toks[t] < 0 || toks[t] >= s->vocab) return 4;
        or_dequant_row(m->embed.dt, m->embed.data, m->embed.scales, m->embed.cols, toks[t], m->bx + t * h);
    }
    float *tmp = (float *)malloc((size_t)h * 4);
    for (int layer = 0; layer < s->n_layers; layer++) {
        for (int t = 0; t < n; t++) {
            memcpy(m->x, m->bx + t * h, (size_t)h * 4);
            or_attention(m, layer, m->pos + t);
            memcpy(m->bx + t * h, m->x, (size_t)h * 4);
        }
        for (int t = 0; t < n; t++)
            or_route_topk(m, layer, m->bx + t * h, m->bxb + t * h, m->bsel + t * OR_MAX_TOPK,
                          m->bw + t * OR_MAX_TOPK);
        for (int e = 0; e < s->n_experts; e++)
            for (int t = 0; t < n; t++)
                for (int i = 0; i < s->top_k; i++)
                    if (m->bsel[t * OR_MAX_TOPK + i] == e) {
                        m->usage[(size_t)layer * s->n_experts + e]++;
                        m->expert_loads++;
                        or_expert_ffn(m, layer, e, m->bxb + t * h, tmp);
                        float wt = m->bw[t * OR_MAX_TOPK + i];
                        float *xo = m->bx + t * h;
                        for (int64_t j = 0; j < h; j++) xo[j] += wt * tmp[j];
                    }
    }
    free(tmp);
    for (int t = 0; t < n; t++) {
        int want = tfall || (want_last && t == n - 1);
        if (want) {
            or_logits(m, m->bx + t * h);
            if (logits_out) memcpy(logits_out + (tfall ? (size_t)t * s->vocab : 0), m->logits, (size_t)s->vocab * 4);
        }
    }
    m->pos += n;
    return 0;
}

int or_model_pos(const or_model *m) { return m->pos; }
void or_model_set_pos(or_model *m, int pos) { m->pos = pos; }
const uint32_t *or_model_usage(const or_model *m) { return m->usage; }
uint64_t or_model_expert_loads(const or_model *m) { return m->expert_loads; }

/* Final hidden state rows of the last forward_batch call (for layer-level checks). */
const float *or_model_bx(const or_model *m) { return m->bx; }
const float *or_model_x(const or_model *m) { return m->x; }

void or_model_free(or_model *m) {
    if (!m) return;
    for (int i = 0; i < m->s.n_layers; i++) { free(m->kc[i]); free(m->vc[i]); }
    free(m->kc); free(m->vc);
    free(m->wq); free(m->wk); free(m->wv); free(m->wo); free(m->router_w);
    free((void *)m->bq); free((void *)m->bk); free((void *)m->bv); free((void *)m->bo);
    free((void *)m->router_b); free((void *)m->attn_norm); free((void *)m->mlp_norm);
    free((void *)m->sink); free((void *)m->qn); free((void *)m->kn);
    free(m->x); free(m->xb); free(m->moe); free(m->q); free(m->k); free(m->v); free(m->ao);
    free(m->att); free(m->hb); free(m->hb2); free(m->rl); free(m->logits);
    free(m->bx); free(m->bxb); free(m->bw); free(m->bsel); free(m->usage);
    free(m->rope_cos); free(m->rope_sin);
    free(m);
}

/* ------------------------------------------------- stand-alone pieces */

/* Router for a batch of normed inputs: logits (AVX2 f32 order + bias), top-k
 * (decode or prefill variant) and weights. */
void or_route(const float *xb, int n_tok, const float *rw, const float *rb, int n_experts, int64_t hidden,
              int k, int router_norm, int prefill_variant, float *logits, int *sel, float *w) {
    float val[OR_MAX_TOPK];
    for (int t = 0; t < n_tok; t++) {
        float *rl = logits + (size_t)t * n_experts;
        or_mv_f32(rw, xb + (size_t)t * hidden, rl, n_experts, hidden);
        or_addbias(rl, rb, n_experts);
        if (prefill_variant) or_topk_prefill(rl, n_experts, k, sel + t * k, val);
        else or_topk_decode(rl, n_experts, k, sel + t * k, val);
        or_route_weights(rl, n_experts, val, k, router_norm, w + t * k);
    }
}

/* xorshift64* sampler state and temperature/top-p sampling;
 * engine/midge.c:642-678 */
static int or_pi_cmp(const void *a, const void *b) {
    float pa = ((const float *)a)[0], pb = ((const float *)b)[0];
    return pa < pb ? 1 : pa > pb ? -1 : 0;
}

int or_sample(const float *logits, int64_t V, float temp, float topp, uint64_t *rng) {
    if (temp <= 0.f) { /* greedy: strict >, first maximum wins */
        int best = 0;
        float bv = logits[0];
        for (int64_t i = 1; i < V; i++) if (logits[i] > bv) { bv = logits[i]; best = (int)i; }
        return best;
    }
    float mx = logits[0];
    for (int64_t i = 1; i < V; i++) if (logits[i] > mx) mx = logits[i];
    float *probs = (float *)malloc(V * 4);
    double den = 0;
    for (int64_t i = 0; i < V; i++) { probs[i] = expf((logits[i] - mx) / temp); den += probs[i]; }
    for (int64_t i = 0; i < V; i++) probs[i] /= (float)den;
    struct { float p; int i; } *pi = malloc(V * 8);
    for (int64_t i = 0; i < V; i++) { pi[i].p = probs[i]; pi[i].i = (int)i; }
    qsort(pi, V, 8, or_pi_cmp);
    double cum = 0;
    int64_t n = 0;
    for (; n < V; n++) { cum += pi[n].p; if (cum >= topp) { n++; break; } }
    uint64_t st = *rng;
    st ^= st >> 12; st ^= st << 25; st ^= st >> 27;
    *rng = st;
    uint32_t u = (uint32_t)((st * 0x2545F4914F6CDD1DULL) >> 32);
    float r = (u >> 8) / 16777216.0f * (float)cum;
    double acc = 0;
    int pick = pi[n - 1].i;
    for (int64_t i = 0; i < n; i++) { acc += pi[i].p; if (r <= acc) { pick = pi[i].i; break; } }
    free(pi);
    free(probs);
    return pick;
}

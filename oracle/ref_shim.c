/* ref_shim.c -- exposes the reference engine's own functions as a library.
 *
 * TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the reference
 * sources where they lie (engine/midge.c, engine/mkern.h, engine/mten.h,
 * engine/mjson.h of drmihirbrahme/midge); no reference source is copied into this
 * repository.  The result, oracle/_ref/libmidgeref.so, is the reference itself,
 * used to pin oracle/oracle.c bit for bit on the same inputs.
 */
#define main midge_reference_main
#include "midge.c"
#undef main

/* wk_matvec on a caller-described matrix (engine/mkern.h:180) */
void ref_matvec(int dt, const void *data, const void *scales, int64_t rows, int64_t cols,
                const float *x, float *y) {
    WT t;
    t.dt = dt; t.rows = rows; t.cols = cols; t.data = data; t.scales = scales;
    wk_matvec(&t, x, y);
}

/* wk_row (engine/mkern.h:201) */
void ref_row(int dt, const void *data, const void *scales, int64_t rows, int64_t cols, int64_t r,
             float *out) {
    WT t;
    t.dt = dt; t.rows = rows; t.cols = cols; t.data = data; t.scales = scales;
    wk_row(&t, r, out);
}

void ref_rmsnorm(const float *x, const float *w, float *out, int64_t n, float eps) {
    wk_rmsnorm(x, w, out, n, eps);
}

uint16_t ref_to_f16(float f) { return wk_to_f16(f); }
float ref_f16(uint16_t h) { return wt_f16(h); }

/* model_load (engine/midge.c:204) on a converted model directory */
void *ref_model_load(const char *dir, int ctx) {
    Model *m = (Model *)calloc(1, sizeof(Model));
    model_load(m, dir, ctx);
    return m;
}

int ref_vocab(void *mp) { return (int)((Model *)mp)->s.vocab; }
int ref_pos(void *mp) { return ((Model *)mp)->pos; }

/* forward (engine/midge.c:552) with logits copied out */
void ref_forward(void *mp, int tok, float *logits) {
    Model *m = (Model *)mp;
    forward(m, tok, 1);
    memcpy(logits, m->logits, (size_t)m->s.vocab * 4);
}

/* forward_batch (engine/midge.c:576) for one chunk, last-position logits only */
void ref_forward_batch(void *mp, const int *toks, int n, float *logits) {
    Model *m = (Model *)mp;
    forward_batch(m, toks, n, 0, 1);
    memcpy(logits, m->logits, (size_t)m->s.vocab * 4);
}

/* route_topk (engine/midge.c:404) on an externally supplied residual row */
void ref_route_topk(void *mp, int layer, const float *x, float *xb, int *sel, float *w) {
    route_topk((Model *)mp, layer, x, xb, sel, w);
}

const uint32_t *ref_usage(void *mp) { return ((Model *)mp)->usage; }

void ref_model_free(void *mp) {
    model_free((Model *)mp);
    free(mp);
}

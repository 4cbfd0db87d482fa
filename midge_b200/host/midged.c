/* midged.c -- the midge engine process on a B200: the reference's command line
 * and stdin/stdout token protocol (engine/midge.c:15-24, :722-841), with every
 * tensor resident in HBM and every forward pass on the GPU through the C ABI
 * of libmidgecuda.so (include/midgecuda.h).
 *
 * Boundary kept from the reference:
 *   argv:   <model_dir> [--ctx N] [--temp F] [--topp F] [--seed N] [--ngen N]
 *           [--stop id,id] [--preload-gb F] [--no-stats] | --bench
 *           plus --gpu N (or MIDGE_GPU) to pick the device
 *   stdin:  ids: / tf: / tfall: / gen: N / set: T P [seed] / quit
 *   stdout: LOADING, READY, T <id>, L <v..> (%.7g), OK <pos>, OK set,
 *           DONE <prompt> <gen> <sec> <expert_loads>
 *   stderr: "# ..." diagnostics; exit 2 = cannot open, 3 = bad spec/tensor,
 *           4 = context full / token out of range (engine/midge.c:209-211,
 *           :136, :195-201, :554-555).
 *   files:  dense.midge / experts.midge read unchanged (mmap), usage.bin
 *           u32[L x E] read at start and written after each gen and at quit.
 * MIDGE_NO_BATCH=1 selects the per-token prefill path (engine/midge.c:788).
 */
#include <errno.h>
#include <fcntl.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include "midgecuda.h"
#include "mjs.h"

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + ts.tv_nsec * 1e-9;
}

/* ------------------------------------------------------------ containers */
typedef struct {
    int fd;
    uint8_t *map;
    size_t size;
    uint8_t *base; /* 64-aligned data start */
    Js *hdr;
} Cont;

static int cont_open(Cont *c, const char *path) { /* engine/mten.h:84-98 layout */
    memset(c, 0, sizeof(*c));
    c->fd = open(path, O_RDONLY);
    if (c->fd < 0) return -1;
    struct stat st;
    if (fstat(c->fd, &st) != 0 || st.st_size < 8) return -1;
    c->size = (size_t)st.st_size;
    c->map = (uint8_t *)mmap(NULL, c->size, PROT_READ, MAP_SHARED, c->fd, 0);
    if (c->map == MAP_FAILED) { c->map = NULL; return -1; }
    uint64_t hl;
    memcpy(&hl, c->map, 8);
    if (hl > c->size - 8) { errno = EINVAL; return -1; }
    c->hdr = js_parse((const char *)c->map + 8, (size_t)hl);
    if (!c->hdr) { errno = EINVAL; return -1; }
    c->base = c->map + ((8 + hl + 63) & ~(uint64_t)63);
    return 0;
}

static void cont_close(Cont *c) {
    js_free(c->hdr);
    if (c->map) munmap(c->map, c->size);
    if (c->fd > 0) close(c->fd);
}

static int dt_code(const char *s) {
    if (!s) return -1;
    if (!strcmp(s, "f32")) return MG_F32;
    if (!strcmp(s, "q8r")) return MG_Q8R;
    if (!strcmp(s, "q4g32")) return MG_Q4G32;
    if (!strcmp(s, "mxfp4")) return MG_MXFP4;
    return -1;
}

static void blob_sizes(int dt, int64_t rows, int64_t cols, size_t *db, size_t *sb) {
    *sb = 0;
    if (cols == 0) { *db = (size_t)rows * 4; return; }
    switch (dt) {
    case MG_F32: *db = (size_t)rows * cols * 4; break;
    case MG_Q8R: *db = (size_t)rows * cols; *sb = (size_t)rows * 4; break;
    default: *db = (size_t)rows * cols / 2; *sb = (size_t)rows * (cols / 32) * 2; break;
    }
}

/* ----------------------------------------------------------------- spec */
/* the engine's spec with the reference's defaults (engine/midge.c:95-138) */
static int spec_load(mg_spec *s, int **sliding, const Js *j) {
    memset(s, 0, sizeof(*s));
    s->hidden = (int64_t)js_num(j, "hidden", 0);
    s->vocab = (int64_t)js_num(j, "vocab", 0);
    s->n_layers = (int)js_num(j, "n_layers", 0);
    s->n_heads = (int)js_num(j, "n_heads", 0);
    s->n_kv_heads = (int)js_num(j, "n_kv_heads", 0);
    s->head_dim = (int)js_num(j, "head_dim", 64);
    s->norm_eps = (float)js_num(j, "norm_eps", 1e-5);
    const Js *moe = js_get(j, "moe");
    s->ffn = (int64_t)js_num(moe, "ffn", 0);
    s->n_experts = (int)js_num(moe, "experts", 0);
    s->top_k = (int)js_num(moe, "top_k", 0);
    s->alpha = (float)js_num(moe, "alpha", 1.702);
    s->limit = (float)js_num(moe, "limit", 7.0);
    const char *act = js_str(moe, "act", "swiglu_clamp");
    s->act_plain = act && !strcmp(act, "swiglu");
    s->router_norm = (int)js_num(moe, "router_norm", 1);
    const Js *attn = js_get(j, "attn");
    s->sliding_window = (int)js_num(attn, "sliding_window", 0);
    s->sinks = (int)js_num(attn, "sinks", 0);
    s->qk_norm = (int)js_num(attn, "qk_norm", 0);
    s->attn_scale = (float)js_num(attn, "scale", s->head_dim > 0 ? 1.0 / __builtin_sqrt((double)s->head_dim) : 1.0);
    if (!s->hidden || !s->vocab || !s->n_layers || !s->ffn || !s->n_experts || !s->top_k) return -1;
    *sliding = (int *)calloc(s->n_layers, sizeof(int));
    const Js *lt = js_get(attn, "layer_types");
    for (int i = 0; i < s->n_layers; i++) {
        const Js *e = js_at(lt, i);
        (*sliding)[i] = e && e->kind == 's' && strstr(e->str, "sliding") != NULL;
    }
    s->layer_sliding = *sliding;
    const Js *rope = js_get(j, "rope");
    s->rope_theta = (float)js_num(rope, "theta", 10000.0);
    const Js *y = js_get(rope, "yarn");
    if (y && y->kind == 'o') {
        s->yarn = 1;
        s->yarn_factor = (float)js_num(y, "factor", 1.0);
        s->yarn_beta_fast = (float)js_num(y, "beta_fast", 32.0);
        s->yarn_beta_slow = (float)js_num(y, "beta_slow", 1.0);
        s->yarn_orig_ctx = (int)js_num(y, "orig_ctx", 4096);
        s->yarn_truncate = (int)js_num(y, "truncate", 0);
    }
    return 0;
}

/* ------------------------------------------------------------- sampling */
/* xorshift64* and temperature / top-p sampling as engine/midge.c:642-678 */
static uint64_t rng_state = 0x853c49e6748fea9bULL;
static uint32_t rng_u32(void) {
    rng_state ^= rng_state >> 12;
    rng_state ^= rng_state << 25;
    rng_state ^= rng_state >> 27;
    return (uint32_t)((rng_state * 0x2545F4914F6CDD1DULL) >> 32);
}

typedef struct { float p; int i; } Prob;
static int prob_desc(const void *a, const void *b) {
    float pa = ((const Prob *)a)->p, pb = ((const Prob *)b)->p;
    return pa < pb ? 1 : pa > pb ? -1 : 0;
}

static int sample_topp(const float *logits, int64_t V, float temp, float topp) {
    float mx = logits[0];
    for (int64_t i = 1; i < V; i++) if (logits[i] > mx) mx = logits[i];
    Prob *pr = (Prob *)malloc(V * sizeof(Prob));
    double den = 0;
    for (int64_t i = 0; i < V; i++) { pr[i].p = expf((logits[i] - mx) / temp); den += pr[i].p; }
    for (int64_t i = 0; i < V; i++) { pr[i].p /= (float)den; pr[i].i = (int)i; }
    qsort(pr, V, sizeof(Prob), prob_desc);
    double cum = 0;
    int64_t n = 0;
    for (; n < V; n++) { cum += pr[n].p; if (cum >= topp) { n++; break; } }
    float r = (rng_u32() >> 8) / 16777216.0f * (float)cum;
    double acc = 0;
    int pick = pr[n - 1].i;
    for (int64_t i = 0; i < n; i++) { acc += pr[i].p; if (r <= acc) { pick = pr[i].i; break; } }
    free(pr);
    return pick;
}

static int argmax_host(const float *l, int64_t V) { /* engine/midge.c:657-660 */
    int best = 0;
    float bv = l[0];
    for (int64_t i = 1; i < V; i++) if (l[i] > bv) { bv = l[i]; best = (int)i; }
    return best;
}

/* ------------------------------------------------------------------ main */
static void die_mg(int rc, const char *what) {
    fprintf(stderr, "# %s: %s\n", what, mg_last_error());
    exit(rc == MG_ERR_RANGE ? 4 : rc == MG_ERR_SPEC ? 3 : rc == MG_ERR_ARG ? 3 : 5);
}

static void print_logits(const float *l, int64_t V) {
    fputc('L', stdout);
    for (int64_t i = 0; i < V; i++) printf(" %.7g", l[i]);
    fputc('\n', stdout);
}

static void usage_io(mg_model *m, const char *dir, const mg_spec *s, int save) {
    char p[1200];
    snprintf(p, sizeof(p), "%s/usage.bin", dir);
    size_t n = (size_t)s->n_layers * s->n_experts;
    uint32_t *u = (uint32_t *)calloc(n, 4);
    if (save) {
        if (mg_model_get_usage(m, u) == MG_OK) {
            FILE *f = fopen(p, "wb");
            if (f) { fwrite(u, 4, n, f); fclose(f); }
        }
    } else {
        FILE *f = fopen(p, "rb");
        if (f) {
            if (fread(u, 4, n, f) == n) mg_model_set_usage(m, u);
            fclose(f);
        }
    }
    free(u);
}

static int run_bench(int device) {
    double gbps = 0;
    int rc = mg_bench_gemv(MG_Q4G32, 2880, 2880, 1, 1.0, device, &gbps); /* engine/midge.c:691 shape */
    if (rc != MG_OK) { fprintf(stderr, "# bench failed: %s\n", mg_last_error()); return 1; }
    printf("BENCH q4g32_gbps=%.3f threads=gpu%d\n", gbps, device);
    return 0;
}

int main(int argc, char **argv) {
    const char *env_gpu = getenv("MIDGE_GPU");
    int device = env_gpu ? atoi(env_gpu) : 0;
    for (int i = 1; i + 1 < argc; i++) if (!strcmp(argv[i], "--gpu")) device = atoi(argv[i + 1]);
    if (argc > 1 && !strcmp(argv[1], "--bench")) return run_bench(device);
    const char *dir = NULL;
    int ctx = 4096, ngen_default = 512, stats = 1;
    float temp = 0.0f, topp = 0.9f;
    uint64_t seed = 42;
    int stops[64], n_stops = 0;
    for (int i = 1; i < argc; i++) { /* engine/midge.c:730-745 */
        if (!strcmp(argv[i], "--ctx") && i + 1 < argc) ctx = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--temp") && i + 1 < argc) temp = (float)atof(argv[++i]);
        else if (!strcmp(argv[i], "--topp") && i + 1 < argc) topp = (float)atof(argv[++i]);
        else if (!strcmp(argv[i], "--seed") && i + 1 < argc) seed = strtoull(argv[++i], NULL, 10);
        else if (!strcmp(argv[i], "--ngen") && i + 1 < argc) ngen_default = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--preload-gb") && i + 1 < argc) ++i; /* experts are HBM-resident */
        else if (!strcmp(argv[i], "--gpu") && i + 1 < argc) ++i;
        else if (!strcmp(argv[i], "--no-stats")) stats = 0;
        else if (!strcmp(argv[i], "--stop") && i + 1 < argc) {
            char *tok = strtok(argv[++i], ",");
            while (tok && n_stops < 64) { stops[n_stops++] = atoi(tok); tok = strtok(NULL, ","); }
        } else if (argv[i][0] != '-') dir = argv[i];
        else { fprintf(stderr, "# unknown arg %s\n", argv[i]); return 2; }
    }
    if (!dir) {
        fprintf(stderr, "usage: midged <model_dir> [--ctx N] [--temp F] [--topp F] [--seed N] [--ngen N] "
                        "[--stop id,id] [--preload-gb F] [--gpu N]\n");
        return 2;
    }
    rng_state = seed ? seed : 1;
    double t0 = now_s();
    setvbuf(stdout, NULL, _IOLBF, 0);
    printf("LOADING\n");
    fflush(stdout);

    char p[1200];
    Cont dense, experts;
    fprintf(stderr, "# loading %s\n", dir);
    snprintf(p, sizeof(p), "%s/dense.midge", dir);
    if (cont_open(&dense, p) != 0) { fprintf(stderr, "# cannot open %s: %s\n", p, strerror(errno)); return 2; }
    snprintf(p, sizeof(p), "%s/experts.midge", dir);
    if (cont_open(&experts, p) != 0) { fprintf(stderr, "# cannot open %s: %s\n", p, strerror(errno)); return 2; }
    const Js *jspec = js_get(dense.hdr, "spec");
    if (!jspec) { fprintf(stderr, "# dense.midge has no embedded spec\n"); return 3; }
    mg_spec spec;
    int *sliding = NULL;
    if (spec_load(&spec, &sliding, jspec) != 0) { fprintf(stderr, "# invalid spec\n"); return 3; }
    const char *edt_name = js_str(experts.hdr, "dt", "?");
    int edt = dt_code(edt_name);
    if (edt < 0) { fprintf(stderr, "# bad experts dtype %s\n", edt_name); return 3; }

    mg_model *m = NULL;
    int rc = mg_model_create(&spec, ctx, 1, device, &m);
    if (rc) die_mg(rc, "model create");
    const Js *tens = js_get(dense.hdr, "tensors");
    for (int i = 0; tens && i < tens->n; i++) {
        const Js *e = tens->kids[i];
        int dt = dt_code(js_str(e, "dt", "f32"));
        const Js *sh = js_get(e, "shape");
        int64_t rows = sh && sh->n > 0 ? (int64_t)sh->kids[0]->num : 0;
        int64_t cols = sh && sh->n > 1 ? (int64_t)sh->kids[1]->num : 0;
        double off = js_num(e, "off", 0), soff = js_num(e, "soff", -1);
        size_t db, sb;
        blob_sizes(dt, rows, cols, &db, &sb);
        if (dt < 0 || dense.base + (size_t)off + db > dense.map + dense.size) {
            fprintf(stderr, "# bad tensor %s\n", tens->keys[i]);
            return 3;
        }
        rc = mg_model_set_dense(m, tens->keys[i], dt, rows, cols, dense.base + (size_t)off,
                                soff >= 0 ? dense.base + (size_t)soff : NULL);
        if (rc) die_mg(rc, tens->keys[i]);
    }
    mg_expert_layout el;
    if (mg_expert_layout_init(&el, edt, spec.hidden, spec.ffn, spec.n_experts) != MG_OK) die_mg(MG_ERR_SPEC, "experts");
    size_t need = (size_t)spec.n_layers * el.layer_stride;
    size_t have = experts.size - (size_t)(experts.base - experts.map);
    if (have < need) { fprintf(stderr, "# experts.midge too small: need %zu data bytes\n", need); return 3; }
    fprintf(stderr, "# uploading experts (%.1f GB) to HBM\n", need / 1e9);
    rc = mg_model_set_experts(m, edt, experts.base, need);
    if (rc) die_mg(rc, "experts upload");
    rc = mg_model_ready(m);
    if (rc) die_mg(rc, "model");
    usage_io(m, dir, &spec, 0);
    cont_close(&experts); /* everything needed now lives in HBM */
    fprintf(stderr, "# midge ready in %.1fs · layers=%d experts=%d topk=%d hidden=%lld vocab=%lld ctx=%d expert_dt=%s gpu=%d\n",
            now_s() - t0, spec.n_layers, spec.n_experts, spec.top_k, (long long)spec.hidden, (long long)spec.vocab,
            ctx, edt_name, device);
    printf("READY\n");
    fflush(stdout);

    const int64_t V = spec.vocab;
    float *logits = (float *)calloc(V, 4);
    int have_logits = 1, next_greedy = 0;  /* logits (host) or the device argmax describe the position */
    const char *nb = getenv("MIDGE_NO_BATCH");
    int no_batch = nb != NULL;
    char *line = NULL;
    size_t cap = 0;
    int prompt_toks = 0;
    while (getline(&line, &cap, stdin) > 0) {
        char *nl = strchr(line, '\n');
        if (nl) *nl = 0;
        if (!strncmp(line, "set:", 4)) { /* engine/midge.c:764-773 */
            char *q = line + 4;
            double t = strtod(q, &q), tp = strtod(q, &q);
            temp = (float)t;
            topp = (float)tp;
            while (*q == ' ') q++;
            if (*q) rng_state = strtoull(q, NULL, 10) | 1ull;
            printf("OK set\n");
            fflush(stdout);
            continue;
        }
        if (!strncmp(line, "ids:", 4) || !strncmp(line, "tf:", 3) || !strncmp(line, "tfall:", 6)) {
            int tf = line[0] == 't', tfall = !strncmp(line, "tfall:", 6);
            char *q = strchr(line, ':') + 1;
            double ts = now_s();
            int count = 0, capn = 64;
            int32_t *toks = (int32_t *)malloc(capn * sizeof(int32_t));
            while (*q) {
                while (*q == ' ') q++;
                if (!*q) break;
                if (count == capn) toks = (int32_t *)realloc(toks, (capn *= 2) * sizeof(int32_t));
                toks[count++] = (int32_t)strtol(q, &q, 10);
            }
            prompt_toks += count;
            if (no_batch) {
                for (int i = 0; i < count; i++) {
                    int32_t am = 0;
                    rc = mg_forward(m, 0, toks[i], logits, &am);
                    if (rc) die_mg(rc, "forward");
                    if (tfall) print_logits(logits, V);
                }
            } else if (count > 0) {
                if (tfall) {
                    float *all = (float *)malloc((size_t)count * V * 4);
                    rc = mg_forward_batch(m, 0, toks, count, 2, all);
                    if (rc) die_mg(rc, "forward_batch");
                    for (int i = 0; i < count; i++) print_logits(all + (size_t)i * V, V);
                    memcpy(logits, all + (size_t)(count - 1) * V, V * 4);
                    free(all);
                } else {
                    rc = mg_forward_batch(m, 0, toks, count, 1, logits);
                    if (rc) die_mg(rc, "forward_batch");
                }
            }
            have_logits = 1;
            free(toks);
            if (tf && !tfall) print_logits(logits, V);
            if (tf) {
                printf("DONE %d 0 %.3f %llu\n", count, now_s() - ts, (unsigned long long)mg_model_expert_loads(m));
                fflush(stdout);
                continue;
            }
            fprintf(stderr, "# prefill %d toks in %.2fs (%.2f tok/s)\n", count, now_s() - ts,
                    count / (now_s() - ts + 1e-9));
            printf("OK %d\n", mg_model_pos(m, 0));
            fflush(stdout);
        } else if (!strncmp(line, "gen:", 4)) { /* engine/midge.c:808-832 */
            int ngen = atoi(line + 4);
            if (ngen <= 0) ngen = ngen_default;
            double ts = now_s();
            uint64_t loads0 = mg_model_expert_loads(m);
            int produced = 0;
            for (int i = 0; i < ngen && mg_model_pos(m, 0) < ctx; i++) {
                int tok;
                if (temp <= 0.f) tok = have_logits ? argmax_host(logits, V) : next_greedy;
                else {
                    if (!have_logits) {
                        rc = mg_model_logits(m, 0, logits);
                        if (rc) die_mg(rc, "logits");
                    }
                    tok = sample_topp(logits, V, temp, topp);
                }
                printf("T %d\n", tok);
                fflush(stdout);
                produced++;
                int is_stop = 0;
                for (int j = 0; j < n_stops; j++) if (stops[j] == tok) is_stop = 1;
                if (is_stop) break;
                int32_t am = 0;
                rc = mg_forward(m, 0, tok, temp <= 0.f ? NULL : logits, &am);
                if (rc) die_mg(rc, "forward");
                have_logits = temp > 0.f;
                next_greedy = am;
            }
            double dt = now_s() - ts;
            if (stats)
                fprintf(stderr, "# gen %d toks in %.2fs (%.2f tok/s) · %llu expert loads · pos=%d\n", produced, dt,
                        produced / (dt + 1e-9), (unsigned long long)(mg_model_expert_loads(m) - loads0),
                        mg_model_pos(m, 0));
            printf("DONE %d %d %.3f %llu\n", prompt_toks, produced, dt,
                   (unsigned long long)(mg_model_expert_loads(m) - loads0));
            fflush(stdout);
            usage_io(m, dir, &spec, 1);
            prompt_toks = 0;
        } else if (!strcmp(line, "quit")) {
            break;
        }
    }
    usage_io(m, dir, &spec, 1);
    free(line);
    free(logits);
    mg_model_free(m);
    cont_close(&dense);
    free(sliding);
    return 0;
}

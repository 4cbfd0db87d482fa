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
 * Extension (opt-in, --seqs N > 1: N concurrent contexts; absent from the
 * reference, which serves one): "seq: i" selects the sequence that ids:,
 * tf:, tfall:, gen: and set:'s seed act on (reply "OK seq i"); "genall: N
 * [i j ...]" decodes the listed sequences (default: every one with a context)
 * together, N steps, one "TS <seq> <id>" line per token, then DONE.  A
 * sequence that draws a stop token or fills its context leaves the batch.
 * Sequence s > 0 starts its generator at seed ^ (s * 0x9E3779B97F4A7C15) | 1.
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
    if (!strcmp(s, "mxfp4e8")) return MG_MXFP4_E8; /* opt-in ue8m0-scale experts (midge_b200/convert_ue8m0.py) */
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

/* ---------------------------------------------------- sequences, sampling */
/* Every next token is chosen on the GPU (mg_model_sample: the reference's
 * greedy argmax or temperature / top-p draw with its xorshift64* generator,
 * engine/midge.c:642-678) from the logits the last forward left in a device
 * row.  The reference holds one context; --seqs N holds N (a protocol
 * extension: seq: selects the sequence ids:/tf:/tfall:/gen: act on, genall:
 * decodes several at once).  Each sequence remembers where its pending
 * next-token logits are: a device row, or a host copy made when another
 * sequence's forward pass was about to overwrite that row. */
typedef struct {
    int has;      /* next-token logits exist (after ids:/tf:/tfall:/gen:) */
    int dev_row;  /* device logits row holding them, or -1 (host copy hl) */
    float *hl;
    uint64_t rng; /* generator state (sequence 0: the reference's rng_state) */
    int prompt;   /* prompt tokens since the last gen (DONE's first field) */
} Seq;

static Seq *S;
static int NS;
static int64_t V;

static void die_mg(int rc, const char *what);

static void to_host(mg_model *m, int s) {
    if (S[s].dev_row < 0) return;
    if (!S[s].hl) S[s].hl = (float *)malloc((size_t)V * 4);
    int rc = mg_model_logits(m, S[s].dev_row, S[s].hl);
    if (rc) die_mg(rc, "logits");
    S[s].dev_row = -1;
}

/* before a forward pass of the sequences in keep[]: the other sequences'
 * pending logits leave the device rows (the pass overwrites them) */
static void park_others(mg_model *m, const int *keep, int nkeep) {
    for (int s = 0; s < NS; s++) {
        int kept = 0;
        for (int j = 0; j < nkeep; j++) kept |= keep[j] == s;
        if (!kept && S[s].has) to_host(m, s);
    }
}

/* the pending logits of sequences list[i] into device rows i (zeros, the
 * reference's fresh m->logits, for a sequence that has none) */
static void place_rows(mg_model *m, const int *list, int n) {
    park_others(m, list, n);
    for (int i = 0; i < n; i++)
        if (S[list[i]].dev_row >= 0 && S[list[i]].dev_row != i) to_host(m, list[i]);
    for (int i = 0; i < n; i++) {
        Seq *q = &S[list[i]];
        if (q->dev_row == i) continue;
        if (!q->hl) q->hl = (float *)calloc((size_t)V, 4);
        int rc = mg_model_put_logits(m, i, q->hl);
        if (rc) die_mg(rc, "logits");
        q->dev_row = i;
        q->has = 1;
    }
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
    int ctx = 4096, ngen_default = 512, stats = 1, n_seqs = 1;
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
        else if (!strcmp(argv[i], "--seqs") && i + 1 < argc) n_seqs = atoi(argv[++i]);
        else if (!strcmp(argv[i], "--stop") && i + 1 < argc) {
            char *tok = strtok(argv[++i], ",");
            while (tok && n_stops < 64) { stops[n_stops++] = atoi(tok); tok = strtok(NULL, ","); }
        } else if (argv[i][0] != '-') dir = argv[i];
        else { fprintf(stderr, "# unknown arg %s\n", argv[i]); return 2; }
    }
    if (!dir) {
        fprintf(stderr, "usage: midged <model_dir> [--ctx N] [--temp F] [--topp F] [--seed N] [--ngen N] "
                        "[--stop id,id] [--preload-gb F] [--gpu N] [--seqs N]\n");
        return 2;
    }
    if (n_seqs < 1 || n_seqs > 16) { fprintf(stderr, "# --seqs %d: 1..16\n", n_seqs); return 2; }
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
    char edt_name[16];  /* copied: the header is freed once the experts are in HBM */
    snprintf(edt_name, sizeof(edt_name), "%s", js_str(experts.hdr, "dt", "?"));
    int edt = dt_code(edt_name);
    if (edt < 0) { fprintf(stderr, "# bad experts dtype %s\n", edt_name); return 3; }

    mg_model *m = NULL;
    int rc = mg_model_create(&spec, ctx, n_seqs, device, &m);
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

    V = spec.vocab;
    NS = n_seqs;
    S = (Seq *)calloc(NS, sizeof(Seq));
    for (int i = 0; i < NS; i++) {
        S[i].dev_row = -1;
        S[i].rng = i == 0 ? (seed ? seed : 1) : ((seed ^ (0x9E3779B97F4A7C15ull * (uint64_t)i)) | 1ull);
    }
    float *logits = (float *)calloc(V, 4);
    const char *nb = getenv("MIDGE_NO_BATCH");
    int no_batch = nb != NULL;
    char *line = NULL;
    size_t cap = 0;
    int cur = 0;  /* the selected sequence */
    while (getline(&line, &cap, stdin) > 0) {
        char *nl = strchr(line, '\n');
        if (nl) *nl = 0;
        if (!strncmp(line, "set:", 4)) { /* engine/midge.c:764-773 */
            char *q = line + 4;
            double t = strtod(q, &q), tp = strtod(q, &q);
            temp = (float)t;
            topp = (float)tp;
            while (*q == ' ') q++;
            if (*q) S[cur].rng = strtoull(q, NULL, 10) | 1ull;
            printf("OK set\n");
            fflush(stdout);
            continue;
        }
        if (!strncmp(line, "seq:", 4)) {
            int i = atoi(line + 4);
            if (i < 0 || i >= NS) { fprintf(stderr, "# sequence %d out of range (--seqs %d)\n", i, NS); exit(4); }
            cur = i;
            printf("OK seq %d\n", cur);
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
            S[cur].prompt += count;
            park_others(m, &cur, 1);
            if (no_batch) {
                for (int i = 0; i < count; i++) {
                    int32_t am = 0;
                    rc = mg_forward(m, cur, toks[i], logits, &am);
                    if (rc) die_mg(rc, "forward");
                    if (tfall) print_logits(logits, V);
                }
            } else if (count > 0) {
                if (tfall) {
                    float *all = (float *)malloc((size_t)count * V * 4);
                    rc = mg_forward_batch(m, cur, toks, count, 2, all);
                    if (rc) die_mg(rc, "forward_batch");
                    for (int i = 0; i < count; i++) print_logits(all + (size_t)i * V, V);
                    memcpy(logits, all + (size_t)(count - 1) * V, V * 4);
                    free(all);
                } else {
                    rc = mg_forward_batch(m, cur, toks, count, 1, logits);
                    if (rc) die_mg(rc, "forward_batch");
                }
            }
            if (count > 0) {  /* the last position's logits: host copy here, device row 0 */
                S[cur].has = 1;
                S[cur].dev_row = 0;
            }
            free(toks);
            if (tf && !tfall) print_logits(logits, V);
            if (tf) {
                printf("DONE %d 0 %.3f %llu\n", count, now_s() - ts, (unsigned long long)mg_model_expert_loads(m));
                fflush(stdout);
                continue;
            }
            fprintf(stderr, "# prefill %d toks in %.2fs (%.2f tok/s)\n", count, now_s() - ts,
                    count / (now_s() - ts + 1e-9));
            printf("OK %d\n", mg_model_pos(m, cur));
            fflush(stdout);
        } else if (!strncmp(line, "gen:", 4)) { /* engine/midge.c:808-832 */
            int ngen = atoi(line + 4);
            if (ngen <= 0) ngen = ngen_default;
            double ts = now_s();
            uint64_t loads0 = mg_model_expert_loads(m);
            int produced = 0;
            place_rows(m, &cur, 1);
            for (int i = 0; i < ngen && mg_model_pos(m, cur) < ctx; i++) {
                int32_t tok = 0;
                rc = mg_model_sample(m, 1, temp, topp, &S[cur].rng, &tok);
                if (rc) die_mg(rc, "sample");
                printf("T %d\n", tok);
                fflush(stdout);
                produced++;
                int is_stop = 0;
                for (int j = 0; j < n_stops; j++) if (stops[j] == tok) is_stop = 1;
                if (is_stop) break;
                rc = mg_forward(m, cur, tok, NULL, NULL);
                if (rc) die_mg(rc, "forward");
                S[cur].dev_row = 0;
            }
            double dt = now_s() - ts;
            if (stats)
                fprintf(stderr, "# gen %d toks in %.2fs (%.2f tok/s) · %llu expert loads · pos=%d\n", produced, dt,
                        produced / (dt + 1e-9), (unsigned long long)(mg_model_expert_loads(m) - loads0),
                        mg_model_pos(m, cur));
            printf("DONE %d %d %.3f %llu\n", S[cur].prompt, produced, dt,
                   (unsigned long long)(mg_model_expert_loads(m) - loads0));
            fflush(stdout);
            usage_io(m, dir, &spec, 1);
            S[cur].prompt = 0;
        } else if (!strncmp(line, "genall:", 7)) { /* extension: concurrent decode of several sequences */
            char *q = line + 7;
            int ngen = (int)strtol(q, &q, 10);
            if (ngen <= 0) ngen = ngen_default;
            int list[16], n = 0;
            while (*q && n < NS) {
                while (*q == ' ') q++;
                if (!*q) break;
                int i = (int)strtol(q, &q, 10);
                if (i < 0 || i >= NS) { fprintf(stderr, "# sequence %d out of range (--seqs %d)\n", i, NS); exit(4); }
                list[n++] = i;
            }
            if (n == 0)
                for (int i = 0; i < NS; i++) if (S[i].has) list[n++] = i;
            double ts = now_s();
            uint64_t loads0 = mg_model_expert_loads(m);
            int produced = 0, prompt = 0;
            for (int i = 0; i < n; i++) { prompt += S[list[i]].prompt; S[list[i]].prompt = 0; }
            if (n > 0) place_rows(m, list, n);
            int32_t toks[16], seqs[16];
            uint64_t rngs[16];
            for (int step = 0; step < ngen && n > 0; step++) {
                for (int i = 0; i < n; i++) rngs[i] = S[list[i]].rng;
                rc = mg_model_sample(m, n, temp, topp, rngs, toks);
                if (rc) die_mg(rc, "sample");
                int a = 0;
                for (int i = 0; i < n; i++) {
                    Seq *sq = &S[list[i]];
                    sq->rng = rngs[i];
                    printf("TS %d %d\n", list[i], toks[i]);
                    produced++;
                    int leave = mg_model_pos(m, list[i]) + 1 > ctx;
                    for (int j = 0; j < n_stops; j++) leave |= stops[j] == toks[i];
                    if (leave) {  /* not forwarded (engine/midge.c:818-820): its logits stay pending */
                        to_host(m, list[i]);
                        continue;
                    }
                    seqs[a] = list[i];
                    toks[a] = toks[i];
                    a++;
                }
                fflush(stdout);
                n = a;
                for (int i = 0; i < n; i++) list[i] = seqs[i];
                if (n == 0) break;
                rc = mg_decode_step(m, n, seqs, toks, NULL, NULL);
                if (rc) die_mg(rc, "decode");
                for (int i = 0; i < n; i++) S[list[i]].dev_row = i;
            }
            double dt = now_s() - ts;
            if (stats)
                fprintf(stderr, "# genall %d toks in %.2fs (%.2f tok/s)\n", produced, dt, produced / (dt + 1e-9));
            printf("DONE %d %d %.3f %llu\n", prompt, produced, dt,
                   (unsigned long long)(mg_model_expert_loads(m) - loads0));
            fflush(stdout);
            usage_io(m, dir, &spec, 1);
        } else if (!strcmp(line, "quit")) {
            break;
        }
    }
    usage_io(m, dir, &spec, 1);
    free(line);
    free(logits);
    for (int i = 0; i < NS; i++) free(S[i].hl);
    free(S);
    mg_model_free(m);
    cont_close(&dense);
    free(sliding);
    return 0;
}

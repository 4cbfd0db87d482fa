/* mjs.h -- a small JSON reader for container headers and model specs.
 *
 * Derived from the reference engine's reader (engine/mjson.h of
 * drmihirbrahme/midge), whose node shape (kind letters o/a/s/n/b/z, num, str,
 * n, keys, kids), cursor and get / at / number-or-default / string-or-default
 * / free interface it keeps so that the host reads specs exactly as midged
 * does; object and array parsing share one loop here, nesting depth is
 * limited and arrays grow by powers of two.
 *
 * Parses a complete document into a tree of nodes (objects keep key order);
 * numbers are doubles; string escapes are decoded (\uXXXX becomes '?', which
 * is all the headers need).  Lookups return NULL for missing keys so callers
 * can apply the engine's defaults.
 */
#ifndef MJS_H
#define MJS_H
#include <stdlib.h>
#include <string.h>

typedef struct Js Js;
struct Js {
    char kind;   /* 'o' object, 'a' array, 's' string, 'n' number, 'b' bool, 'z' null */
    double num;
    char *str;
    int n;
    char **keys;
    Js **kids;
};

typedef struct { const char *p, *end; int bad; } JsIn;

static void js_skip(JsIn *in) {
    while (in->p < in->end && (*in->p == ' ' || *in->p == '\n' || *in->p == '\r' || *in->p == '\t')) in->p++;
}

static Js *js_node(char kind) {
    Js *j = (Js *)calloc(1, sizeof(Js));
    j->kind = kind;
    return j;
}

static void js_add(Js *parent, char *key, Js *kid) {
    if ((parent->n & (parent->n - 1)) == 0) { /* grow at powers of two */
        int cap = parent->n ? parent->n * 2 : 1;
        parent->kids = (Js **)realloc(parent->kids, sizeof(Js *) * cap);
        if (parent->kind == 'o') parent->keys = (char **)realloc(parent->keys, sizeof(char *) * cap);
    }
    if (parent->kind == 'o') parent->keys[parent->n] = key;
    parent->kids[parent->n++] = kid;
}

static char *js_string(JsIn *in) {
    if (in->p >= in->end || *in->p != '"') { in->bad = 1; return NULL; }
    in->p++;
    size_t cap = 16, len = 0;
    char *s = (char *)malloc(cap);
    while (in->p < in->end && *in->p != '"') {
        char c = *in->p++;
        if (c == '\\' && in->p < in->end) {
            char e = *in->p++;
            c = e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e == 'b' ? '\b' : e == 'f' ? '\f' : e;
            if (e == 'u') { in->p += (in->end - in->p >= 4) ? 4 : in->end - in->p; c = '?'; }
        }
        if (len + 2 > cap) s = (char *)realloc(s, cap *= 2);
        s[len++] = c;
    }
    if (in->p < in->end) in->p++; else in->bad = 1;
    s[len] = 0;
    return s;
}

static Js *js_value(JsIn *in, int depth) {
    js_skip(in);
    if (in->p >= in->end || depth > 64) { in->bad = 1; return NULL; }
    char c = *in->p;
    if (c == '{' || c == '[') {
        Js *j = js_node(c == '{' ? 'o' : 'a');
        char close = c == '{' ? '}' : ']';
        in->p++;
        js_skip(in);
        if (in->p < in->end && *in->p == close) { in->p++; return j; }
        while (!in->bad) {
            char *key = NULL;
            if (j->kind == 'o') {
                js_skip(in);
                key = js_string(in);
                js_skip(in);
                if (in->p >= in->end || *in->p != ':') { in->bad = 1; free(key); break; }
                in->p++;
            }
            Js *v = js_value(in, depth + 1);
            if (!v) { free(key); break; }
            js_add(j, key, v);
            js_skip(in);
            if (in->p < in->end && *in->p == ',') { in->p++; continue; }
            if (in->p < in->end && *in->p == close) { in->p++; break; }
            in->bad = 1;
        }
        return j;
    }
    if (c == '"') {
        Js *j = js_node('s');
        j->str = js_string(in);
        return j;
    }
    if (!strncmp(in->p, "true", 4) || !strncmp(in->p, "false", 5)) {
        Js *j = js_node('b');
        j->num = in->p[0] == 't';
        in->p += in->p[0] == 't' ? 4 : 5;
        return j;
    }
    if (!strncmp(in->p, "null", 4)) { in->p += 4; return js_node('z'); }
    char *e = NULL;
    double v = strtod(in->p, &e);
    if (e == in->p) { in->bad = 1; return NULL; }
    Js *j = js_node('n');
    j->num = v;
    in->p = e;
    return j;
}

static Js *js_parse(const char *text, size_t len) {
    JsIn in = {text, text + len, 0};
    Js *j = js_value(&in, 0);
    return in.bad ? NULL : j;
}

static Js *js_get(const Js *o, const char *key) {
    if (!o || o->kind != 'o') return NULL;
    for (int i = 0; i < o->n; i++) if (o->keys[i] && !strcmp(o->keys[i], key)) return o->kids[i];
    return NULL;
}

static Js *js_at(const Js *a, int i) { return (a && a->kind == 'a' && i >= 0 && i < a->n) ? a->kids[i] : NULL; }

static double js_num(const Js *o, const char *key, double dflt) {
    Js *v = js_get(o, key);
    return (v && (v->kind == 'n' || v->kind == 'b')) ? v->num : dflt;
}

static const char *js_str(const Js *o, const char *key, const char *dflt) {
    Js *v = js_get(o, key);
    return (v && v->kind == 's') ? v->str : dflt;
}

static void js_free(Js *j) {
    if (!j) return;
    for (int i = 0; i < j->n; i++) {
        js_free(j->kids[i]);
        if (j->keys) free(j->keys[i]);
    }
    free(j->kids);
    free(j->keys);
    free(j->str);
    free(j);
}
#endif /* MJS_H */

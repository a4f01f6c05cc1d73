/* Minimal GGUF reader for the oracle (TEST INFRASTRUCTURE ONLY). See gguf_min.h. */
#include "gguf_min.h"

#include <fcntl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static char g_err[256];
const char *gm_error(void) { return g_err; }

size_t gm_type_row_bytes(int type, int64_t n) {
    switch (type) {
        case GM_T_F32: return (size_t) n * 4;
        case GM_T_F16: return (size_t) n * 2;
        case GM_T_Q4_0: return (size_t) (n / 32) * 18;
        case GM_T_Q4_1: return (size_t) (n / 32) * 20;
        case GM_T_Q8_0: return (size_t) (n / 32) * 34;
        case GM_T_Q6_K: return (size_t) (n / 256) * 210;
        default: return 0;
    }
}

typedef struct { const uint8_t *p, *end; int bad; } rd;
static uint64_t take(rd *r, size_t n) {
    uint64_t v = 0;
    if (r->bad || (size_t) (r->end - r->p) < n) { r->bad = 1; return 0; }
    memcpy(&v, r->p, n);
    r->p += n;
    return v;
}
static char *take_str(rd *r) {
    uint64_t n = take(r, 8);
    if (r->bad || (uint64_t) (r->end - r->p) < n) { r->bad = 1; return NULL; }
    char *s = (char *) malloc(n + 1);
    memcpy(s, r->p, n);
    s[n] = 0;
    r->p += n;
    return s;
}
static size_t scalar_size(int t) {
    switch (t) {
        case GM_V_U8: case GM_V_I8: case GM_V_BOOL: return 1;
        case GM_V_U16: case GM_V_I16: return 2;
        case GM_V_U32: case GM_V_I32: case GM_V_F32: return 4;
        case GM_V_U64: case GM_V_I64: case GM_V_F64: return 8;
        default: return 0;
    }
}
static void skip_value(rd *r, int t) {
    if (t == GM_V_STR) { uint64_t n = take(r, 8); if (!r->bad && (uint64_t) (r->end - r->p) >= n) r->p += n; else r->bad = 1; return; }
    size_t s = scalar_size(t);
    if (!s) { r->bad = 1; return; }
    if ((size_t) (r->end - r->p) < s) { r->bad = 1; return; }
    r->p += s;
}

int gm_open(const char *path, gm_file *f) {
    memset(f, 0, sizeof *f);
    int fd = open(path, O_RDONLY);
    if (fd < 0) { snprintf(g_err, sizeof g_err, "cannot open %s", path); return -1; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { close(fd); snprintf(g_err, sizeof g_err, "%s: too short", path); return -1; }
    void *m = mmap(NULL, (size_t) st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (m == MAP_FAILED) { snprintf(g_err, sizeof g_err, "%s: mmap failed", path); return -1; }
    f->map = m;
    f->size = (size_t) st.st_size;
    rd r = { (const uint8_t *) m, (const uint8_t *) m + st.st_size, 0 };
    if (take(&r, 4) != 0x46554747u) { snprintf(g_err, sizeof g_err, "%s: not a GGUF file", path); gm_close(f); return -1; }
    uint32_t ver = (uint32_t) take(&r, 4);
    if (ver < 2 || ver > 3) { snprintf(g_err, sizeof g_err, "%s: GGUF version %u", path, ver); gm_close(f); return -1; }
    uint64_t nt = take(&r, 8), nkv = take(&r, 8);
    if (nt > (1u << 20) || nkv > (1u << 20)) { snprintf(g_err, sizeof g_err, "%s: bad counts", path); gm_close(f); return -1; }
    f->kv = (gm_kv *) calloc(nkv ? nkv : 1, sizeof(gm_kv));
    f->t = (gm_tensor *) calloc(nt ? nt : 1, sizeof(gm_tensor));
    uint64_t align = 32;
    for (uint64_t i = 0; i < nkv && !r.bad; i++) {
        gm_kv *kv = &f->kv[i];
        kv->key = take_str(&r);
        kv->type = (int) take(&r, 4);
        kv->val = r.p;
        f->n_kv = (int) i + 1;
        if (kv->type == GM_V_ARR) {
            kv->arr_type = (int) take(&r, 4);
            kv->arr_n = take(&r, 8);
            kv->arr_data = r.p;
            for (uint64_t k = 0; k < kv->arr_n && !r.bad; k++) skip_value(&r, kv->arr_type);
        } else {
            skip_value(&r, kv->type);
        }
        if (!r.bad && kv->key && strcmp(kv->key, "general.alignment") == 0 && kv->type == GM_V_U32) {
            uint32_t a; memcpy(&a, kv->val, 4); align = a ? a : 32;
        }
    }
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        gm_tensor *t = &f->t[i];
        t->name = take_str(&r);
        t->n_dims = (int) take(&r, 4);
        f->n_tensors = (int) i + 1;
        if (t->n_dims < 1 || t->n_dims > 4) { r.bad = 1; break; }
        for (int d = 0; d < 4; d++) t->ne[d] = d < t->n_dims ? (int64_t) take(&r, 8) : 1;
        t->type = (int) take(&r, 4);
        t->data = (const uint8_t *) (uintptr_t) take(&r, 8);   /* offset for now */
    }
    if (r.bad) { snprintf(g_err, sizeof g_err, "%s: truncated header", path); gm_close(f); return -1; }
    size_t hdr = (size_t) (r.p - (const uint8_t *) m);
    size_t base = (hdr + align - 1) / align * align;
    for (int i = 0; i < f->n_tensors; i++) {
        gm_tensor *t = &f->t[i];
        t->row_bytes = gm_type_row_bytes(t->type, t->ne[0]);
        t->nbytes = t->row_bytes * (size_t) (t->ne[1] * t->ne[2] * t->ne[3]);
        size_t off = base + (size_t) (uintptr_t) t->data;
        if (!t->row_bytes || off + t->nbytes > f->size) {
            snprintf(g_err, sizeof g_err, "%s: tensor %s has an unsupported type or runs past the end", path, t->name);
            gm_close(f);
            return -1;
        }
        t->data = (const uint8_t *) m + off;
    }
    return 0;
}

void gm_close(gm_file *f) {
    for (int i = 0; i < f->n_kv; i++) free(f->kv[i].key);
    for (int i = 0; i < f->n_tensors; i++) free(f->t[i].name);
    free(f->kv);
    free(f->t);
    if (f->map) munmap(f->map, f->size);
    memset(f, 0, sizeof *f);
}

const gm_tensor *gm_find(const gm_file *f, const char *name) {
    for (int i = 0; i < f->n_tensors; i++) if (f->t[i].name && strcmp(f->t[i].name, name) == 0) return &f->t[i];
    return NULL;
}
int gm_key(const gm_file *f, const char *key) {
    for (int i = 0; i < f->n_kv; i++) if (f->kv[i].key && strcmp(f->kv[i].key, key) == 0) return i;
    return -1;
}
int64_t gm_key_i(const gm_file *f, const char *key, int64_t def) {
    int k = gm_key(f, key);
    if (k < 0) return def;
    const gm_kv *kv = &f->kv[k];
    if (kv->type == GM_V_U32) { uint32_t v; memcpy(&v, kv->val, 4); return v; }
    if (kv->type == GM_V_I32) { int32_t v; memcpy(&v, kv->val, 4); return v; }
    if (kv->type == GM_V_U64) { uint64_t v; memcpy(&v, kv->val, 8); return (int64_t) v; }
    return def;
}
float gm_key_f(const gm_file *f, const char *key, float def) {
    int k = gm_key(f, key);
    if (k < 0 || f->kv[k].type != GM_V_F32) return def;
    float v;
    memcpy(&v, f->kv[k].val, 4);
    return v;
}

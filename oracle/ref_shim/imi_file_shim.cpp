// imi_file (the reference's imi/model.h interface) on top of the oracle's own GGUF reader, plus the three gguf_*
// calls seoul.cpp makes. TEST INFRASTRUCTURE ONLY. Behaviour follows imi/model.cpp: get() exits on a missing
// required tensor (model.cpp:108-115), keep() gives a tensor its own 64-byte aligned copy (model.cpp:138-150),
// drop_data() lets the file's bytes go (model.cpp:152-163). The CPU_REPACK buffer is never used here.
#include "model.h"
#include "gguf_min.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <immintrin.h>

struct gguf_context { gm_file f; };
struct ggml_context { std::vector<ggml_tensor> t; };

extern "C" {
int64_t gguf_find_key(const gguf_context *ctx, const char *key) { return gm_key(&ctx->f, key); }
const void *gguf_get_arr_data(const gguf_context *ctx, int64_t k) { return ctx->f.kv[k].arr_data; }
size_t gguf_get_arr_n(const gguf_context *ctx, int64_t k) { return (size_t) ctx->f.kv[k].arr_n; }
uint16_t ggml_fp32_to_fp16(float f) { return (uint16_t) _cvtss_sh(f, 0); }
}

ggml_backend_buffer_type_t imi_repack_buft() { return nullptr; }

bool imi_file::load(const std::string &path, bool repack) {
    (void) repack;
    meta = new gguf_context;
    if (gm_open(path.c_str(), &meta->f) != 0) {
        fprintf(stderr, "imi: cannot read %s (%s)\n", path.c_str(), gm_error());
        delete meta;
        meta = nullptr;
        return false;
    }
    ctx = new ggml_context;
    ctx->t.resize(meta->f.n_tensors);
    for (int i = 0; i < meta->f.n_tensors; i++) {
        const gm_tensor &s = meta->f.t[i];
        ggml_tensor &t = ctx->t[i];
        memset(&t, 0, sizeof t);
        t.type = (ggml_type) s.type;
        for (int d = 0; d < 4; d++) t.ne[d] = s.ne[d];
        t.nb[1] = s.row_bytes;
        t.nb[0] = s.ne[0] ? s.row_bytes / (size_t) s.ne[0] : 0;
        t.nb[2] = t.nb[1] * (size_t) s.ne[1];
        t.nb[3] = t.nb[2] * (size_t) s.ne[2];
        t.data = (void *) s.data;
        snprintf(t.name, sizeof t.name, "%s", s.name);
    }
    data = meta->f.map;
    size = meta->f.size;
    return true;
}

ggml_tensor *imi_file::get(const std::string &name, bool required) const {
    for (auto &t : ctx->t) if (name == t.name) return const_cast<ggml_tensor *>(&t);
    if (required) {
        fprintf(stderr, "imi: missing tensor %s\n", name.c_str());
        exit(1);
    }
    return nullptr;
}

int64_t imi_file::key_i(const std::string &name, int64_t def) const { return gm_key_i(&meta->f, name.c_str(), def); }
float imi_file::key_f(const std::string &name, float def) const { return gm_key_f(&meta->f, name.c_str(), def); }

static bool in_map(const ggml_tensor *t, const void *data, size_t size) {
    return data && t->data && (const char *) t->data >= (const char *) data && (const char *) t->data < (const char *) data + size;
}

ggml_tensor *imi_file::keep(const std::string &name, bool required) {
    ggml_tensor *t = get(name, required);
    if (!t || !in_map(t, data, size)) return t;
    const size_t n = t->nb[1] * (size_t) t->ne[1] * (size_t) t->ne[2] * (size_t) t->ne[3];
    void *p = nullptr;
    if (posix_memalign(&p, 64, (n + 63) / 64 * 64) != 0) { fprintf(stderr, "imi: out of memory keeping %s\n", t->name); exit(1); }
    memcpy(p, t->data, n);
    t->data = p;
    kept.push_back(p);
    return t;
}

void imi_file::drop_data() {
    if (!data) return;
    for (auto &t : ctx->t) if (in_map(&t, data, size)) t.data = nullptr;
    data = nullptr;   // the map itself stays: the keys (and arrays) still point into it
    size = 0;
}

imi_file::~imi_file() {
    for (void *p : kept) free(p);
    delete ctx;
    if (meta) { gm_close(&meta->f); delete meta; }
}

// imi_file_cuda.h - imi's model file (imi/model.h:17-36) over the engine library's own GGUF reader, header-only over
// imi_cuda.h, for callers that read the file's keys and tensors beside the brain.
//
// The reference reads GGUF through ggml's gguf library; this build has no ggml, so the same calls are provided over the
// library's reader: imi_file::load / get / key_i / key_f / keep / drop_data with the reference's meaning, and the gguf
// accessors the reference's callers use on `f.meta` (the tokenizer: gguf_find_key, gguf_get_arr_n, gguf_get_arr_data,
// gguf_get_arr_str, imi/core/words.cpp:49-88) on this header's own gguf_context. A tensor from get() carries the
// ggml_tensor fields callers read (type, ne, nb, data, name). Use this header instead of model.h (and ggml's headers):
// the two define the same names.
// Differences, all deliberate: the file is memory-mapped rather than read into one aligned block, so keep() and
// drop_data() only bookkeep (the bytes stay readable until the imi_file is destroyed); there is no CPU_REPACK buffer.
#pragma once
#include "imi_cuda.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>

// GGUF value types (the gguf format's numbering, as ggml's gguf.h names them)
enum gguf_type {
    GGUF_TYPE_UINT8 = 0, GGUF_TYPE_INT8 = 1, GGUF_TYPE_UINT16 = 2, GGUF_TYPE_INT16 = 3, GGUF_TYPE_UINT32 = 4,
    GGUF_TYPE_INT32 = 5, GGUF_TYPE_FLOAT32 = 6, GGUF_TYPE_BOOL = 7, GGUF_TYPE_STRING = 8, GGUF_TYPE_ARRAY = 9,
    GGUF_TYPE_UINT64 = 10, GGUF_TYPE_INT64 = 11, GGUF_TYPE_FLOAT64 = 12
};

// the file's keys: this header's gguf_context is the library's reader
struct gguf_context;
inline const imi_cuda_file *imi_gguf(const gguf_context *c) { return reinterpret_cast<const imi_cuda_file *>(c); }
inline int64_t gguf_find_key(const gguf_context *c, const char *key) { return imi_cuda_file_find_key(imi_gguf(c), key); }
inline int64_t gguf_get_n_kv(const gguf_context *c) { return imi_cuda_file_n_keys(imi_gguf(c)); }
inline const char *gguf_get_key(const gguf_context *c, int64_t k) { return imi_cuda_file_key_name(imi_gguf(c), k); }
inline enum gguf_type gguf_get_kv_type(const gguf_context *c, int64_t k) {
    return (enum gguf_type) imi_cuda_file_key_type(imi_gguf(c), k);
}
inline enum gguf_type gguf_get_arr_type(const gguf_context *c, int64_t k) {
    return (enum gguf_type) imi_cuda_file_arr_type(imi_gguf(c), k);
}
inline size_t gguf_get_arr_n(const gguf_context *c, int64_t k) { return (size_t) imi_cuda_file_arr_n(imi_gguf(c), k); }
inline const void *gguf_get_arr_data(const gguf_context *c, int64_t k) { return imi_cuda_file_arr_data(imi_gguf(c), k); }
inline const char *gguf_get_arr_str(const gguf_context *c, int64_t k, size_t i) {
    return imi_cuda_file_arr_str(imi_gguf(c), k, (uint64_t) i);
}
template <class T>
inline T imi_gguf_scalar(const gguf_context *c, int64_t k) {
    T v{};
    const void *p = imi_cuda_file_key_data(imi_gguf(c), k);
    if (p) memcpy(&v, p, sizeof v);
    return v;
}
inline uint32_t gguf_get_val_u32(const gguf_context *c, int64_t k) { return imi_gguf_scalar<uint32_t>(c, k); }
inline int32_t gguf_get_val_i32(const gguf_context *c, int64_t k) { return imi_gguf_scalar<int32_t>(c, k); }
inline uint64_t gguf_get_val_u64(const gguf_context *c, int64_t k) { return imi_gguf_scalar<uint64_t>(c, k); }
inline float gguf_get_val_f32(const gguf_context *c, int64_t k) { return imi_gguf_scalar<float>(c, k); }
inline bool gguf_get_val_bool(const gguf_context *c, int64_t k) { return imi_gguf_scalar<uint8_t>(c, k) != 0; }
inline const char *gguf_get_val_str(const gguf_context *c, int64_t k) { return imi_cuda_file_key_str(imi_gguf(c), k); }

// a tensor's header as the reference's callers read it (ggml_tensor: type, ne, nb, data, name)
struct ggml_tensor {
    int type = -1;
    int64_t ne[4] = { 1, 1, 1, 1 };
    size_t nb[4] = { 0, 0, 0, 0 };
    void *data = nullptr;
    char name[64] = {};
};

struct imi_file {
    gguf_context *meta = nullptr;   // the library's reader (gguf_* above)
    void *data = nullptr;           // not used: the file stays memory-mapped
    size_t size = 0;

    // imi/model.cpp:48-106: false (with a message on stderr) when the file cannot be read; repack is accepted and
    // ignored (no CPU kernels here)
    bool load(const std::string &path, bool repack = false) {
        (void) repack;
        imi_cuda_file *h = nullptr;
        if (imi_cuda_file_open(path.c_str(), &h) != IMI_OK) {
            fprintf(stderr, "imi: cannot read %s (%s)\n", path.c_str(), imi_cuda_error());
            return false;
        }
        close();
        meta = reinterpret_cast<gguf_context *>(h);
        return true;
    }
    // model.cpp:108-115: a missing required tensor ends the program
    ggml_tensor *get(const std::string &name, bool required = true) const {
        auto it = tensors.find(name);
        if (it != tensors.end()) return it->second.get();
        std::unique_ptr<ggml_tensor> t(new ggml_tensor);
        const void *d = nullptr;
        size_t nbytes = 0;
        if (!meta || imi_cuda_file_tensor(imi_gguf(meta), name.c_str(), &t->type, t->ne, &d, &nbytes) != 0) {
            if (required) {
                fprintf(stderr, "imi: missing tensor %s\n", name.c_str());
                exit(1);
            }
            return nullptr;
        }
        t->data = const_cast<void *>(d);
        const int64_t rows = t->ne[1] * t->ne[2] * t->ne[3];
        t->nb[1] = rows ? nbytes / (size_t) rows : 0;
        t->nb[2] = t->nb[1] * (size_t) t->ne[1];
        t->nb[3] = t->nb[2] * (size_t) t->ne[2];
        t->nb[0] = t->ne[0] ? t->nb[1] / (size_t) t->ne[0] : 0;   // whole bytes for unquantized types
        snprintf(t->name, sizeof t->name, "%s", name.c_str());
        ggml_tensor *raw = t.get();
        tensors.emplace(name, std::move(t));
        return raw;
    }
    // model.cpp:117-131
    int64_t key_i(const std::string &name, int64_t def) const {
        const int64_t k = meta ? gguf_find_key(meta, name.c_str()) : -1;
        if (k < 0) return def;
        switch (gguf_get_kv_type(meta, k)) {
            case GGUF_TYPE_UINT32: return gguf_get_val_u32(meta, k);
            case GGUF_TYPE_INT32: return gguf_get_val_i32(meta, k);
            case GGUF_TYPE_UINT64: return (int64_t) gguf_get_val_u64(meta, k);
            default: return def;
        }
    }
    float key_f(const std::string &name, float def) const {
        const int64_t k = meta ? gguf_find_key(meta, name.c_str()) : -1;
        return k < 0 ? def : gguf_get_val_f32(meta, k);
    }
    // model.cpp:138-163: the tensor's bytes stay readable (the file is mapped until this imi_file goes)
    ggml_tensor *keep(const std::string &name, bool required = true) { return get(name, required); }
    void drop_data() {}
    imi_file() = default;
    imi_file(const imi_file &) = delete;
    imi_file &operator=(const imi_file &) = delete;
    ~imi_file() { close(); }

private:
    mutable std::map<std::string, std::unique_ptr<ggml_tensor>> tensors;
    void close() {
        tensors.clear();
        imi_cuda_file_close(reinterpret_cast<imi_cuda_file *>(meta));
        meta = nullptr;
    }
};

// GGUF reader (format versions 2 and 3): header, key/values, tensor infos, aligned data. See gguf_file.h.
#include "gguf_file.h"

#include <cstring>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace imi {

size_t ggml_row_bytes(int type, int64_t n) {
    switch (type) {
        case T_F32: return (size_t) n * 4;
        case T_F16: return (size_t) n * 2;
        case T_Q4_0: return n % 32 ? 0 : (size_t) (n / 32) * 18;
        case T_Q4_1: return n % 32 ? 0 : (size_t) (n / 32) * 20;
        case T_Q8_0: return n % 32 ? 0 : (size_t) (n / 32) * 34;
        case T_Q6_K: return n % 256 ? 0 : (size_t) (n / 256) * 210;
        default: return 0;
    }
}

namespace {
struct reader {
    const uint8_t *p, *end;
    bool bad = false;
    template <class T> T get() {
        T v{};
        if (bad || (size_t) (end - p) < sizeof(T)) { bad = true; return v; }
        memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (bad || (uint64_t) (end - p) < n) { bad = true; return {}; }
        std::string s((const char *) p, n);
        p += n;
        return s;
    }
    void skip(int t) {
        static const int sz[13] = { 1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8 };
        if (t == 8) { str(); return; }
        if (t < 0 || t > 12 || t == 9) { bad = true; return; }
        if ((size_t) (end - p) < (size_t) sz[t]) { bad = true; return; }
        p += sz[t];
    }
};
}  // namespace

bool gguf_file::open(const std::string &path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) { error = "cannot open " + path; return false; }
    struct stat st;
    if (fstat(fd, &st) != 0 || st.st_size < 24) { ::close(fd); error = path + ": not a GGUF file"; return false; }
    void *m = mmap(nullptr, (size_t) st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (m == MAP_FAILED) { error = path + ": mmap failed"; return false; }
    map_ = m;
    size_ = (size_t) st.st_size;
    reader r{ (const uint8_t *) m, (const uint8_t *) m + size_ };
    if (r.get<uint32_t>() != 0x46554747u) { error = path + ": not a GGUF file"; return false; }
    const uint32_t ver = r.get<uint32_t>();
    if (ver < 2 || ver > 3) { error = path + ": unsupported GGUF version " + std::to_string(ver); return false; }
    const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
    if (nt > (1u << 20) || nkv > (1u << 20)) { error = path + ": corrupt header"; return false; }
    uint64_t align = 32;
    values.resize(nkv);
    for (auto &v : values) {
        v.key = r.str();
        v.type = (int) r.get<uint32_t>();
        v.val = r.p;
        if (v.type == 9) {
            v.arr_type = (int) r.get<uint32_t>();
            v.arr_n = r.get<uint64_t>();
            v.arr = r.p;
            for (uint64_t k = 0; k < v.arr_n && !r.bad; k++) r.skip(v.arr_type);
        } else {
            r.skip(v.type);
        }
        if (r.bad) break;
        if (v.key == "general.alignment" && v.type == 4) { uint32_t a; memcpy(&a, v.val, 4); align = a ? a : 32; }
    }
    tensors.resize(nt);
    std::vector<uint64_t> offs(nt);
    for (uint64_t i = 0; i < nt && !r.bad; i++) {
        gguf_tensor &t = tensors[i];
        t.name = r.str();
        t.n_dims = (int) r.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) { r.bad = true; break; }
        for (int d = 0; d < t.n_dims; d++) t.ne[d] = (int64_t) r.get<uint64_t>();
        t.type = (int) r.get<uint32_t>();
        offs[i] = r.get<uint64_t>();
    }
    if (r.bad) { error = path + ": truncated header"; return false; }
    const size_t hdr = (size_t) (r.p - (const uint8_t *) m), base = (hdr + align - 1) / align * align;
    for (uint64_t i = 0; i < nt; i++) {
        gguf_tensor &t = tensors[i];
        t.row_bytes = ggml_row_bytes(t.type, t.ne[0]);
        t.nbytes = t.row_bytes * (size_t) (t.ne[1] * t.ne[2] * t.ne[3]);
        if (t.row_bytes == 0) continue;   // a type the engine never reads: kept only by name
        if (base + offs[i] + t.nbytes > size_) { error = path + ": tensor " + t.name + " runs past the end"; return false; }
        t.data = (const uint8_t *) m + base + offs[i];
    }
    return true;
}

gguf_file::~gguf_file() {
    if (map_) munmap(map_, size_);
}

const gguf_tensor *gguf_file::tensor(const std::string &name) const {
    for (auto &t : tensors) if (t.name == name) return &t;
    return nullptr;
}
const gguf_value *gguf_file::value(const std::string &name) const {
    for (auto &v : values) if (v.key == name) return &v;
    return nullptr;
}
int64_t gguf_file::key_i(const std::string &name, int64_t def) const {
    const gguf_value *v = value(name);
    if (!v) return def;
    if (v->type == 4) { uint32_t x; memcpy(&x, v->val, 4); return x; }
    if (v->type == 5) { int32_t x; memcpy(&x, v->val, 4); return x; }
    if (v->type == 10) { uint64_t x; memcpy(&x, v->val, 8); return (int64_t) x; }
    return def;
}
float gguf_file::key_f(const std::string &name, float def) const {
    const gguf_value *v = value(name);
    if (!v || v->type != 6) return def;
    float x;
    memcpy(&x, v->val, 4);
    return x;
}

}  // namespace imi

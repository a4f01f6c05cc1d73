// GGUF model file, read-only and memory-mapped: the engine's replacement for imi_file (imi/model.h:12-36), which
// reads through ggml's gguf library. Keys and tensors are looked up by name; tensor bytes stay in the map until the
// engine has copied them to the device.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace imi {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q8_0 = 8, T_Q6_K = 14 };

struct gguf_tensor {
    std::string name;
    int type = -1, n_dims = 0;
    int64_t ne[4] = { 1, 1, 1, 1 };   // fastest first
    size_t row_bytes = 0, nbytes = 0;
    const uint8_t *data = nullptr;
};

struct gguf_value {
    std::string key;
    int type = -1;                      // gguf value type
    const uint8_t *val = nullptr;       // scalar / string body
    int arr_type = -1;
    uint64_t arr_n = 0;
    const uint8_t *arr = nullptr;
};

class gguf_file {
public:
    ~gguf_file();
    // false with a message in `error` on failure
    bool open(const std::string &path);
    const gguf_tensor *tensor(const std::string &name) const;
    int64_t key_i(const std::string &name, int64_t def) const;   // imi_file::key_i, model.cpp:117-126
    float key_f(const std::string &name, float def) const;       // imi_file::key_f, model.cpp:128-131
    const gguf_value *value(const std::string &name) const;
    std::string error;
    std::vector<gguf_tensor> tensors;
    std::vector<gguf_value> values;

private:
    void *map_ = nullptr;
    size_t size_ = 0;
};

size_t ggml_row_bytes(int type, int64_t n);

}  // namespace imi

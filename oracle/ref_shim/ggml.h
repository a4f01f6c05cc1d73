/* Shim for building the reference's imi/core/{seoul,tables}.cpp unmodified (TEST INFRASTRUCTURE ONLY).
 * ggml itself is not vendored under the reference tree; these are the few declarations those two files use,
 * written from scratch: the tensor header fields (type, ne, nb, data, name) and the ggml type ids of the GGUF
 * format. Nothing here is ggml code. */
#pragma once
#include <stddef.h>
#include <stdint.h>

enum ggml_type {
    GGML_TYPE_F32 = 0,
    GGML_TYPE_F16 = 1,
    GGML_TYPE_Q4_0 = 2,
    GGML_TYPE_Q4_1 = 3,
    GGML_TYPE_Q8_0 = 8,
#ifndef GGML_TYPE_Q6_K   /* the Q4_0 word-table build maps this name to GGML_TYPE_Q4_0 on the command line */
    GGML_TYPE_Q6_K = 14,
#endif
};

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[4];   /* elements, fastest first */
    size_t nb[4];    /* strides in bytes */
    void *data;
    char name[64];
};
struct ggml_context;

#ifdef __cplusplus
extern "C" {
#endif
uint16_t ggml_fp32_to_fp16(float f);
#ifdef __cplusplus
}
#endif

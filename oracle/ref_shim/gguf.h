/* Shim (TEST INFRASTRUCTURE ONLY): the three gguf calls imi/core/seoul.cpp makes (seoul.cpp:110-113). */
#pragma once
#include <stddef.h>
#include <stdint.h>
struct gguf_context;
#ifdef __cplusplus
extern "C" {
#endif
int64_t gguf_find_key(const struct gguf_context *ctx, const char *key);
const void *gguf_get_arr_data(const struct gguf_context *ctx, int64_t key_id);
size_t gguf_get_arr_n(const struct gguf_context *ctx, int64_t key_id);
#ifdef __cplusplus
}
#endif

/* Minimal GGUF (v2/v3) reader for the oracle. TEST INFRASTRUCTURE ONLY: nothing in the product links this.
 *
 * The reference reads GGUF through ggml's gguf library (imi/model.cpp:84-142, gguf_init_from_file), which is not
 * vendored in the reference tree. This reader is written from the public GGUF layout: magic "GGUF", version,
 * tensor count, key/value count, key/values, tensor infos (name, dims fastest-first, ggml type, offset), then the
 * tensor data at general.alignment (default 32). The file is mapped read-only; tensor data points into the map. */
#ifndef GGUF_MIN_H
#define GGUF_MIN_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

enum { GM_T_F32 = 0, GM_T_F16 = 1, GM_T_Q4_0 = 2, GM_T_Q4_1 = 3, GM_T_Q8_0 = 8, GM_T_Q6_K = 14 };
enum { GM_V_U8 = 0, GM_V_I8, GM_V_U16, GM_V_I16, GM_V_U32, GM_V_I32, GM_V_F32, GM_V_BOOL, GM_V_STR, GM_V_ARR,
       GM_V_U64, GM_V_I64, GM_V_F64 };

typedef struct {
    char *name;
    int type, n_dims;
    int64_t ne[4];        /* fastest first, unused dims 1 */
    size_t row_bytes;     /* bytes of one ne[0]-row */
    size_t nbytes;
    const uint8_t *data;  /* into the map */
} gm_tensor;

typedef struct {
    char *key;
    int type;             /* GM_V_* */
    const uint8_t *val;   /* scalar value, string (u64 len + bytes) or array body */
    int arr_type;         /* for arrays */
    uint64_t arr_n;
    const uint8_t *arr_data;
} gm_kv;

typedef struct {
    void *map;
    size_t size;
    int n_tensors, n_kv;
    gm_tensor *t;
    gm_kv *kv;
} gm_file;

/* 0 on success; on failure a message is left in gm_error() */
int gm_open(const char *path, gm_file *f);
void gm_close(gm_file *f);
const char *gm_error(void);
const gm_tensor *gm_find(const gm_file *f, const char *name);
int gm_key(const gm_file *f, const char *key);  /* index or -1 */
int64_t gm_key_i(const gm_file *f, const char *key, int64_t def);
float gm_key_f(const gm_file *f, const char *key, float def);
size_t gm_type_row_bytes(int type, int64_t n);  /* 0 for unknown types */

#ifdef __cplusplus
}
#endif
#endif

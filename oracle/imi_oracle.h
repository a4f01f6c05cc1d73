/* CPU restatement of imi's brain token loop (the oracle). TEST INFRASTRUCTURE ONLY: the product never links or
 * calls this; tests, __graft_entry__.smoke() and bench.py's cpu_baseline use it as the checker.
 *
 * Every float operation follows the order of imi's AVX2 path (imi/core/vec.h, imi/core/tables.cpp,
 * imi/core/seoul.cpp) so that, built with -ffp-contract=off, its results are bit-identical to the reference's own
 * code compiled unmodified from the reference tree (oracle/_ref). Pinned against that build by tests/test_oracle.py. */
#ifndef IMI_ORACLE_H
#define IMI_ORACLE_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_model or_model;
typedef struct or_state or_state;

/* load a Seoul/LFM3 GGUF (Q4_0 layer tables, Q4_0 tied word table). NULL on error (message in or_error()). */
or_model *or_load(const char *path, int n_ctx, int n_threads);
void or_free(or_model *m);
const char *or_error(void);
/* n_embd, n_vocab, n_ctx, n_layer, n_head, n_head_kv, head_dim, n_ff, d_conv, n_attn */
void or_info(const or_model *m, int out[10]);

or_state *or_state_new(const or_model *m);
void or_state_free(or_state *s);
void or_state_reset(const or_model *m, or_state *s);
int or_state_pos(const or_state *s);
const float *or_hidden(const or_state *s);
const float *or_logits(const or_state *s);
/* caches, for checks of the device state: K/V of attention layer ai, [n_ctx][kvd] fp16 bits; conv state of layer il,
 * [d_conv][n_embd] oldest first */
const uint16_t *or_k_cache(const or_state *s, int ai);
const uint16_t *or_v_cache(const or_state *s, int ai);
const float *or_conv_state(const or_state *s, int il);
/* test harness: overwrite position, K/V of positions 0..pos-1 ([n_attn][pos][kvd]) and conv memory
 * ([n_conv][d_conv][n_embd], conv layers in order) with another implementation's; -1 if pos > n_ctx */
int or_state_import(const or_model *m, or_state *s, int pos, const uint16_t *k, const uint16_t *v, const float *conv);

/* one position: token >= 0, or embd[n_embd]. 0 ok, 1 context full (state unchanged), as seoul.cpp:352-357 */
int or_step(const or_model *m, or_state *s, int32_t token, const float *embd, int want_logits);
/* n positions (tokens or embd[n][n_embd]); hidden_all[n][n_embd] optional. Same numbers as n steps: seoul.cpp:490-655 */
int or_step_batch(const or_model *m, or_state *s, const int32_t *tokens, const float *embd, int n, int want_logits,
                  float *hidden_all);

/* ---- kernel-level pieces (known-answer tests) ---- */
float or_rms_scale(const float *x, int n, float eps);                       /* vec.h:20-34 (AVX2 order) */
void or_cut(const float *x, int n, int8_t *q, float *d, float *s);           /* imi_q8::from, tables.cpp:100-109 */
/* per (row, block) integer dots of a Q4_0 matrix (GGUF rows) with 8-bit codes: s[rows][cols/32] */
void or_block_dots(const uint8_t *q4, int rows, int cols, const int8_t *xq, int32_t *s);
/* imi_q4_group's per-row result (tables.cpp:127-143) for ncol inputs, columns independent: out[ncol][rows] */
void or_q4_matvec(const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd, const float *xs, int ncol,
                  float *out, int n_threads);
uint16_t or_f2h(float f);   /* round to nearest even, as _cvtss_sh(f, 0) */
float or_h2f(uint16_t h);   /* imi_h2f, tables.cpp:20-29 */
/* the NEOX rotation table used by seoul.cpp:19-28 for one position: cos and sin of angle i (n/2 each) */
void or_rope_angles(int pos, int n, float base, const float *freq_factor, float *cs, float *sn);

/* ---- the Q6_K word table of the product's own files (next on the path; no GPU path yet) ---- */
void or_q8k_from(const float *x, int n, int8_t *q, float *d, int16_t *bsums);   /* imi_q8k::from, tables.cpp:200-213 */
/* one Q6_K row (210 B per 256 values) against an imi_q8k input, imi's AVX2 order (tables.cpp:235-278) */
float or_q6k_row(const uint8_t *row, const int8_t *xq, const float *xd, const int16_t *bsums, int nblocks);
void or_q6k_dequant_row(const uint8_t *row, float *y, int nblocks);             /* tables.cpp:216-233 */

#ifdef __cplusplus
}
#endif
#endif

/* CPU restatement of imi's brain token loop (the oracle). TEST INFRASTRUCTURE ONLY. See imi_oracle.h.
 *
 * Citations are to the reference tree: imi/core/seoul.cpp (the step), imi/core/tables.cpp (4-bit kernel and 8-bit
 * input cut), imi/core/vec.h (norms, cut), imi/model.cpp (file). Each float operation is written out in the order
 * imi's AVX2 code performs it; fmaf() stands for _mm256_fmadd_ps and friends. Rows of a table are independent, so
 * the OpenMP split over rows does not change any result. */
#include "imi_oracle.h"
#include "gguf_min.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char g_err[256];
const char *or_error(void) { return g_err; }

typedef struct { const uint8_t *w; int rows, cols; size_t row_bytes; int has_m; } or_table;   /* GGUF Q4_0 / Q4_1 rows */

typedef struct {
    const float *attn_norm, *post_attn_norm, *ffn_norm, *post_ffn_norm, *conv_w, *q_norm, *k_norm;
    or_table in_proj, out_proj, q, k, v, gate, o, ffn_gate, ffn_up, down;
    int conv, swa, ai;
} or_layer;

struct or_model {
    gm_file f;
    or_layer *L;
    or_table tok;
    int tok_q6k;   /* the word table is Q6_K (the product's own files) rather than Q4_0 */
    const float *out_norm, *rope_freqs;
    int n_layer, n_embd, n_vocab, n_head, n_head_kv, head_dim, n_ff, d_conv, n_swa, n_ctx, n_attn, n_threads;
    float eps, rope_base, rope_base_swa;
};

typedef struct { int8_t *q; float *d, *s; } q8v;

struct or_state {
    int n_layer, n_attn;
    uint16_t **k, **v;
    float **conv;
    int pos;
    float *hidden, *logits;
    /* scratch */
    float *x, *h, *big, *att, *y, *act, *fo, *sc;
    q8v qi;
    int16_t *bs;   /* code sums per 16 of the Q6_K head's input cut */
};

/* ---------------- small math (imi/core/vec.h, imi/core/tables.cpp:20-38) ---------------- */

float or_h2f(uint16_t h) {   /* tables.cpp:20-29 */
    const uint32_t s = (uint32_t) (h & 0x8000) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff;
    uint32_t b;
    if (e == 0) {
        if (m == 0) b = s;
        else { float f = (float) m / 1024.0f / 16384.0f; memcpy(&b, &f, 4); b |= s; }
    } else if (e == 31) b = s | 0x7f800000 | (m << 13);
    else b = s | ((e + 112) << 23) | (m << 13);
    float f; memcpy(&f, &b, 4); return f;
}

uint16_t or_f2h(float f) {   /* round to nearest even: the F16C conversion imi_f2h uses (tables.cpp:30-37) */
    uint32_t x; memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000, ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t) (sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 | ((ax >> 13) & 0x3ff) : 0));
    if (ax >= 0x477ff000u) return (uint16_t) (sign | 0x7c00);
    if (ax < 0x38800000u) {   /* below the smallest normal half: a multiple of 2^-24 */
        float af; memcpy(&af, &ax, 4);
        return (uint16_t) (sign | (uint32_t) rintf(af * 16777216.0f));
    }
    uint32_t h = ((((ax >> 23) - 112) << 10) | ((ax >> 13) & 0x3ff)), rem = ax & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (h & 1))) h++;
    return (uint16_t) (sign | h);
}

/* imi_rms_scale, AVX2 order (vec.h:20-28): 4 x 8 lane accumulators over strides of 32, lanes added a0+a1, a2+a3, then
 * the horizontal sum of imi_hsum (vec.h:12-16) */
float or_rms_scale(const float *x, int n, float eps) {
    float a[32];
    for (int l = 0; l < 32; l++) a[l] = 0.0f;
    for (int i = 0; i < n; i += 32)
        for (int l = 0; l < 32; l++) a[l] = fmaf(x[i + l], x[i + l], a[l]);
    float t[8];
    for (int l = 0; l < 8; l++) t[l] = (a[l] + a[8 + l]) + (a[16 + l] + a[24 + l]);
    float r[4];
    for (int m = 0; m < 4; m++) r[m] = t[m] + t[m + 4];
    const float s = (r[0] + r[2]) + (r[1] + r[3]);
    return 1.0f / sqrtf(s / (float) n + eps);
}
static void norm_mul(const float *x, const float *w, float *o, int n, float eps) {   /* vec.h:36-39 */
    const float sc = or_rms_scale(x, n, eps);
    for (int i = 0; i < n; i++) o[i] = x[i] * sc * w[i];
}
static void norm_mul_add(const float *y, const float *w, float *x, int n, float eps) {   /* vec.h:41-44 */
    const float sc = or_rms_scale(y, n, eps);
    for (int i = 0; i < n; i++) x[i] += y[i] * sc * w[i];
}
/* imi_cut32 (vec.h:47-77): d = max|x| / 127, q = round-half-even(x / d) via x * (1/d) */
static float cut32(const float *x, int8_t *q, int *sum) {
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) { const float v = fabsf(x[i]); amax = amax > v ? amax : v; }
    const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
    int s = 0;
    for (int i = 0; i < 32; i++) { const int c = (int) rintf(x[i] * id); q[i] = (int8_t) c; s += c; }
    *sum = s;
    return d;
}
void or_cut(const float *x, int n, int8_t *q, float *d, float *s) {   /* imi_q8::from, tables.cpp:100-109 */
    for (int j = 0; j < n / 32; j++) {
        int sum;
        d[j] = cut32(x + 32 * j, q + 32 * j, &sum);
        s[j] = d[j] * (float) sum;
    }
}

/* ---------------- the 4-bit table kernel ---------------- */

static inline int block_dot(const uint8_t *blk, const int8_t *xq) {   /* codes: byte i = col i | col 16+i << 4 */
    const uint8_t *qs = blk + 2;
    int s = 0;
    for (int i = 0; i < 16; i++) s += (qs[i] & 15) * xq[i] + (qs[i] >> 4) * xq[16 + i];
    return s;
}
/* one row of group_avx2<false> (tables.cpp:127-143): two fma chains over the blocks in order, then acc - 8 cor */
static float row_dot(const uint8_t *row, int nb, const int8_t *xq, const float *xd, const float *xs) {
    float acc = 0.0f, cor = 0.0f;
    for (int j = 0; j < nb; j++) {
        const uint8_t *blk = row + 18 * (size_t) j;
        uint16_t dh; memcpy(&dh, blk, 2);
        const float dd = or_h2f(dh);
        acc = fmaf((float) block_dot(blk, xq + 32 * j), dd * xd[j], acc);
        cor = fmaf(dd, xs[j], cor);
    }
    return fmaf(-8.0f, cor, acc);
}
/* one row of group_avx2<true> (Q4_1 blocks: d, m, 16 code bytes): the same acc chain, cor = fma(m, s_j, cor), and
 * acc + cor with one rounding (tables.cpp:136-142) */
static float row_dot_m(const uint8_t *row, int nb, const int8_t *xq, const float *xd, const float *xs) {
    float acc = 0.0f, cor = 0.0f;
    for (int j = 0; j < nb; j++) {
        const uint8_t *blk = row + 20 * (size_t) j;
        uint16_t dh, mh; memcpy(&dh, blk, 2); memcpy(&mh, blk + 2, 2);
        acc = fmaf((float) block_dot(blk + 2, xq + 32 * j), or_h2f(dh) * xd[j], acc);   /* codes at blk + 4 */
        cor = fmaf(or_h2f(mh), xs[j], cor);
    }
    return acc + cor;
}
static void matvec(const or_table *W, const q8v *x, float *out, int nt) {
    const int nb = W->cols / 32;
    #pragma omp parallel for num_threads(nt) schedule(static)
    for (int r = 0; r < W->rows; r++)
        out[r] = W->has_m ? row_dot_m(W->w + (size_t) r * W->row_bytes, nb, x->q, x->d, x->s)
                          : row_dot(W->w + (size_t) r * W->row_bytes, nb, x->q, x->d, x->s);
}
void or_block_dots(const uint8_t *q4, int rows, int cols, const int8_t *xq, int32_t *s) {
    const int nb = cols / 32;
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < nb; j++) s[(size_t) r * nb + j] = block_dot(q4 + ((size_t) r * nb + j) * 18, xq + 32 * j);
}
void or_q4_matvec(const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd, const float *xs, int ncol,
                  float *out, int n_threads) {
    const int nb = cols / 32;
    for (int c = 0; c < ncol; c++) {
        #pragma omp parallel for num_threads(n_threads > 0 ? n_threads : 1) schedule(static)
        for (int r = 0; r < rows; r++)
            out[(size_t) c * rows + r] = row_dot(q4 + (size_t) r * nb * 18, nb, xq + (size_t) c * cols,
                                                 xd + (size_t) c * nb, xs + (size_t) c * nb);
    }
}

/* ---------------- attention pieces (seoul.cpp:17-48) ---------------- */

void or_rope_angles(int pos, int n, float base, const float *ff, float *cs, float *sn) {   /* seoul.cpp:19-28 */
    const float scale = powf(base, -2.0f / (float) n);
    float th = (float) pos;
    for (int i = 0; i < n / 2; i++) {
        const float a = th / (ff ? ff[i] : 1.0f);
        cs[i] = cosf(a);
        sn[i] = sinf(a);
        th *= scale;
    }
}
static void rope(float *v, int n, int pos, float base, const float *ff) {
    float cs[256], sn[256];
    or_rope_angles(pos, n, base, ff, cs, sn);
    for (int i = 0; i < n / 2; i++) {
        const float x0 = v[i], x1 = v[i + n / 2];
        v[i] = x0 * cs[i] - x1 * sn[i];
        v[i + n / 2] = x0 * sn[i] + x1 * cs[i];
    }
}
static float dot_h(const float *q, const uint16_t *k, int n) {   /* seoul.cpp:29-35: 8 lanes, then imi_hsum order */
    float a[8] = { 0 };
    for (int i = 0; i < n; i += 8)
        for (int l = 0; l < 8; l++) a[l] = fmaf(q[i + l], or_h2f(k[i + l]), a[l]);
    const float r0 = a[0] + a[4], r1 = a[1] + a[5], r2 = a[2] + a[6], r3 = a[3] + a[7];
    return (r0 + r2) + (r1 + r3);
}
/* imi calls the C library's expf (seoul.cpp:48,446,451). Built with -DOR_EXPF_CR (liboracle_cr.so) the oracle uses
 * the correctly rounded exponential instead, the one the engine computes on the device: the two builds differ only
 * there, which lets the tests tell expf's own rounding apart from everything else. */
#ifdef OR_EXPF_CR
static inline float or_expf(float x) { return (float) exp((double) x); }
#else
static inline float or_expf(float x) { return expf(x); }
#endif
static inline float silu(float x) { return x / (1.0f + or_expf(-x)); }   /* seoul.cpp:48 */

/* ---------------- load (seoul.cpp:93-186 with a Q4_0 tied word table) ---------------- */

static int table(const gm_file *f, const char *name, or_table *t) {
    const gm_tensor *g = gm_find(f, name);
    if (!g) { snprintf(g_err, sizeof g_err, "missing tensor %s", name); return -1; }
    if (g->type != GM_T_Q4_0 && g->type != GM_T_Q4_1) {
        snprintf(g_err, sizeof g_err, "%s: only Q4_0 / Q4_1 tables are read here", name);
        return -1;
    }
    t->w = g->data; t->cols = (int) g->ne[0]; t->rows = (int) g->ne[1]; t->row_bytes = g->row_bytes;
    t->has_m = g->type == GM_T_Q4_1;
    return 0;
}
static const float *f32(const gm_file *f, const char *name, int required) {
    const gm_tensor *g = gm_find(f, name);
    if (!g) { if (required) snprintf(g_err, sizeof g_err, "missing tensor %s", name); return NULL; }
    return g->type == GM_T_F32 ? (const float *) g->data : NULL;
}

or_model *or_load(const char *path, int n_ctx, int n_threads) {
    or_model *m = (or_model *) calloc(1, sizeof *m);
    if (gm_open(path, &m->f) != 0) { snprintf(g_err, sizeof g_err, "%s", gm_error()); free(m); return NULL; }
    gm_file *f = &m->f;
    char nm[128];
    {
        const gm_tensor *te = gm_find(f, "token_embd.weight");
        if (te && te->type == GM_T_Q6_K) {   /* seoul.cpp:95-98: the reference's own word-table format */
            m->tok.w = te->data; m->tok.cols = (int) te->ne[0]; m->tok.rows = (int) te->ne[1];
            m->tok.row_bytes = te->row_bytes; m->tok_q6k = 1;
        } else if (table(f, "token_embd.weight", &m->tok)) goto fail;
    }
    m->n_embd = m->tok.cols; m->n_vocab = m->tok.rows;
    if (!(m->out_norm = f32(f, "output_norm.weight", 1))) goto fail;
    m->rope_freqs = f32(f, "rope_freqs.weight", 0);
    m->eps = gm_key_f(f, "lfm3.attention.layer_norm_rms_epsilon", 1e-5f);
    m->rope_base = gm_key_f(f, "lfm3.rope.freq_base", 1e6f);
    m->rope_base_swa = gm_key_f(f, "lfm3.rope.freq_base_swa", 1e4f);
    m->n_swa = (int) gm_key_i(f, "lfm3.attention.sliding_window", 0);
    m->d_conv = (int) gm_key_i(f, "lfm3.shortconv.l_cache", 7) - 1;
    m->n_head = (int) gm_key_i(f, "lfm3.attention.head_count", 16);
    m->head_dim = (int) gm_key_i(f, "lfm3.attention.key_length", 128);
    m->n_layer = (int) gm_key_i(f, "lfm3.block_count", 0);
    m->n_ctx = n_ctx;
    m->n_threads = n_threads > 0 ? n_threads : 1;
    m->L = (or_layer *) calloc(m->n_layer > 0 ? m->n_layer : 1, sizeof(or_layer));
    const int kswa = gm_key(f, "lfm3.attention.sliding_window_pattern");
    for (int il = 0; il < m->n_layer; il++) {
        or_layer *L = &m->L[il];
#define P(s) (snprintf(nm, sizeof nm, "blk.%d." s, il), nm)
        if (!(L->attn_norm = f32(f, P("attn_norm.weight"), 1))) goto fail;
        if (!(L->post_attn_norm = f32(f, P("post_attention_norm.weight"), 1))) goto fail;
        if (!(L->ffn_norm = f32(f, P("ffn_norm.weight"), 1))) goto fail;
        if (!(L->post_ffn_norm = f32(f, P("post_ffw_norm.weight"), 1))) goto fail;
        if ((L->conv_w = f32(f, P("shortconv.conv.weight"), 0))) {
            L->conv = 1;
            if (table(f, P("shortconv.in_proj.weight"), &L->in_proj) || table(f, P("shortconv.out_proj.weight"), &L->out_proj)) goto fail;
        } else {
            if (table(f, P("attn_q.weight"), &L->q) || table(f, P("attn_k.weight"), &L->k) ||
                table(f, P("attn_v.weight"), &L->v) || table(f, P("attn_gate.weight"), &L->gate) ||
                table(f, P("attn_output.weight"), &L->o)) goto fail;
            if (!(L->q_norm = f32(f, P("attn_q_norm.weight"), 1)) || !(L->k_norm = f32(f, P("attn_k_norm.weight"), 1))) goto fail;
            L->swa = (kswa >= 0 && (uint64_t) il < f->kv[kswa].arr_n) ? f->kv[kswa].arr_data[il] != 0 : 0;
            L->ai = m->n_attn++;
            m->n_head_kv = L->k.rows / m->head_dim;
        }
        if (table(f, P("ffn_gate.weight"), &L->ffn_gate) || table(f, P("ffn_up.weight"), &L->ffn_up) ||
            table(f, P("ffn_down.weight"), &L->down)) goto fail;
        m->n_ff = L->ffn_gate.rows;
#undef P
    }
    return m;
fail:
    or_free(m);
    return NULL;
}

void or_free(or_model *m) {
    if (!m) return;
    free(m->L);
    gm_close(&m->f);
    free(m);
}

void or_info(const or_model *m, int o[10]) {
    o[0] = m->n_embd; o[1] = m->n_vocab; o[2] = m->n_ctx; o[3] = m->n_layer; o[4] = m->n_head; o[5] = m->n_head_kv;
    o[6] = m->head_dim; o[7] = m->n_ff; o[8] = m->d_conv; o[9] = m->n_attn;
}

/* ---------------- conversation state (seoul.h:21-26, seoul.cpp:166-171,188-206) ---------------- */

or_state *or_state_new(const or_model *m) {
    or_state *s = (or_state *) calloc(1, sizeof *s);
    s->n_layer = m->n_layer;
    s->n_attn = m->n_attn;
    const int E = m->n_embd, kvd = m->n_head_kv * m->head_dim, HD = m->n_head * m->head_dim;
    int wide = E > m->n_ff ? E : m->n_ff;
    if (HD > wide) wide = HD;
    int big = 3 * E, qr = HD + 2 * kvd + m->n_head;
    if (qr > big) big = qr;
    if (m->n_ff > big) big = m->n_ff;
    s->k = (uint16_t **) calloc(m->n_attn + 1, sizeof(void *));
    s->v = (uint16_t **) calloc(m->n_attn + 1, sizeof(void *));
    for (int a = 0; a < m->n_attn; a++) {
        s->k[a] = (uint16_t *) calloc((size_t) m->n_ctx * kvd, 2);
        s->v[a] = (uint16_t *) calloc((size_t) m->n_ctx * kvd, 2);
    }
    s->conv = (float **) calloc(m->n_layer + 1, sizeof(void *));
    for (int il = 0; il < m->n_layer; il++)
        if (m->L[il].conv) s->conv[il] = (float *) calloc((size_t) m->d_conv * E, 4);
    s->hidden = (float *) calloc(E, 4);
    s->logits = (float *) calloc(m->n_vocab, 4);
    s->x = (float *) calloc(E, 4);
    s->h = (float *) calloc(wide, 4);
    s->big = (float *) calloc(big, 4);
    s->att = (float *) calloc(HD, 4);
    s->y = (float *) calloc(E, 4);
    s->act = (float *) calloc(m->n_ff, 4);
    s->fo = (float *) calloc(E, 4);
    s->sc = (float *) calloc(m->n_ctx + 1, 4);
    s->qi.q = (int8_t *) calloc(wide, 1);
    s->qi.d = (float *) calloc(wide / 32 + 1, 4);
    s->qi.s = (float *) calloc(wide / 32 + 1, 4);
    s->bs = (int16_t *) calloc(E / 16 + 1, 2);
    return s;
}
void or_state_free(or_state *s) {
    if (!s) return;
    for (int a = 0; a < s->n_attn; a++) { free(s->k[a]); free(s->v[a]); }
    free(s->k); free(s->v);
    for (int il = 0; il < s->n_layer; il++) free(s->conv[il]);
    free(s->conv);
    free(s->hidden); free(s->logits); free(s->x); free(s->h); free(s->big); free(s->att); free(s->y); free(s->act);
    free(s->fo); free(s->sc); free(s->qi.q); free(s->qi.d); free(s->qi.s); free(s->bs);
    free(s);
}
void or_state_reset(const or_model *m, or_state *s) {   /* seoul.cpp:188-191 (caches are overwritten before use) */
    s->pos = 0;
    for (int il = 0; il < m->n_layer; il++) if (s->conv[il]) memset(s->conv[il], 0, (size_t) m->d_conv * m->n_embd * 4);
}
int or_state_pos(const or_state *s) { return s->pos; }
const float *or_hidden(const or_state *s) { return s->hidden; }
const float *or_logits(const or_state *s) { return s->logits; }
const uint16_t *or_k_cache(const or_state *s, int ai) { return s->k[ai]; }
const uint16_t *or_v_cache(const or_state *s, int ai) { return s->v[ai]; }
const float *or_conv_state(const or_state *s, int il) { return s->conv[il]; }

/* test harness: start from another implementation's memory (k, v [n_attn][pos][kvd] fp16 bits; conv
 * [n_conv][d_conv][n_embd] fp32 per conv layer in layer order, oldest tap first; imi's layout, seoul.h:43-47), so one
 * step here and one step of the engine read identical memory. -1 if pos does not fit n_ctx. */
int or_state_import(const or_model *m, or_state *s, int pos, const uint16_t *k, const uint16_t *v, const float *conv) {
    if (pos < 0 || pos > m->n_ctx) return -1;
    const size_t kvd = (size_t) m->n_head_kv * m->head_dim, E = (size_t) m->n_embd;
    for (int a = 0; a < m->n_attn; a++) {
        memcpy(s->k[a], k + (size_t) a * pos * kvd, (size_t) pos * kvd * 2);
        memcpy(s->v[a], v + (size_t) a * pos * kvd, (size_t) pos * kvd * 2);
    }
    int ci = 0;
    for (int il = 0; il < m->n_layer; il++)
        if (s->conv[il]) memcpy(s->conv[il], conv + (size_t) (ci++) * m->d_conv * E, (size_t) m->d_conv * E * 4);
    s->pos = pos;
    return 0;
}

/* ---------------- one position (seoul.cpp:359-488) ---------------- */

/* the word scores of the hidden state: Q6_K (seoul.cpp:479-487 with imi_q8k / imi_q6k_row) or the Q4_0 adapter */
static void head(const or_model *m, or_state *s, int nt) {
    const int E = m->n_embd;
    if (m->tok_q6k) {
        or_q8k_from(s->hidden, E, s->qi.q, s->qi.d, s->bs);
#pragma omp parallel for num_threads(nt) schedule(static)
        for (int r = 0; r < m->n_vocab; r++)
            s->logits[r] = or_q6k_row(m->tok.w + (size_t) r * m->tok.row_bytes, s->qi.q, s->qi.d, s->bs, E / 256);
        return;
    }
    or_cut(s->hidden, E, s->qi.q, s->qi.d, s->qi.s);
    matvec(&m->tok, &s->qi, s->logits, nt);
}

static void lookup(const or_model *m, int32_t token, float *x) {   /* the word row, d * (code - 8) */
    if (m->tok_q6k) {   /* seoul.cpp:363: imi_q6k_dequant_row */
        or_q6k_dequant_row(m->tok.w + (size_t) token * m->tok.row_bytes, x, m->n_embd / 256);
        return;
    }
    const uint8_t *b = m->tok.w + (size_t) token * m->tok.row_bytes;
    for (int j = 0; j < m->n_embd / 32; j++, b += 18) {
        uint16_t dh; memcpy(&dh, b, 2);
        const float dd = or_h2f(dh);
        for (int i = 0; i < 16; i++) {
            x[32 * j + i] = dd * (float) ((b[2 + i] & 15) - 8);
            x[32 * j + 16 + i] = dd * (float) ((b[2 + i] >> 4) - 8);
        }
    }
}

static void run(const or_model *m, or_state *S, int32_t token, const float *embd, int want_logits) {
    const int E = m->n_embd, D = m->head_dim, H = m->n_head, kvd = m->n_head_kv * D, grp = H / m->n_head_kv;
    const int nt = m->n_threads, pos = S->pos;
    const float eps = m->eps;
    float *x = S->x;
    if (token >= 0) lookup(m, token, x); else memcpy(x, embd, (size_t) E * 4);   /* seoul.cpp:363-364 */
    for (int il = 0; il < m->n_layer; il++) {
        const or_layer *L = &m->L[il];
        norm_mul(x, L->attn_norm, S->h, E, eps);                                  /* seoul.cpp:404-405 */
        or_cut(S->h, E, S->qi.q, S->qi.d, S->qi.s);
        if (L->conv) {                                                            /* seoul.cpp:407-423 */
            matvec(&L->in_proj, &S->qi, S->big, nt);
            const float *b = S->big, *cc = b + E, *xx = b + 2 * E, *w = L->conv_w;
            float *st = S->conv[il], *u = S->h;
            const int K = m->d_conv + 1;
            for (int e = 0; e < E; e++) u[e] = b[e] * xx[e] * w[(size_t) e * K + m->d_conv];
            for (int k = 0; k < m->d_conv; k++)
                for (int e = 0; e < E; e++) u[e] += st[(size_t) k * E + e] * w[(size_t) e * K + k];
            for (int e = 0; e < E; e++) u[e] *= cc[e];
            or_cut(u, E, S->qi.q, S->qi.d, S->qi.s);
            matvec(&L->out_proj, &S->qi, S->y, nt);
            memmove(st, st + E, (size_t) (m->d_conv - 1) * E * 4);
            for (int e = 0; e < E; e++) st[(size_t) (m->d_conv - 1) * E + e] = b[e] * xx[e];
        } else {                                                                  /* seoul.cpp:424-460 */
            float *qkv = S->big;
            matvec(&L->q, &S->qi, qkv, nt);
            matvec(&L->k, &S->qi, qkv + H * D, nt);
            matvec(&L->v, &S->qi, qkv + H * D + kvd, nt);
            matvec(&L->gate, &S->qi, qkv + H * D + 2 * kvd, nt);
            const float base = L->swa ? m->rope_base_swa : m->rope_base;
            const float *ff = L->swa ? NULL : m->rope_freqs;
            uint16_t *kc = S->k[L->ai], *vc = S->v[L->ai];
            const int s0 = (L->swa && m->n_swa > 0) ? (pos - m->n_swa + 1 > 0 ? pos - m->n_swa + 1 : 0) : 0;
            const int nk = pos - s0 + 1;
            const float scale = 1.0f / sqrtf((float) D);
            for (int g = 0; g < m->n_head_kv; g++) {
                float kk[512];
                norm_mul(qkv + H * D + g * D, L->k_norm, kk, D, eps);
                rope(kk, D, pos, base, ff);
                const float *vv = qkv + H * D + kvd + g * D;
                for (int i = 0; i < D; i++) {
                    kc[(size_t) pos * kvd + g * D + i] = or_f2h(kk[i]);
                    vc[(size_t) pos * kvd + g * D + i] = or_f2h(vv[i]);
                }
                for (int hh = 0; hh < grp; hh++) {
                    const int h = g * grp + hh;
                    float q[512], o[512];
                    norm_mul(qkv + h * D, L->q_norm, q, D, eps);
                    rope(q, D, pos, base, ff);
                    float *sc = S->sc, mx = -INFINITY;
                    for (int t = 0; t < nk; t++) {
                        sc[t] = dot_h(q, kc + (size_t) (s0 + t) * kvd + g * D, D) * scale;
                        mx = mx < sc[t] ? sc[t] : mx;
                    }
                    double sum = 0;
                    for (int t = 0; t < nk; t++) { sc[t] = or_expf(sc[t] - mx); sum += sc[t]; }
                    const float inv = (float) (1.0 / sum);
                    for (int i = 0; i < D; i++) o[i] = 0.0f;
                    for (int t = 0; t < nk; t++) {
                        const float p = sc[t] * inv;
                        const uint16_t *vr = vc + (size_t) (s0 + t) * kvd + g * D;
                        for (int i = 0; i < D; i++) o[i] = fmaf(p, or_h2f(vr[i]), o[i]);
                    }
                    const float gate = 1.0f / (1.0f + or_expf(-qkv[H * D + 2 * kvd + h]));
                    for (int i = 0; i < D; i++) S->att[h * D + i] = o[i] * gate;
                }
            }
            or_cut(S->att, H * D, S->qi.q, S->qi.d, S->qi.s);
            matvec(&L->o, &S->qi, S->y, nt);
        }
        norm_mul_add(S->y, L->post_attn_norm, x, E, eps);                         /* seoul.cpp:462 */
        norm_mul(x, L->ffn_norm, S->h, E, eps);                                  /* seoul.cpp:464-470 */
        or_cut(S->h, E, S->qi.q, S->qi.d, S->qi.s);
        matvec(&L->ffn_gate, &S->qi, S->big, nt);                                /* gate rows, then up rows */
        matvec(&L->ffn_up, &S->qi, S->act, nt);
        for (int i = 0; i < m->n_ff; i++) S->act[i] = silu(S->big[i]) * S->act[i];   /* seoul.cpp:384-391 */
        or_cut(S->act, m->n_ff, S->qi.q, S->qi.d, S->qi.s);
        matvec(&L->down, &S->qi, S->fo, nt);
        norm_mul_add(S->fo, L->post_ffn_norm, x, E, eps);                        /* seoul.cpp:473 */
    }
    norm_mul(x, m->out_norm, S->hidden, E, eps);                                  /* seoul.cpp:475-477 */
    if (want_logits) head(m, S, nt);                                              /* seoul.cpp:479-487 */
}

int or_step(const or_model *m, or_state *s, int32_t token, const float *embd, int want_logits) {
    if (s->pos >= m->n_ctx) return 1;   /* seoul.cpp:353: "context full", no step */
    run(m, s, token, embd, want_logits);
    s->pos++;
    return 0;
}

int or_step_batch(const or_model *m, or_state *s, const int32_t *tokens, const float *embd, int n, int want_logits,
                  float *hidden_all) {
    const int E = m->n_embd, NB = 64;   /* seoul.h:90 */
    for (int i0 = 0; i0 < n; i0 += NB) {
        const int c = n - i0 < NB ? n - i0 : NB;
        if (s->pos + c > m->n_ctx) return 1;   /* seoul.cpp:498 */
        for (int p = 0; p < c; p++) {
            run(m, s, tokens ? tokens[i0 + p] : -1, embd ? embd + (size_t) (i0 + p) * E : NULL, 0);
            if (hidden_all) memcpy(hidden_all + (size_t) (i0 + p) * E, s->hidden, (size_t) E * 4);
            s->pos++;
        }
    }
    if (want_logits) head(m, s, m->n_threads);   /* seoul.cpp:507-516: the last position's scores */
    return 0;
}
/* ---- Q6_K word table (imi_q8k / imi_q6k_row / imi_q6k_dequant_row, tables.cpp:200-287) ---- */

/* imi_q8k::from (tables.cpp:200-213): per 256 values amax, d = amax/127, id = d ? 1/d : 0, q = lrintf(x * id),
 * bsums = the sum of each 16 codes */
void or_q8k_from(const float *x, int n, int8_t *q, float *d, int16_t *bsums) {
    for (int j = 0; j < n / 256; j++) {
        const float *v = x + 256 * j;
        float amax = 0.0f;
        for (int i = 0; i < 256; i++) amax = fmaxf(amax, fabsf(v[i]));
        const float dd = amax / 127.0f, id = dd != 0.0f ? 1.0f / dd : 0.0f;
        for (int i = 0; i < 256; i++) q[256 * j + i] = (int8_t) lrintf(v[i] * id);
        for (int s = 0; s < 16; s++) {
            int t = 0;
            for (int i = 0; i < 16; i++) t += q[256 * j + 16 * s + i];
            bsums[16 * j + s] = (int16_t) t;
        }
        d[j] = dd;
    }
}

/* the 6-bit code of value t (0..255) of a Q6_K block: low 4 bits from ql, high 2 from qh (tables.cpp:223-227) */
static inline int q6k_code(const uint8_t *blk, int t) {
    const int n = t / 128, r = t % 128, k = r / 32, l = r % 32;
    const uint8_t *ql = blk + 64 * n, *qh = blk + 128 + 32 * n;
    const int lo = k == 0 ? (ql[l] & 15) : k == 1 ? (ql[l + 32] & 15) : k == 2 ? (ql[l] >> 4) : (ql[l + 32] >> 4);
    return lo | (((qh[l] >> (2 * k)) & 3) << 4);
}

/* imi_q6k_row, AVX2 order (tables.cpp:235-278). Integer part per 256 block in 8 lanes: lane m takes values
 * 128n + 32k + 4m .. +3 (n < 2, k < 4) times the scale of their 16 (scales[8n + 2k + (m >= 4)]), minus
 * 32 * (scales[2m] * bsums[2m] + scales[2m+1] * bsums[2m+1]); exact in int32. Float part: lane m accumulates
 * fma(d_block * d_x, (float) int_m, acc_m) over the blocks in order; the 8 lanes end as
 * ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)). */
float or_q6k_row(const uint8_t *row, const int8_t *xq, const float *xd, const int16_t *bsums, int nblocks) {
    float acc[8] = { 0 };
    for (int i = 0; i < nblocks; i++) {
        const uint8_t *blk = row + 210 * (size_t) i;
        const int8_t *sc = (const int8_t *) (blk + 192);
        const uint16_t dh = (uint16_t) (blk[208] | (blk[209] << 8));
        const int8_t *x = xq + 256 * (size_t) i;
        const int16_t *bs = bsums + 16 * (size_t) i;
        int32_t lane[8];
        for (int m = 0; m < 8; m++) lane[m] = 0;
        for (int n = 0; n < 2; n++)
            for (int k = 0; k < 4; k++)
                for (int v = 0; v < 32; v++) {
                    const int t = 128 * n + 32 * k + v;
                    lane[v / 4] += q6k_code(blk, t) * x[t] * sc[8 * n + 2 * k + (v >= 16)];
                }
        for (int m = 0; m < 8; m++) lane[m] -= 32 * (sc[2 * m] * bs[2 * m] + sc[2 * m + 1] * bs[2 * m + 1]);
        const float s = or_h2f(dh) * xd[i];
        for (int m = 0; m < 8; m++) acc[m] = fmaf(s, (float) lane[m], acc[m]);
    }
    const float r0 = acc[0] + acc[4], r1 = acc[1] + acc[5], r2 = acc[2] + acc[6], r3 = acc[3] + acc[7];
    return (r0 + r2) + (r1 + r3);
}

/* imi_q6k_dequant_row (tables.cpp:216-233): value = d * scale * (code - 32), left to right */
void or_q6k_dequant_row(const uint8_t *row, float *y, int nblocks) {
    for (int i = 0; i < nblocks; i++) {
        const uint8_t *blk = row + 210 * (size_t) i;
        const int8_t *sc = (const int8_t *) (blk + 192);
        const float d = or_h2f((uint16_t) (blk[208] | (blk[209] << 8)));
        for (int t = 0; t < 256; t++) y[256 * i + t] = d * (float) sc[t / 16] * (float) (q6k_code(blk, t) - 32);
    }
}

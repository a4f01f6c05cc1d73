// C entry points over the reference's own imi_seoul and table kernels, for the Python test harness and the CPU
// baseline (TEST INFRASTRUCTURE ONLY). Everything computed here runs the reference's code: imi/core/seoul.cpp
// (load/step/step2/step_batch/new_state/swap_state) and imi/core/tables.cpp (imi_q4, imi_q8, imi_q8b kernels).
#include "seoul.h"

#include <cstdio>
#include <cstring>
#include <vector>

extern "C" {

void *oref_load(const char *path, int threads, int n_ctx) {
    imi_seoul *b = new imi_seoul;
    if (!b->load(path, threads, n_ctx)) { delete b; return nullptr; }
    return b;
}
void oref_free(void *h) { delete (imi_seoul *) h; }
void oref_reset(void *h) { ((imi_seoul *) h)->reset(); }
int oref_pos(void *h) { return ((imi_seoul *) h)->pos; }
void oref_info(void *h, int *o) {
    imi_seoul *b = (imi_seoul *) h;
    o[0] = b->n_embd; o[1] = b->n_vocab; o[2] = b->n_ctx; o[3] = (int) b->layers.size();
    o[4] = b->n_head; o[5] = b->n_head_kv; o[6] = b->head_dim; o[7] = b->n_ff; o[8] = b->d_conv; o[9] = b->n_threads;
}
void oref_step(void *h, int token, const float *embd, int want_logits) { ((imi_seoul *) h)->step(token, embd, want_logits != 0); }
void oref_step_batch(void *h, const int *tokens, const float *embd, int n, int want_logits, float *hidden_all) {
    ((imi_seoul *) h)->step_batch(tokens, embd, n, want_logits != 0, hidden_all);
}
const float *oref_hidden(void *h) { return ((imi_seoul *) h)->hidden.data(); }
const float *oref_logits(void *h) { return ((imi_seoul *) h)->logits.data(); }

void *oref_state_new(void *h) { return new imi_seoul_state(((imi_seoul *) h)->new_state()); }
void oref_state_free(void *s) { delete (imi_seoul_state *) s; }
void oref_swap(void *h, void *s) { ((imi_seoul *) h)->swap_state(*(imi_seoul_state *) s); }
int oref_state_pos(void *s) { return ((imi_seoul_state *) s)->pos; }
const float *oref_state_hidden(void *s) { return ((imi_seoul_state *) s)->hidden.data(); }
const float *oref_state_logits(void *s) { return ((imi_seoul_state *) s)->logits.data(); }
void oref_step2(void *h, int ta, const float *ea, int la, void *sb, int tb, const float *eb, int lb) {
    ((imi_seoul *) h)->step2(ta, ea, la != 0, *(imi_seoul_state *) sb, tb, eb, lb != 0);
}
double oref_bench_tables(void *h, int ncol, int reps) { return ((imi_seoul *) h)->bench_tables(ncol, reps); }

// ---- table kernels on a raw Q4_0 matrix (GGUF rows of 18-byte blocks) ----
static bool build_q4(imi_q4 &W, ggml_tensor &t, const void *q4, int rows, int cols) {
    memset(&t, 0, sizeof t);
    t.type = GGML_TYPE_Q4_0; t.ne[0] = cols; t.ne[1] = rows; t.ne[2] = t.ne[3] = 1;
    t.nb[1] = (size_t) cols / 32 * 18; t.data = (void *) q4;
    std::vector<std::pair<const ggml_tensor *, int>> o;
    for (int r = 0; r < rows; r++) o.push_back({ &t, r });
    return W.build(o);
}
// imi_q8::from: codes, scales and scale*sum per 32 values (tables.cpp:100-109)
void oref_cut(const float *x, int n, int8_t *q, float *d, float *s) {
    imi_q8 X; X.from(x, n);
    memcpy(q, X.q.data(), n); memcpy(d, X.d.data(), n / 32 * 4); memcpy(s, X.s.data(), n / 32 * 4);
}
// out[c][rows] for ncol inputs x[c][cols]: ncol 1 -> imi_q4_group, 2 -> imi_q4_group2, else imi_q8b + group_batch
int oref_q4_matvec(const void *q4, int rows, int cols, const float *x, int ncol, float *out) {
    imi_q4 W; ggml_tensor t;
    if (rows % 8 || cols % 32 || ncol < 1 || ncol > 64 || !build_q4(W, t, q4, rows, cols)) return -1;
    if (ncol <= 2) {
        imi_q8 X0, X1; X0.from(x, cols); if (ncol == 2) X1.from(x + cols, cols);
        for (int g = 0; g < rows / 8; g++) {
            if (ncol == 1) imi_q4_group(W, X0, g, out + 8 * g);
            else imi_q4_group2(W, X0, X1, g, out + 8 * g, out + rows + 8 * g);
        }
    } else {
        imi_q8b X; X.shape(ncol, cols);
        for (int c = 0; c < ncol; c++) X.set(c, x + (size_t) c * cols);
        std::vector<float> tmp(8 * ncol);
        for (int g = 0; g < rows / 8; g++) {
            imi_q4_group_batch(W, X, g, tmp.data());
            for (int c = 0; c < ncol; c++) memcpy(out + (size_t) c * rows + 8 * g, tmp.data() + 8 * c, 32);
        }
    }
    W.release();
    return 0;
}
}

// imi_brain_cuda.h - imi's older brain interface (imi/brain.h:33-64: load / reset / step, the hidden state and the word
// scores) on the B200 engine, header-only over imi_cuda.h.
//
// imi_brain steps the same Seoul / LFM3 backbone as imi_seoul, built as a ggml graph per step (brain.cpp:149-278);
// here it is the engine's step, so a caller of imi_brain switches by including this header instead of brain.h and
// linking libimi_cuda.so. Members kept: the model file `f` (imi_file_cuda.h), the shape (n_embd, n_vocab, n_head,
// n_head_kv, head_dim, d_conv, n_swa, n_ctx, eps, rope bases), pos, n_threads, hidden, logits. The ggml graph, its
// tensors and the stacked-table bookkeeping of brain.h have no counterpart (the engine owns its layout on the device).
// Errors as imi: load returns false with a message; a step past n_ctx prints "context full" and does nothing.
#pragma once
#include "imi_seoul_cuda.h"

struct imi_brain {
private:
    imi_seoul s;   // first: the public references below point into it

public:
    imi_file &f;
    int n_embd = 0, n_vocab = 0, n_head = 0, n_head_kv = 0, head_dim = 0, d_conv = 0, n_swa = 0, n_ctx = 0;
    float eps = 1e-5f, rope_base = 1e6f, rope_base_swa = 1e4f;
    int pos = 0, n_threads = 4;
    std::vector<float> &hidden, &logits;   // valid until the next step, as imi's

    imi_brain() : f(s.f), hidden(s.hidden), logits(s.logits) {}
    imi_brain(const imi_brain &) = delete;
    imi_brain &operator=(const imi_brain &) = delete;

    // brain.h:60 load(path, threads, ctx_len)
    bool load(const std::string &path, int threads, int ctx_len) {
        if (!s.load(path, threads, ctx_len)) return false;
        n_embd = s.n_embd; n_vocab = s.n_vocab; n_head = s.n_head; n_head_kv = s.n_head_kv; head_dim = s.head_dim;
        d_conv = s.d_conv; n_swa = s.n_swa; n_ctx = s.n_ctx; eps = s.eps; rope_base = s.rope_base;
        rope_base_swa = s.rope_base_swa; n_threads = threads;
        pos = 0;
        return true;
    }
    void reset() {   // brain.h:61
        s.reset();
        pos = 0;
    }
    // brain.h:62-63: a word (token >= 0) or a ready input vector (embd); want_logits = score words
    void step(int32_t token, const float *embd, bool want_logits) {
        s.step(token, embd, want_logits);
        pos = s.pos;
    }
};

// imi_seoul_cuda.h - imi's brain interface (imi/core/seoul.h:21-72) on the B200 engine, header-only over imi_cuda.h.
//
// A caller of imi_seoul switches by including this header instead of core/seoul.h and linking libimi_cuda.so:
// the same members (n_embd, n_vocab, n_ctx, pos, hidden, logits), the same calls (load, reset, step, step_batch,
// new_state, swap_state, step2, bench_tables) with the same meaning and error behaviour (load returns false with a
// message on stderr; a step past n_ctx prints "context full" and does nothing, seoul.cpp:209,353,498).
// Differences, all deliberate: the thread count and shared team arguments are accepted and ignored (the GPU needs
// no thread team); the device is chosen by IMI_CUDA_DEVICE (default 0); hidden / logits are copied back after each
// step (logits only when asked for), so they stay valid until the next step as in imi. The model file `f` is the
// library's own GGUF reader (imi_file_cuda.h: the same calls as imi/model.h). The research timers (seoul.h:54): a step
// is one CUDA graph on the device, so t_tables receives each step's whole device time in ms (table reads, attention and
// the small math together) and t_sync, t_attn stay 0 (no barrier waits; attention is not timed apart).
#pragma once
#include "imi_cuda.h"
#include "imi_file_cuda.h"

#include <cstdio>
#include <cstdlib>
#include <string>
#include <utility>
#include <vector>

struct imi_seoul_state {
    imi_cuda_state *s = nullptr;
    int pos = 0;
    std::vector<float> hidden, logits;
    imi_seoul_state() = default;
    imi_seoul_state(const imi_seoul_state &) = delete;
    imi_seoul_state &operator=(const imi_seoul_state &) = delete;
    imi_seoul_state(imi_seoul_state &&o) noexcept { *this = std::move(o); }
    imi_seoul_state &operator=(imi_seoul_state &&o) noexcept {
        std::swap(s, o.s);
        std::swap(pos, o.pos);
        hidden.swap(o.hidden);
        logits.swap(o.logits);
        return *this;
    }
    ~imi_seoul_state() { imi_cuda_state_free(s); }
};

struct imi_seoul {
    imi_file f;
    int n_embd = 0, n_vocab = 0, n_head = 0, n_head_kv = 0, head_dim = 0, n_ff = 0, d_conv = 0, n_swa = 0, n_ctx = 0;
    float eps = 1e-5f, rope_base = 1e6f, rope_base_swa = 1e4f;
    int pos = 0, n_threads = 1;
    std::vector<float> hidden, logits;
    double t_tables = 0, t_sync = 0, t_attn = 0;   // ms (see above)
    imi_cuda_engine *engine = nullptr;

    // seoul.cpp:93 load(path, threads, ctx_len, shared team): the last two steps of state fit on the device
    bool load(const std::string &path, int threads, int ctx_len, void *shared = nullptr) {
        (void) shared;
        n_threads = threads;
        if (!f.load(path)) return false;
        eps = f.key_f("lfm3.attention.layer_norm_rms_epsilon", 1e-5f);   // seoul.cpp:101-104
        rope_base = f.key_f("lfm3.rope.freq_base", 1e6f);
        rope_base_swa = f.key_f("lfm3.rope.freq_base_swa", 1e4f);
        const char *dev = getenv("IMI_CUDA_DEVICE");
        if (imi_cuda_load(path.c_str(), dev ? atoi(dev) : 0, ctx_len, 8, &engine) != IMI_OK) {
            fprintf(stderr, "imi-seoul: %s\n", imi_cuda_error());
            return false;
        }
        imi_cuda_info info;
        imi_cuda_get_info(engine, &info);
        n_embd = info.n_embd; n_vocab = info.n_vocab; n_head = info.n_head; n_head_kv = info.n_head_kv;
        head_dim = info.head_dim; n_ff = info.n_ff; d_conv = info.d_conv; n_swa = info.n_swa; n_ctx = info.n_ctx;
        if (imi_cuda_state_new(engine, &own.s) != IMI_OK) {
            fprintf(stderr, "imi-seoul: %s\n", imi_cuda_error());
            return false;
        }
        hidden.assign(n_embd, 0.0f);
        logits.assign(n_vocab, 0.0f);
        return true;
    }
    void reset() {   // seoul.cpp:188-191
        imi_cuda_state_reset(own.s);
        pos = 0;
    }
    void step(int32_t token, const float *embd, bool want_logits) {   // seoul.cpp:352-357
        if (!ok(imi_cuda_step(own.s, token, embd, want_logits))) return;
        pos = imi_cuda_state_pos(own.s);
        t_tables += imi_cuda_last_step_ms(engine);
        fetch(own.s, hidden, want_logits ? &logits : nullptr);
    }
    void step_batch(const int32_t *tokens, const float *embd, int n, bool want_logits, float *hidden_all = nullptr) {
        const imi_cuda_status st = imi_cuda_step_batch(own.s, tokens, embd, n, want_logits, hidden_all);
        pos = imi_cuda_state_pos(own.s);
        if (!ok(st)) return;
        fetch(own.s, hidden, want_logits ? &logits : nullptr);
    }
    imi_seoul_state new_state() const {   // seoul.cpp:193-201
        imi_seoul_state s;
        imi_cuda_state_new(engine, &s.s);
        s.hidden.assign(n_embd, 0.0f);
        s.logits.assign(n_vocab, 0.0f);
        return s;
    }
    void swap_state(imi_seoul_state &s) {   // seoul.cpp:203-206: no copying
        std::swap(own.s, s.s);
        std::swap(pos, s.pos);
        hidden.swap(s.hidden);
        logits.swap(s.logits);
    }
    // seoul.cpp:208-220: two conversations one position each, every table read once for both
    void step2(int32_t token_a, const float *embd_a, bool logits_a, imi_seoul_state &b, int32_t token_b,
               const float *embd_b, bool logits_b) {
        if (!ok(imi_cuda_step2(own.s, token_a, embd_a, logits_a, b.s, token_b, embd_b, logits_b))) return;
        pos = imi_cuda_state_pos(own.s);
        t_tables += imi_cuda_last_step_ms(engine);
        b.pos = imi_cuda_state_pos(b.s);
        fetch(own.s, hidden, logits_a ? &logits : nullptr);
        fetch(b.s, b.hidden, logits_b ? &b.logits : nullptr);
    }
    double bench_tables(int ncol, int reps) {   // seoul.cpp:657-685 (mean, not best, of reps)
        float ms = 0;
        size_t bytes = 0;
        return imi_cuda_bench_tables(engine, ncol, reps, &ms, &bytes) == IMI_OK ? ms : -1.0;
    }
    ~imi_seoul() {
        imi_cuda_state_free(own.s);
        own.s = nullptr;
        imi_cuda_free(engine);
    }

private:
    imi_seoul_state own;
    bool ok(imi_cuda_status st) const {
        if (st == IMI_OK) return true;
        if (st == IMI_E_CTX_FULL) fprintf(stderr, "imi-seoul: context full (%d)\n", n_ctx);
        else fprintf(stderr, "imi-seoul: %s\n", imi_cuda_error());
        return false;
    }
    static void fetch(imi_cuda_state *s, std::vector<float> &h, std::vector<float> *l) {
        imi_cuda_get_hidden(s, h.data());
        if (l) imi_cuda_get_logits(s, l->data());
    }
};

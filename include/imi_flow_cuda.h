// imi_flow_cuda.h - the riding caller of imi's live pipelines on the B200 engine, header-only over imi_cuda.h.
//
// imi/core/flow.cpp:114-126 (the same step order as imi/app/live.cpp:412-415 and imi/core/instant.cpp:448-452):
// a voice conversation steps one frame at a time (the talker's feedback vector in, hidden state out, no word
// scores: talk.h:32-34), a text conversation steps greedy words (word in, word scores, first-maximum pick:
// flow.cpp:57-62). While both have work, each text word rides on a frame's step (imi_cuda_step2: every table read
// once for both); otherwise each steps alone. Every conversation gets exactly the numbers its own steps would give,
// so the outputs do not depend on `ride`; only the time does.
//
// What the reference keeps in its own objects is a callback here: the talker (`voice`: the next frame from the
// voice conversation's hidden state, imi_talker::next, talk.h:56-58) and the end of a text part (`on_end`: flow.cpp
// 63-73 re-prompts the text conversation for its translation). The text pick is read on the device
// (imi_cuda_get_argmax: 8 bytes back, not the word scores) and the voice's hidden state is read back after each
// of its steps (n_embd floats), which is all the talker consumes.
#pragma once
#include "imi_cuda.h"

#include <cstddef>
#include <cstdint>
#include <functional>
#include <vector>

// the brain side of flow.cpp's text_job (flow.cpp:26-33)
struct imi_flow_text {
    imi_cuda_state *s = nullptr;   // the text conversation (prompt already read, with word scores)
    int32_t pending = -1;          // the next word to step; -1: nothing to step
    int32_t stop = -1;             // the end word (words.im_end, flow.cpp:62)
    size_t cap = 512;              // most words of this part (flow.cpp:61: 512 hearing, 600 translating)
    std::vector<int32_t> got;      // the words picked in this part
};

struct imi_flow_counts {           // flow.cpp:53: shared steps, text steps alone, voice steps alone
    int ride = 0, text_alone = 0, voice_alone = 0;
};

// after a step of the text conversation (or its prompt): the next word, or the end of this part (flow.cpp:57-76).
// on_end(t) may start the next part (reset, read a new prompt, clear got, set cap) and return true to pick again.
inline imi_cuda_status imi_flow_pick(imi_flow_text &t, const std::function<bool(imi_flow_text &)> &on_end) {
    for (;;) {
        int32_t best = 0;
        float v = 0.0f;
        const imi_cuda_status st = imi_cuda_get_argmax(t.s, &best, &v);
        if (st != IMI_OK) return st;
        if (best != t.stop && t.got.size() < t.cap) {
            t.got.push_back(best);
            t.pending = best;
            return IMI_OK;
        }
        t.pending = -1;
        if (!on_end || !on_end(t)) return IMI_OK;
    }
}

// one voice utterance beside the text conversation, to the end of both (flow.cpp:114-126). voice_s: the voice
// conversation (its prompt already read); voice(hidden, fb): the next frame's feedback vector fb[n_embd] from the
// voice's hidden state, false when speech is over. hidden[n_embd] is the caller's buffer, holding the voice's hidden
// state on entry (after its prompt) and after every voice step. text may be null or hold no pending word.
inline imi_cuda_status imi_flow_run(imi_cuda_state *voice_s, float *hidden, int n_embd,
                                    const std::function<bool(const float *hidden, float *fb)> &voice, imi_flow_text *text,
                                    const std::function<bool(imi_flow_text &)> &on_end, bool ride,
                                    imi_flow_counts *counts) {
    std::vector<float> fb((size_t) n_embd);
    imi_flow_counts n;
    imi_cuda_status st = IMI_OK;
    bool speaking = true;
    auto text_step = [&]() -> imi_cuda_status {
        const imi_cuda_status r = imi_cuda_step(text->s, text->pending, nullptr, 1);
        if (r != IMI_OK) return r;
        n.text_alone++;
        return imi_flow_pick(*text, on_end);
    };
    while (st == IMI_OK && (speaking || (text && text->pending >= 0))) {
        if (speaking) speaking = voice(hidden, fb.data());
        const bool has_text = text && text->pending >= 0;
        if (speaking && has_text && ride) {
            st = imi_cuda_step2(voice_s, -1, fb.data(), 0, text->s, text->pending, nullptr, 1);
            if (st == IMI_OK) st = imi_cuda_get_hidden(voice_s, hidden);
            if (st == IMI_OK) {
                n.ride++;
                st = imi_flow_pick(*text, on_end);
            }
            continue;
        }
        if (speaking) {
            st = imi_cuda_step(voice_s, -1, fb.data(), 0);
            if (st == IMI_OK) st = imi_cuda_get_hidden(voice_s, hidden);
            if (st == IMI_OK) n.voice_alone++;
        }
        if (st == IMI_OK && has_text) st = text_step();
    }
    if (counts) *counts = n;
    return st;
}

// flow_check: the riding caller (include/imi_flow_cuda.h) on one GPU, run twice on the same inputs, once with every
// text word riding a voice frame's step and once with every step alone (flow.cpp's RIDE 1 / 0), after one untimed
// run. Prints one JSON line: both runs' text picks, a hash of every hidden state the voice callback saw, the step
// counts and the host time of each run; exit 0 when the two runs agree bit for bit, 1 when they differ, 2 on an
// engine error.
//   flow_check MODEL.gguf FRAMES CAP1 CAP2 SEED
// Voice stand-in: the next frame is fb[i] = 0.5 h[i] / (1 + |h[i]|) + 0.01 (k mod 7) from the voice's hidden state
// h after frame k (any function of h will do: the talker's only input from the brain is that hidden state).
// Text: a prompt of 16 ids, CAP1 greedy words, then a re-prompt of 10 ids (reset first, as flow.cpp:66-67) and CAP2
// greedy words. Ids come from a 64-bit LCG of SEED so that a checker can replay them.
#include "imi_flow_cuda.h"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

static uint64_t lcg = 1;
static int32_t next_id(int n_vocab) {
    lcg = lcg * 6364136223846793005ULL + 1442695040888963407ULL;
    return (int32_t) ((lcg >> 33) % (uint64_t) n_vocab);
}

struct run_out {
    std::vector<int32_t> picks;
    uint64_t hash = 1469598103934665603ULL;
    imi_flow_counts n;
    double ms = 0;
};

static int fail(const char *what) {
    fprintf(stderr, "flow_check: %s: %s\n", what, imi_cuda_error());
    return 2;
}

int main(int argc, char **argv) {
    if (argc < 6) { fprintf(stderr, "usage: flow_check MODEL.gguf FRAMES CAP1 CAP2 SEED\n"); return 2; }
    const int frames = atoi(argv[2]), cap1 = atoi(argv[3]), cap2 = atoi(argv[4]);
    const uint64_t seed = strtoull(argv[5], nullptr, 10);
    imi_cuda_engine *e = nullptr;
    if (imi_cuda_load(argv[1], 0, 2048, 2, &e) != IMI_OK) return fail("load");
    imi_cuda_info info;
    imi_cuda_get_info(e, &info);
    const int E = info.n_embd, V = info.n_vocab;
    lcg = seed;
    std::vector<int32_t> voice_prompt(12), text_prompt(16), re_prompt(10);
    for (auto &t : voice_prompt) t = next_id(V);
    for (auto &t : text_prompt) t = next_id(V);
    for (auto &t : re_prompt) t = next_id(V);
    imi_cuda_state *vs = nullptr, *ts = nullptr;
    if (imi_cuda_state_new(e, &vs) != IMI_OK || imi_cuda_state_new(e, &ts) != IMI_OK) return fail("state_new");

    auto one = [&](bool ride, run_out &o) -> int {
        std::vector<float> h((size_t) E);
        if (imi_cuda_state_reset(vs) != IMI_OK || imi_cuda_state_reset(ts) != IMI_OK) return fail("reset");
        const auto t0 = std::chrono::steady_clock::now();
        if (imi_cuda_step_batch(vs, voice_prompt.data(), nullptr, (int) voice_prompt.size(), 0, nullptr) != IMI_OK ||
            imi_cuda_get_hidden(vs, h.data()) != IMI_OK)
            return fail("voice prompt");
        if (imi_cuda_step_batch(ts, text_prompt.data(), nullptr, (int) text_prompt.size(), 1, nullptr) != IMI_OK)
            return fail("text prompt");
        imi_flow_text t;
        t.s = ts;
        t.cap = (size_t) cap1;
        int part = 1;
        auto on_end = [&](imi_flow_text &x) -> bool {
            o.picks.insert(o.picks.end(), x.got.begin(), x.got.end());
            x.got.clear();
            if (part != 1) return false;
            part = 2;
            x.cap = (size_t) cap2;
            return imi_cuda_state_reset(x.s) == IMI_OK &&
                   imi_cuda_step_batch(x.s, re_prompt.data(), nullptr, (int) re_prompt.size(), 1, nullptr) == IMI_OK;
        };
        if (imi_flow_pick(t, on_end) != IMI_OK) return fail("first pick");
        int k = 0;
        auto voice = [&](const float *hid, float *fb) -> bool {
            const unsigned char *b = (const unsigned char *) hid;
            for (size_t i = 0; i < (size_t) E * 4; i++) o.hash = (o.hash ^ b[i]) * 1099511628211ULL;
            if (k >= frames) return false;
            for (int i = 0; i < E; i++) fb[i] = 0.5f * hid[i] / (1.0f + std::fabs(hid[i])) + 0.01f * (float) (k % 7);
            k++;
            return true;
        };
        if (imi_flow_run(vs, h.data(), E, voice, &t, on_end, ride, &o.n) != IMI_OK) return fail("flow");
        o.ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        return 0;
    };
    run_out warm, alone, rode;
    int r = one(true, warm);
    if (!r) r = one(false, alone);
    if (!r) r = one(true, rode);
    if (r) return r;
    const bool same = alone.picks == rode.picks && alone.hash == rode.hash && warm.picks == rode.picks &&
                      warm.hash == rode.hash;
    std::string picks;
    for (size_t i = 0; i < rode.picks.size(); i++) picks += (i ? "," : "") + std::to_string(rode.picks[i]);
    std::string ids;
    for (auto *v : { &voice_prompt, &text_prompt, &re_prompt }) {
        ids += ids.empty() ? "[" : ",[";
        for (size_t i = 0; i < v->size(); i++) ids += (i ? "," : "") + std::to_string((*v)[i]);
        ids += "]";
    }
    printf("{\"same\": %s, \"frames\": %d, \"picks\": [%s], \"prompts\": [%s], \"hash\": \"%016llx\", "
           "\"ride\": {\"ms\": %.3f, \"shared\": %d, \"text_alone\": %d, \"voice_alone\": %d}, "
           "\"alone\": {\"ms\": %.3f, \"shared\": %d, \"text_alone\": %d, \"voice_alone\": %d}}\n",
           same ? "true" : "false", frames, picks.c_str(), ids.c_str(), (unsigned long long) rode.hash, rode.ms,
           rode.n.ride, rode.n.text_alone, rode.n.voice_alone, alone.ms, alone.n.ride, alone.n.text_alone,
           alone.n.voice_alone);
    imi_cuda_state_free(vs);
    imi_cuda_state_free(ts);
    imi_cuda_free(e);
    return same ? 0 : 1;
}

// flow_fake: the riding caller (include/imi_flow_cuda.h) against a fake of the C-ABI calls it makes, on the CPU.
// The fake keeps per conversation a position and a hidden value and "picks" a word from them, and logs every call,
// so the test can check the caller's step order (flow.cpp:114-126) without a GPU.
//   flow_fake RIDE FRAMES CAP1 CAP2 STOP_AT
// STOP_AT >= 0: the fake picks the stop word at that text position. Prints the call log, one call per line, then
// "picks ..." and "counts ride text_alone voice_alone".
#include "imi_flow_cuda.h"

#include <cstdio>
#include <cstdlib>
#include <string>

struct imi_cuda_state {
    int pos = 0;
    float h = 0.0f;
    const char *name = "";
};
static int stop_at = -1;
static const int32_t STOP = 999;

static void advance(imi_cuda_state *s, int32_t token, const float *embd) {
    s->h = token >= 0 ? (float) token : embd[0];
    s->pos++;
}
extern "C" {
imi_cuda_status imi_cuda_step(imi_cuda_state *s, int32_t token, const float *embd, int want_logits) {
    printf("step %s %d %s\n", s->name, token, want_logits ? "logits" : "hidden");
    advance(s, token, embd);
    return IMI_OK;
}
imi_cuda_status imi_cuda_step2(imi_cuda_state *a, int32_t token_a, const float *embd_a, int logits_a, imi_cuda_state *b,
                               int32_t token_b, const float *embd_b, int logits_b) {
    printf("step2 %s %d %s + %s %d %s\n", a->name, token_a, logits_a ? "logits" : "hidden", b->name, token_b,
           logits_b ? "logits" : "hidden");
    advance(a, token_a, embd_a);
    advance(b, token_b, embd_b);
    return IMI_OK;
}
imi_cuda_status imi_cuda_get_argmax(const imi_cuda_state *s, int32_t *id, float *value) {
    *id = s->pos == stop_at ? STOP : 100 + s->pos;
    *value = 0.0f;
    return IMI_OK;
}
imi_cuda_status imi_cuda_get_hidden(const imi_cuda_state *s, float *out) {
    out[0] = s->h;
    out[1] = (float) s->pos;
    return IMI_OK;
}
}

int main(int argc, char **argv) {
    if (argc < 6) return 2;
    const bool ride = atoi(argv[1]) != 0;
    const int frames = atoi(argv[2]), cap1 = atoi(argv[3]), cap2 = atoi(argv[4]);
    stop_at = atoi(argv[5]);
    imi_cuda_state voice, text;
    voice.name = "voice";
    text.name = "text";
    text.pos = 10;   // its prompt
    imi_flow_text t;
    t.s = &text;
    t.stop = STOP;
    t.cap = (size_t) cap1;
    std::vector<int32_t> picks;
    int part = 1;
    auto on_end = [&](imi_flow_text &x) -> bool {
        picks.insert(picks.end(), x.got.begin(), x.got.end());
        x.got.clear();
        printf("end of part %d\n", part);
        if (part++ != 1) return false;
        x.cap = (size_t) cap2;
        x.s->pos = 20;   // the re-prompt
        return true;
    };
    if (imi_flow_pick(t, on_end) != IMI_OK) return 1;
    int k = 0;
    auto next = [&](const float *hid, float *fb) -> bool {
        if (k >= frames) return false;
        fb[0] = hid[1] + 0.5f;   // the frame depends on the voice's latest state
        k++;
        return true;
    };
    float hidden[2] = { 0.0f, 0.0f };
    imi_flow_counts n;
    if (imi_flow_run(&voice, hidden, 2, next, &t, on_end, ride, &n) != IMI_OK) return 1;
    printf("picks");
    for (int32_t p : picks) printf(" %d", p);
    printf("\ncounts %d %d %d\n", n.ride, n.text_alone, n.voice_alone);
    return 0;
}

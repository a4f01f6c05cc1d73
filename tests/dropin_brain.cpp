// imi_brain (imi/brain.h:33-64) on the engine through the drop-in headers: load a model, step the given tokens with
// word scores, write every position's hidden state and scores (imi's answer-key layout: int32 n_embd, n_vocab, n;
// per position int32 token, f32 hidden, f32 logits), and read a few keys of the model file through brain.f.
//   dropin_brain MODEL.gguf OUT.bin TOKEN...
#include "brain.h"

#include <cstdio>
#include <cstdlib>
#include <vector>

int main(int argc, char **argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: dropin_brain MODEL.gguf OUT.bin TOKEN...\n");
        return 1;
    }
    imi_brain br;
    if (!br.load(argv[1], 4, 256)) return 1;
    // the model file beside the brain: keys by imi_file and by the gguf accessors the tokenizer uses
    const int64_t blocks = br.f.key_i("lfm3.block_count", -1);
    const int64_t k = gguf_find_key(br.f.meta, "lfm3.attention.sliding_window_pattern");
    const size_t n_pat = k >= 0 ? gguf_get_arr_n(br.f.meta, k) : 0;
    ggml_tensor *te = br.f.get("token_embd.weight");
    printf("{\"blocks\": %lld, \"pattern\": %zu, \"embd_rows\": %lld, \"n_embd\": %d}\n", (long long) blocks, n_pat,
           (long long) te->ne[1], br.n_embd);
    FILE *out = fopen(argv[2], "wb");
    if (!out) return 1;
    const int32_t ne = br.n_embd, nv = br.n_vocab, n = argc - 3;
    fwrite(&ne, 4, 1, out);
    fwrite(&nv, 4, 1, out);
    fwrite(&n, 4, 1, out);
    for (int i = 0; i < n; i++) {
        const int32_t t = atoi(argv[3 + i]);
        br.step(t, nullptr, true);
        fwrite(&t, 4, 1, out);
        fwrite(br.hidden.data(), 4, ne, out);
        fwrite(br.logits.data(), 4, nv, out);
    }
    fclose(out);
    return br.pos == n ? 0 : 1;
}

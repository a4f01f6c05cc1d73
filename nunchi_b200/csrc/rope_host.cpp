// The rotary angles' cosines and sines for every position, computed on the host with the C library's cosf/sinf
// exactly as imi computes them inside each step (imi/core/seoul.cpp:19-28): scale = base^(-2/n), th starts at pos and
// is multiplied by scale once per pair, angle = th / freq_factor[i]. Built once at load; the attention kernels read
// one row per position. Compiled with -ffp-contract=off so every operation rounds as written.
#include <cmath>
#include <cstddef>

namespace imi {
void rope_table(int n_ctx, int n, float base, const float *ff, float *cs, float *sn) {
    const float scale = powf(base, -2.0f / (float) n);
    for (int pos = 0; pos < n_ctx; pos++) {
        float th = (float) pos;
        float *c = cs + (size_t) pos * (n / 2), *s = sn + (size_t) pos * (n / 2);
        for (int i = 0; i < n / 2; i++) {
            const float a = th / (ff ? ff[i] : 1.0f);
            c[i] = cosf(a);
            s[i] = sinf(a);
            th *= scale;
        }
    }
}
}  // namespace imi

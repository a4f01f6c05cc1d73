// A Q4_0 tied word table for the reference's brain (TEST INFRASTRUCTURE ONLY).
//
// imi_seoul accepts only a Q6_K word table (imi/core/seoul.cpp:95-96); the benchmark configuration's tied
// embedding / LM head is Q4_0. seoul.cpp is compiled unmodified with its three word-table hooks renamed on the
// command line (imi_q6k_dequant_row, imi_q6k_row, imi_q8k) to the functions below, which give the Q4_0 table
// imi's own 4-bit semantics:
//  * lookup: value = d * (code - 8), code i of a block from the low nibble of byte i, code 16+i from the high one;
//  * scores: the input cut to 8-bit per 32 values with imi_cut32 (imi/core/vec.h:47-77, as imi_q8::from,
//    tables.cpp:100-109), then per row the exact accumulation of imi's 4-bit kernel group_avx2<false>
//    (tables.cpp:127-143): acc = fma(float(block dot), d * dx, acc); cor = fma(d, dx * sum(q), cor); out = acc - 8 cor
//    (one rounding, _mm256_fnmadd_ps), blocks in order.
#include "tables.h"
#include "vec.h"

#include <cmath>
#include <cstring>

void oref_q8_head::from(const float *x, int nn) {
    n = nn;
    const int nb = n / 32;
    q.resize(n); d.resize(nb); bsums.resize(nb);
    for (int j = 0; j < nb; j++) {
        int sum;
        d[j] = imi_cut32(x + 32 * j, &q[32 * j], &sum);
        bsums[j] = (int16_t) sum;   // |sum| <= 32 * 127 fits
    }
}

float oref_q4_0_head_row(const void *row, const oref_q8_head &X, int nblocks256) {
    const uint8_t *b = (const uint8_t *) row;
    const int nb = nblocks256 * 8;
    float acc = 0.0f, cor = 0.0f;
    for (int j = 0; j < nb; j++, b += 18) {
        uint16_t dh; memcpy(&dh, b, 2);
        const uint8_t *qs = b + 2;
        const int8_t *xq = X.q.data() + 32 * j;
        int s = 0;
        for (int i = 0; i < 16; i++) s += (qs[i] & 15) * xq[i] + (qs[i] >> 4) * xq[16 + i];
        const float dd = imi_h2f(dh);
        acc = fmaf((float) s, dd * X.d[j], acc);
        cor = fmaf(dd, X.d[j] * (float) X.bsums[j], cor);
    }
    return fmaf(-8.0f, cor, acc);
}

void oref_q4_0_lookup_row(const void *row, float *y, int nblocks256) {
    const uint8_t *b = (const uint8_t *) row;
    for (int j = 0; j < nblocks256 * 8; j++, b += 18) {
        uint16_t dh; memcpy(&dh, b, 2);
        const float dd = imi_h2f(dh);
        for (int i = 0; i < 16; i++) {
            y[32 * j + i] = dd * (float) ((b[2 + i] & 15) - 8);
            y[32 * j + 16 + i] = dd * (float) ((b[2 + i] >> 4) - 8);
        }
    }
}

// Known-answer access to the reference's own Q6_K word-table functions (TEST INFRASTRUCTURE ONLY):
// imi_q8k::from, imi_q6k_row and imi_q6k_dequant_row of imi/core/tables.cpp:200-287, compiled unmodified in
// tables.o. This file is built without the Q4_0 word-table renames, so the names below reach the real functions.
#include "tables.h"

#include <cstring>

extern "C" {

void oref_q8k_from(const float *x, int n, int8_t *q, float *d, int16_t *bsums) {
    imi_q8k X;
    X.from(x, n);
    memcpy(q, X.q.data(), (size_t) n);
    memcpy(d, X.d.data(), sizeof(float) * (size_t) (n / 256));
    memcpy(bsums, X.bsums.data(), sizeof(int16_t) * (size_t) (n / 16));
}

float oref_q6k_row(const void *row, const float *x, int nblocks) {
    imi_q8k X;
    X.from(x, 256 * nblocks);
    return imi_q6k_row(row, X, nblocks);
}

void oref_q6k_dequant_row(const void *row, float *y, int nblocks) { imi_q6k_dequant_row(row, y, nblocks); }

}  // extern "C"

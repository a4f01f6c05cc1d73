// Host entry points of the kernels (kernels.cu).
#pragma once
#include "common.cuh"
#include "tc_prep.cuh"
#include "tc_table.cuh"

namespace imi {
// one table read; `pro` / `epi` pick the input preparation and the output stage (common.cuh: Pro, Epi)
cudaError_t launch_table(int pro, int epi, const MvArgs &a, int grid, cudaStream_t st, bool pdl);
size_t table_smem(int pro, int cols, int sr, int ncol, int n_embd, int ab_len, int d_conv, int nstage, int has_m = 0);
int table_nc_slot(int ncol);
cudaError_t launch_attn(const AttnArgs &a, cudaStream_t st, bool pdl);
bool attn_supported(int head_dim, int grp, int n_ctx);
// the same attention for many columns, one CTA per (kv head, column) for the query heads sharing it (GQA)
cudaError_t launch_attn_grp(const AttnArgs &a, cudaStream_t st, bool pdl);
bool attn_grp_supported(int head_dim, int grp, int n_ctx);
cudaError_t launch_kvwrite(const AttnArgs &a, cudaStream_t st, bool pdl);
cudaError_t launch_final(const FinalArgs &a, cudaStream_t st, bool pdl);
cudaError_t prepare_kernels();
cudaError_t launch_q8_cut(const float *x, int n, int8_t *q, float *d, float *s, cudaStream_t st);
// the Q6_K word table: the 256-value input cut (imi_q8k::from) and the word scores (imi_q6k_row), n and cols
// multiples of 256
cudaError_t launch_q8k_cut(const float *x, int n, int8_t *q, float *d, int16_t *bsums, cudaStream_t st);
cudaError_t launch_q6k_scores(const uint8_t *W, int rows, int nb, const int8_t *xq, const float *xd,
                              const int16_t *bsums, float *out, cudaStream_t st);
// the Q6_K word table inside a step: word scores for ncol inputs, the greedy pick and the end of the step
cudaError_t launch_q6k_head(const Q6HeadArgs &a, cudaStream_t st, bool pdl);
int q6k_head_ctas(int rows, int nb, int nc);   // its grid (0: rows too wide)
// a table's tiled copy for the tensor-core read (tc_table.cuh: k_tc_tile), tc_tiled_bytes(rows, cols) at dst
cudaError_t launch_tc_tile(const uint8_t *W, int rows, int cols, int row_bytes, uint8_t *dst, cudaStream_t st);
// the tensor-core batched table read (tc_table.cuh); a.G in {16, 32, 64}
cudaError_t launch_tc_table(const TcArgs &a, int grid, cudaStream_t st, bool pdl);
// the conversation records of a step's n columns into 32-byte slots of dst (device)
cudaError_t launch_gather_sess(const Col *cols, int n, uint8_t *dst, cudaStream_t st);
// the batched read's input preparation: one CTA per column
cudaError_t launch_tc_prep(const TcPrepArgs &a, cudaStream_t st, bool pdl);
// one CTA waiting on an mbarrier nothing completes, for at most `limit` clock cycles (the bounded waits' failure path)
cudaError_t launch_wait_check(long long limit, int *err, cudaStream_t st);
// GGUF Q4_0 rows (device) into the table kernel's row layout (device), on stream st
cudaError_t launch_q4_repack(const uint8_t *src, int rows, int nb, uint8_t *dst, cudaStream_t st);
}  // namespace imi

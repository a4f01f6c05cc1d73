// k_tc_prep: the small math imi's threads repeat before every table read (norms, residual adds, the short conv, the
// 8-bit cut; seoul.cpp:402-474 and run_batch 562-623), for the tensor-core batched read: one CTA per column (a
// conversation of a multi-session step or a position of a prefill chunk), imi's float order exactly as the
// small-batch table kernel's input preparation (table.cuh: table_prologue), the cut codes written straight into the
// batched read's column operand with the blocks' scales and scale * code sums (tc_table.cuh: tc_xb_code,
// tc_xb_scale). The small-batch kernel prepares every column in every CTA (a few columns); with dozens of
// columns that work would be repeated on every SM, so here it is done once, spread over the columns.
#pragma once
#include "common.cuh"
#include "tc_table.cuh"

namespace imi {

enum TcPro : int {
    TP_EMBED_NORM = 0,   // x = word row | input vector | the last pick's word row; x -> xout; h = norm(x) * wpre
    TP_RESID_NORM = 1,   // x = xin + norm(in) * wpost -> xout; h = norm(x) * wpre
    TP_CONV = 2,         // u = c * (b*x*w_last + sum_k st_k * w_k), st from this chunk's columns or the conv memory
    TP_CUT = 3,          // the input as it is (SiLU output)
    TP_Q8 = 4,           // 8-bit codes, scales and sums made by the producer (attention output): repacked only
    TP_FINAL = 5         // x = xin + norm(in) * wpost; hidden = norm(x) * wpre (out_norm) -> hid_out
};
constexpr int TP_THREADS = 256;
constexpr int TP_PQ = 4;   // float4 chunks of an n_embd vector per thread at most (n_embd <= 4 * 4 * TP_THREADS)

struct TcPrepArgs {
    const Col *cols_d;
    int ncol, pro;
    int K;                 // length of the prepared vector (the next table's width)
    int G;                 // columns per group of the batched read's operand
    uint8_t *xb;           // operand out: [group][K / TC_KS][tc_xb_bytes(G)] (8-bit codes, scales, scale * code sums)
    const float *in;       // per column: the previous table's output (RESID, FINAL), SiLU output (CUT), b|c|x (CONV)
    int in_stride;
    const float *xin;      // residual stream in / out, per column
    float *xout;
    int x_stride;
    const float *wpost, *wpre;
    float eps;
    const uint8_t *emb;    // word table (EMBED: lookup)
    int emb_row_bytes, emb_q6k;
    const float *conv_w;   // [d_conv + 1][n_embd]
    int d_conv, conv_layer, n_embd;
    int ring_conv;         // TP_CONV: 1 writes this conv layer's memory slot of each column's position (decode)
    int ring_layer;        // TP_RESID_NORM: >= 0 writes that conv layer's memory slots from ring_src (prefill chunk)
    const float *ring_src;
    int ring_src_stride;
    const int8_t *q8_q;    // TP_Q8: [c][K] codes, [c][K/32] scales and sums
    const float *q8_d, *q8_s;
};

#if defined(__CUDACC__) && defined(IMI_KERNELS)   // device code: compiled in kernels.cu only
// the 4 codes of values 4q..4q+3 of column c (packed as cut32_g8 returns them: value 4q + u in byte u) into the
// operand; the block's scale and scale * code sum by lane 8m of the block's group
__device__ __forceinline__ void tp_put(const TcPrepArgs &a, int c, int q, uint32_t w, float d, int sum, bool act) {
    const int G = a.G, g = c / G, cg = c - g * G, K = a.K;
    if (!act) return;
    *(uint32_t *) (a.xb + tc_xb_code(G, K, g, cg, 4 * q)) = w;
    if ((q & 7) == 0) {
        *(float *) (a.xb + tc_xb_scale(G, K, g, cg, q >> 3, 0)) = d;
        *(float *) (a.xb + tc_xb_scale(G, K, g, cg, q >> 3, 1)) = __fmul_rn(d, (float) sum);
    }
}
// cut the float4 chunk q of a K-long vector (8 lanes per 32-value block) and store it; every lane of the warp calls it
__device__ __forceinline__ void tp_cut(const TcPrepArgs &a, int c, int q, float4 v, bool act) {
    float d;
    int sum;
    const uint32_t w = cut32_g8(act ? v : make_float4(0.0f, 0.0f, 0.0f, 0.0f), d, sum);
    tp_put(a, c, q, w, d, sum, act);
}

__global__ void __launch_bounds__(TP_THREADS) k_tc_prep(const __grid_constant__ TcPrepArgs a) {
    extern __shared__ __align__(16) uint8_t smp[];
    float *v = (float *) smp;                  // the vector being normed (n_embd) or cut (K)
    __shared__ float red[2];
    const int c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5;
    const int E = a.n_embd, K = a.K, pro = a.pro;
    pdl_trigger();
    // before the wait (none of it is written by the launches in flight): the column's record and, for the norms,
    // this thread's chunks of both norm weights
    const Col col = a.cols_d[c];
    const bool normed = pro == TP_EMBED_NORM || pro == TP_RESID_NORM || pro == TP_FINAL;
    const bool resid = pro == TP_RESID_NORM || pro == TP_FINAL;
    float4 wpo[TP_PQ], wpr[TP_PQ];
    if (normed) {
#pragma unroll
        for (int k = 0; k < TP_PQ; k++) {
            const int q = tid + k * TP_THREADS;
            if (q < E / 4) {
                wpr[k] = ((const float4 *) a.wpre)[q];
                if (resid) wpo[k] = ((const float4 *) a.wpost)[q];
            }
        }
    }
    pdl_wait();
    if (pro == TP_Q8) {   // codes made by the producer: repack into the operand, copy the blocks' scale and sum
        const int nq = K / 4;
        for (int q0 = 0; q0 < nq; q0 += TP_THREADS) {
            const int q = q0 + tid;
            if (q < nq) {
                const uint32_t w = *(const uint32_t *) (a.q8_q + (size_t) c * K + 4 * q);
                const int G = a.G, g = c / G, cg = c - g * G;
                *(uint32_t *) (a.xb + tc_xb_code(G, K, g, cg, 4 * q)) = w;
                if ((q & 7) == 0) {
                    *(float *) (a.xb + tc_xb_scale(G, K, g, cg, q >> 3, 0)) = a.q8_d[(size_t) c * (K / 32) + (q >> 3)];
                    *(float *) (a.xb + tc_xb_scale(G, K, g, cg, q >> 3, 1)) = a.q8_s[(size_t) c * (K / 32) + (q >> 3)];
                }
            }
        }
        return;
    }
    if (pro == TP_CUT) {   // seoul.cpp:469: the SiLU output as it is; a thread's chunks load together, then are cut
        const float4 *in = (const float4 *) (a.in + (size_t) c * a.in_stride);
        const int nq = K / 4;
        constexpr int U = 8;
        for (int q0 = 0; q0 < nq; q0 += U * TP_THREADS) {
            float4 vv[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int q = q0 + u * TP_THREADS + tid;
                vv[u] = q < nq ? in[q] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (q0 + u * TP_THREADS >= nq) break;   // CTA-uniform
                const int q = q0 + u * TP_THREADS + tid;
                tp_cut(a, c, q, vv[u], q < nq);
            }
        }
        return;
    }
    const int nq = E / 4;
    if (pro == TP_CONV) {
        // seoul.cpp:410-414 (run) and 566-576 (run_batch): u = c * (b*x*w[d_conv] + sum_k st_k * w_k), st_k the b*x of
        // position p - d_conv + k: from this chunk's earlier columns when that position is in the chunk (columns of
        // one conversation at consecutive positions), else from the conv memory ring (slot of position p: p mod R)
        const int R = a.d_conv + 1, p0 = col.s->pos, p = p0 + col.off;
        const float4 *bcx = (const float4 *) (a.in + (size_t) c * a.in_stride);
        const float4 *wl = (const float4 *) (a.conv_w + (size_t) a.d_conv * E);
        const float *ring = col.ring + (size_t) a.conv_layer * R * E;
        float4 *slot = a.ring_conv ? (float4 *) (ring + (size_t) (p % R) * E) : nullptr;
        for (int q0 = 0; q0 < nq; q0 += TP_THREADS) {
            const int q = q0 + tid;
            const bool act = q < nq;
            const int qs = act ? q : 0;
            const float4 sv = mul4(bcx[qs], bcx[2 * nq + qs]);
            float4 u = mul4(sv, wl[qs]);
            for (int k = 0; k < a.d_conv; k++) {
                const int qp = p - a.d_conv + k;
                const float4 *wk = (const float4 *) (a.conv_w + (size_t) k * E);
                float4 pk;
                if (qp >= p0) {   // column c - d_conv + k of this chunk
                    const float4 *ob = (const float4 *) (a.in + (size_t) (c - a.d_conv + k) * a.in_stride);
                    pk = mul4(mul4(ob[qs], ob[2 * nq + qs]), wk[qs]);
                } else {
                    pk = mul4(__ldcg((const float4 *) (ring + (size_t) (((qp % R) + R) % R) * E) + qs), wk[qs]);
                }
                u = add4(u, pk);
            }
            tp_cut(a, c, q, mul4(u, bcx[nq + qs]), act);
            if (slot && act) slot[q] = sv;   // conv memory: slot p mod R takes b*x (seoul.cpp:419-423)
        }
        return;
    }
    // TP_EMBED_NORM, TP_RESID_NORM, TP_FINAL: the vector into shared memory, imi's RMS order by one warp; thread t
    // holds chunks t, t + TP_THREADS, ... (at most TP_PQ) in registers
    if (resid) {   // x = xin + norm(r) * w_post (imi_norm_mul_add, vec.h:41-44); r and x arrive in one round of loads
        const float4 *r4 = (const float4 *) (a.in + (size_t) c * a.in_stride);
        const float4 *x4 = (const float4 *) (a.xin + (size_t) c * a.x_stride);
        float4 xr[TP_PQ];
#pragma unroll
        for (int k = 0; k < TP_PQ; k++) {
            const int q = tid + k * TP_THREADS;
            if (q < nq) {
                ((float4 *) v)[q] = r4[q];
                xr[k] = x4[q];
            }
        }
        __syncthreads();
        if (warp == 0) {
            const float sc = warp_rms_scale(v, E, a.eps);
            if (tid == 0) red[0] = sc;
        }
        __syncthreads();
        const float sc = red[0];
#pragma unroll
        for (int k = 0; k < TP_PQ; k++) {
            const int q = tid + k * TP_THREADS;
            if (q < nq) {
                const float4 y = add4(xr[k], mul4(scl4(((float4 *) v)[q], sc), wpo[k]));
                ((float4 *) v)[q] = y;
                if (a.xout) ((float4 *) (a.xout + (size_t) c * a.x_stride))[q] = y;
            }
        }
    } else {   // the word row of a token (given, or the conversation's last pick) or the input vector
        const int tok = col.token == -2 ? col.s->next_token : col.token;
        for (int q = tid; q < nq; q += TP_THREADS) {
            float4 x;
            if (tok >= 0) {
                const uint8_t *row = a.emb + (size_t) tok * a.emb_row_bytes;
                x = a.emb_q6k ? word_chunk_q6k(row, q) : word_chunk(row, E, q);
            } else {
                x = ((const float4 *) col.embd)[q];
            }
            ((float4 *) v)[q] = x;
            if (a.xout) ((float4 *) (a.xout + (size_t) c * a.x_stride))[q] = x;
        }
    }
    __syncthreads();
    if (warp == 0) {   // h = norm(x) * w_pre (imi_norm_mul, vec.h:36-39)
        const float sc = warp_rms_scale(v, E, a.eps);
        if (tid == 0) red[1] = sc;
    }
    __syncthreads();
    const float sc = red[1];
    float *hid = pro == TP_FINAL ? col.hid_out : nullptr;
#pragma unroll
    for (int k = 0; k < TP_PQ; k++) {
        if (k * TP_THREADS >= nq) break;   // CTA-uniform
        const int q = tid + k * TP_THREADS;
        const bool act = q < nq;
        const float4 h = act ? mul4(scl4(((float4 *) v)[q], sc), wpr[k]) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (hid && act) ((float4 *) hid)[q] = h;
        tp_cut(a, c, q, h, act);
    }
    // conv memory of a prefill chunk: the slot of the column's position takes b*x (seoul.cpp:419-423), written one
    // launch after the conv read it (no column of the chunk reads a slot this launch writes). The columns are
    // consecutive positions of one conversation and columns c and c + d_conv + 1 share a slot: only the last
    // d_conv + 1 columns write, so the memory ends holding the chunk's last positions whatever order the CTAs run in
    if (a.ring_layer >= 0 && c + a.d_conv + 1 >= a.ncol) {
        const int R = a.d_conv + 1, p = col.s->pos + col.off;
        const float4 *bcx = (const float4 *) (a.ring_src + (size_t) c * a.ring_src_stride);
        float4 *slot = (float4 *) (col.ring + ((size_t) a.ring_layer * R + p % R) * E);
        for (int q = tid; q < nq; q += TP_THREADS) slot[q] = mul4(bcx[q], bcx[2 * nq + q]);
    }
}
#endif

}  // namespace imi

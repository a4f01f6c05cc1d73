// k_table: one 4-bit table times up to 8 inputs ("columns"): the replacement of imi_q4_group / imi_q4_group2 /
// imi_q4_group_batch (imi/core/tables.cpp:127-177,419-477) together with the small math imi's threads repeat before
// every table read (norms, residual adds, the short conv, the 8-bit cut; seoul.cpp:402-474).
//
// Per CTA: a contiguous slice of rows. Weights arrive in stages by TMA bulk copies (cp.async.bulk + mbarrier),
// issued before the kernel waits on its predecessor (programmatic dependent launch), so a table's first bytes stream
// while the previous launch finishes. Every CTA prepares the input itself (it is tiny), as every imi thread does.
//
// Two warp roles per CTA, pipelined over the stages through double-buffered shared memory and named barriers:
//   integer warps (8): dot_j = sum of 32 4-bit codes x 32 8-bit input codes for every (row, block j), with dp4a,
//                       stored as floats (exact: |dot| < 2^24), plus the rows' block scales;
//   chain warps (4):    one thread per (input, row): the float result in the exact order of group_avx2<false>
//                       (tables.cpp:127-143):  acc = fma(dot_j, d_j * dx_j, acc),  cor = fma(d_j, sx_j, cor)  for j in
//                       order, out = acc - 8 cor with one rounding; then the output stage (store, SiLU(gate)*up, or
//                       word scores with the first-maximum pick).
#pragma once
#include "common.cuh"

namespace imi {

// named barriers (0 is __syncthreads)
// READY + b: the integer warps hand buffer b to chain warp b; FREE + b: chain warp b hands it back (each barrier has
// the integer threads and one chain warp)
enum : int { NB_INT = 1, NB_READY = 2 /* +buffer */, NB_FREE = 2 + MV_NBUF /* +buffer */, NB_TAIL = 2 + 2 * MV_NBUF };
static_assert(NB_TAIL < 16 && MV_NBUF == MV_CWARPS, "named barriers: one buffer per chain warp");
constexpr int NB_PAIR = MV_ITHREADS + 32;
__device__ __forceinline__ void nbar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void nbar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// ---------------- input preparation ----------------
// Each thread owns the float4 chunks q = tid, tid + MV_THREADS, ... of an n_embd vector in every phase. MV_THREADS is
// a multiple of 32, so the 8 lanes holding chunks 8m..8m+7 hold one 32-value block, which cut_chunk cuts in place:
// the residual update, the norm and the 8-bit cut stay in registers; only the RMS reductions (one warp per column,
// imi's lane order) read the vector from shared memory.
constexpr int PQ = (6144 / 4 + MV_THREADS - 1) / MV_THREADS;   // chunks per thread (n_embd <= 6144)
struct PreRegs {
    float4 wpr[PQ], wpo[PQ];
};

// the word table row of `tok`, chunk q: d * (code - 8) for values 4q..4q+3 (codes of block j at bytes 16j..,
// values 0..15 in the low nibbles, 16..31 in the high ones; scales after the codes)
__device__ __forceinline__ float4 word_chunk(const uint8_t *row, int cols, int q) {
    const int j = q >> 3, k0 = (4 * q) & 31;
    const uint32_t w = *(const uint32_t *) (row + 16 * j + (k0 & 15));
    const float d = h2f(*(const uint16_t *) (row + cols / 2 + 2 * j));
    const int sh = k0 < 16 ? 0 : 4;
    return make_float4(__fmul_rn(d, (float) ((int) ((w >> sh) & 15) - 8)),
                       __fmul_rn(d, (float) ((int) ((w >> (8 + sh)) & 15) - 8)),
                       __fmul_rn(d, (float) ((int) ((w >> (16 + sh)) & 15) - 8)),
                       __fmul_rn(d, (float) ((int) ((w >> (24 + sh)) & 15) - 8)));
}
// the same for a Q6_K word row (imi_q6k_dequant_row, tables.cpp:216-233): value = d * scale * (code - 32), left to
// right; code of value t of a block = low 4 bits from ql, high 2 from qh
__device__ __forceinline__ float4 word_chunk_q6k(const uint8_t *row, int q) {
    const uint8_t *b = row + (size_t) (q >> 6) * 210;
    const int t = (4 * q) & 255, n = t >> 7, k = (t & 127) >> 5, l = t & 31;
    const float d = h2f((uint16_t) (b[208] | (b[209] << 8)));
    const float ds = __fmul_rn(d, (float) (int8_t) b[192 + (t >> 4)]);
    const uint8_t *ql = b + 64 * n + (k & 1) * 32 + l, *qh = b + 128 + 32 * n + l;
    float v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int lo = k < 2 ? (ql[u] & 15) : (ql[u] >> 4), code = lo | (((qh[u] >> (2 * k)) & 3) << 4);
        v[u] = __fmul_rn(ds, (float) (code - 32));
    }
    return make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ float4 word_row_chunk(const MvArgs &a, const uint8_t *row, int cols, int q) {
    return a.emb_q6k ? word_chunk_q6k(row, q) : word_chunk(row, cols, q);
}
__device__ __forceinline__ float4 mul4(float4 a, float4 b) {
    return make_float4(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y), __fmul_rn(a.z, b.z), __fmul_rn(a.w, b.w));
}
__device__ __forceinline__ float4 add4(float4 a, float4 b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
__device__ __forceinline__ float4 scl4(float4 a, float s) {
    return make_float4(__fmul_rn(a.x, s), __fmul_rn(a.y, s), __fmul_rn(a.z, s), __fmul_rn(a.w, s));
}
// ring slot of position qp (negative before position d_conv: those slots hold zeros)
__device__ __forceinline__ int ring_slot(int qp, int R) { return ((qp % R) + R) % R; }

// conv tap products st_k * w_k (seoul.cpp:410-414) of one column for this thread's chunks, for the taps whose
// position lies before the step (read from the conv memory ring, positions counted from `p0`): prod[k][n_embd]
__device__ __forceinline__ void conv_ring_products(const MvArgs &a, const PreCol &pc, int p0, float *prod) {
    const int E = a.n_embd, nq = E / 4, R = a.d_conv + 1, p = p0 + pc.off;
    const float *ring = pc.ring + (size_t) a.conv_layer * R * E;
    for (int k = 0; k < a.d_conv; k++) {
        const int qp = p - a.d_conv + k;
        if (qp >= p0) break;   // this tap and the later ones come from this step's own columns
        const float4 *st = (const float4 *) (ring + (size_t) ring_slot(qp, R) * E);
        const float4 *wk = (const float4 *) (a.conv_w + (size_t) k * E);
        for (int q = threadIdx.x; q < nq; q += MV_THREADS)
            ((float4 *) (prod + (size_t) k * E))[q] = mul4(__ldcg(st + q), wk[q]);
    }
}

// Part 1, before the dependency wait: what does not depend on the launches in flight. The column descriptors (written
// before the step was launched) into shared memory, the norm weights into registers, the word row of a given token,
// and (up to 2 columns) the products of the conv taps read from the conv memory under the position read now; part 2
// reads the position again and recomputes those products if it moved (it moves only at the end of a step).
template <int PRO, int NC>
__device__ __forceinline__ void table_preload(const MvArgs &a, const MvPlan &P, uint8_t *sm, PreRegs &pr) {
    if (PRO == P_Q8IN || PRO == P_CUT) return;
    const int tid = threadIdx.x, nc = a.ncol, E = a.n_embd, nq = E / 4;
    PreCol *pc = (PreCol *) (sm + P.pc);
    float *vb = (float *) (sm + P.vb);
    const int VL = mv_vb_len(PRO, a.cols, E, NC, a.d_conv);
    if (tid < nc) {
        const Col &col = a.cols_d[tid];
        PreCol c;
        c.s = col.s;
        c.ring = col.ring;
        c.embd = col.embd;
        c.off = col.off;
        c.tok = col.token;
        c.pos = PRO == P_CONV ? ld_relaxed(&col.s->pos) : 0;
        c.pad = 0;
        pc[tid] = c;
    }
    const bool norm = PRO == P_EMBED_NORM || PRO == P_RESID_NORM || PRO == P_FINAL;
    const bool resid = PRO == P_RESID_NORM || PRO == P_FINAL;
    if (norm) {
#pragma unroll
        for (int k = 0; k < PQ; k++) {
            const int q = tid + k * MV_THREADS;
            if (q < nq) {
                pr.wpr[k] = ((const float4 *) a.wpre)[q];
                if (resid) pr.wpo[k] = ((const float4 *) a.wpost)[q];
            }
        }
    }
    __syncthreads();
    if (PRO == P_EMBED_NORM) {
        for (int c = 0; c < nc; c++) {
            const int tok = pc[c].tok;
            if (tok >= 0) {
                const uint8_t *row = a.emb + (size_t) tok * a.emb_row_bytes;
                for (int q = tid; q < nq; q += MV_THREADS) ((float4 *) (vb + c * VL))[q] = word_row_chunk(a, row, E, q);
            } else if (tok == -1) {
                for (int q = tid; q < nq; q += MV_THREADS) ((float4 *) (vb + c * VL))[q] = ((const float4 *) pc[c].embd)[q];
            }
        }
    } else if (PRO == P_CONV && NC <= 2) {
        for (int c = 0; c < nc; c++) conv_ring_products(a, pc[c], pc[c].pos, vb + c * VL);
    }
}

// Part 2, after the dependency wait, all MV_THREADS threads, all columns; ends with a __syncthreads. The activations
// the previous launches produced arrive in one batch (cp.async, one L2 round trip).
// late_weights() issues the table's bulk copies for the norm/residual reads (P_RESID_NORM, P_FINAL) once the
// activations are in shared memory: those few latency-critical loads go ahead of the copies, which still arrive before
// the long input preparation ends
template <int PRO, int NC, class LateW>
__device__ void table_prologue(const MvArgs &a, const MvPlan &P, uint8_t *sm, const PreRegs &pr, LateW &&late_weights) {
    int8_t *xq = (int8_t *) (sm + P.xq);
    float *xd = (float *) (sm + P.xd), *xs = (float *) (sm + P.xs), *vb = (float *) (sm + P.vb);
    float *red = (float *) (sm + P.red);
    const PreCol *pc = (const PreCol *) (sm + P.pc);
    const int tid = threadIdx.x, warp = tid >> 5, nc = a.ncol, K = a.cols, nb = K / 32, E = a.n_embd, nq = E / 4;
    const int VL = mv_vb_len(PRO, K, E, NC, a.d_conv);
    if (PRO == P_Q8IN) {   // codes made by the producer of the input (or given): [c][K], [c][K/32]
        for (int i = tid; i < nc * K / 16; i += MV_THREADS) cp16(xq + 16 * i, a.q8_q + 16 * i);
        for (int j = tid; j < nc * nb; j += MV_THREADS) {
            xd[j] = a.q8_d[j];
            xs[j] = a.q8_s[j];
        }
        cp_wait_all();
        __syncthreads();
        return;
    }
    if (PRO == P_CUT) {   // the input as it is (seoul.cpp:457,469)
        const int nk = K / 4;
        for (int c = 0; c < nc; c++)
            for (int q0 = 0; q0 < nk; q0 += MV_THREADS) {
                const int q = q0 + tid;
                const bool act = q < nk;
                const float4 v = act ? ((const float4 *) (a.in + (size_t) c * a.in_stride))[q] : make_float4(0, 0, 0, 0);
                cut_chunk(v, act, q, xq + c * K, xd + c * nb, xs + c * nb);
            }
        __syncthreads();
        return;
    }
    if (PRO == P_CONV) {
        // seoul.cpp:410-414 (run) and 566-576 (run_batch): u = c * (b*x*w[d_conv] + sum_k st_k * w_k), st_k the b*x of
        // position p - d_conv + k: from this step's earlier columns of the same conversation when that position is in
        // this step, else from the conv memory ring; u is cut where it is made
        const int R = a.d_conv + 1;
        const float4 *wl = (const float4 *) (a.conv_w + (size_t) a.d_conv * E);
        for (int c = 0; c < nc; c++) {
            const PreCol &col = pc[c];
            const int p0 = ld_relaxed(&col.s->pos), p = p0 + col.off;
            const bool pre = NC <= 2 && p0 == col.pos;   // the products made before the wait hold for this position
            const float *prod = vb + c * VL;
            const float4 *bcx = (const float4 *) (a.in + (size_t) c * a.in_stride);
            const float *ring = col.ring + (size_t) a.conv_layer * R * E;
            float4 *slot = a.ring_layer >= 0 ? (float4 *) (ring + (size_t) (p % R) * E) : nullptr;
            for (int q0 = 0; q0 < nq; q0 += 2 * MV_THREADS) {   // two chunks per round, their loads first
                int qq[2];
                bool act[2];
                float4 bv[2], cv[2], xv[2], wv[2];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    qq[h] = q0 + tid + h * MV_THREADS;
                    act[h] = qq[h] < nq;
                    const int qs = act[h] ? qq[h] : 0;
                    bv[h] = bcx[qs];
                    cv[h] = bcx[nq + qs];
                    xv[h] = bcx[2 * nq + qs];
                    wv[h] = wl[qs];
                }
                float4 sv[2], u[2];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    sv[h] = mul4(bv[h], xv[h]);
                    u[h] = mul4(sv[h], wv[h]);
                }
                for (int k = 0; k < a.d_conv; k++) {
                    const int qp = p - a.d_conv + k;
                    const float4 *wk = (const float4 *) (a.conv_w + (size_t) k * E);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const int qs = act[h] ? qq[h] : 0;
                        float4 pk;
                        if (qp >= p0) {   // column c - d_conv + k of this step (a prefill chunk of one conversation)
                            const float4 *ob = (const float4 *) (a.in + (size_t) (c - a.d_conv + k) * a.in_stride);
                            pk = mul4(mul4(ob[qs], ob[2 * nq + qs]), wk[qs]);
                        } else if (pre) {
                            pk = ((const float4 *) (prod + (size_t) k * E))[qs];
                        } else {
                            pk = mul4(__ldcg((const float4 *) (ring + (size_t) ring_slot(qp, R) * E) + qs), wk[qs]);
                        }
                        u[h] = add4(u[h], pk);
                    }
                }
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    if (q0 + h * MV_THREADS < nq)   // CTA-uniform: skip rounds with no chunk at all
                        cut_chunk(mul4(u[h], cv[h]), act[h], qq[h], xq + c * K, xd + c * nb, xs + c * nb);
                    // conv memory: slot p mod (d_conv + 1) takes b*x (seoul.cpp:419-423); no column of this step reads
                    // it (the host sets ring_layer here only for steps of distinct conversations); spread over the CTAs
                    if (slot && act[h] && (int) (qq[h] % gridDim.x) == (int) blockIdx.x) slot[qq[h]] = sv[h];
                }
            }
        }
        __syncthreads();
        return;
    }
    // P_EMBED_NORM, P_RESID_NORM, P_FINAL
    const bool resid = PRO == P_RESID_NORM || PRO == P_FINAL;
    const bool x_in_smem = NC <= 2;   // the residual staged beside r (else read where it is used)
    if (resid) {   // [c]: r (the table output to post-norm) then x (the residual stream)
        for (int c = 0; c < nc; c++)
            for (int q = tid; q < nq; q += MV_THREADS) {
                cp16(vb + c * VL + 4 * q, a.in + (size_t) c * a.in_stride + 4 * q);
                if (x_in_smem) cp16(vb + c * VL + E + 4 * q, a.xin + (size_t) c * a.x_stride + 4 * q);
            }
        cp_wait_all();
    } else {
        for (int c = 0; c < nc; c++) {
            if (pc[c].tok != -2) continue;   // the greedy pick of the conversation's last step
            const uint8_t *row = a.emb + (size_t) pc[c].s->next_token * a.emb_row_bytes;
            for (int q = tid; q < nq; q += MV_THREADS) ((float4 *) (vb + c * VL))[q] = word_row_chunk(a, row, E, q);
        }
    }
    __syncthreads();
    late_weights();
    if (resid) {   // x += norm(r) * w_post (imi_norm_mul_add, vec.h:41-44); the new x replaces r in place
        if (warp < nc) {
            const float sc = warp_rms_scale(vb + warp * VL, E, a.eps);
            if ((tid & 31) == 0) red[warp] = sc;
        }
        __syncthreads();
        for (int c = 0; c < nc; c++) {
            const float sc = red[c];
            float4 *v4 = (float4 *) (vb + c * VL);
            const float4 *x4 = x_in_smem ? (const float4 *) (vb + c * VL + E) : (const float4 *) (a.xin + (size_t) c * a.x_stride);
#pragma unroll
            for (int k = 0; k < PQ; k++) {
                const int q = tid + k * MV_THREADS;
                if (q < nq) {
                    const float4 y = add4(x4[q], mul4(scl4(v4[q], sc), pr.wpo[k]));
                    v4[q] = y;
                    if (a.xout && (int) (q % gridDim.x) == (int) blockIdx.x)   // the residual stream, spread over CTAs
                        ((float4 *) (a.xout + (size_t) c * a.x_stride))[q] = y;
                }
            }
        }
        __syncthreads();
    } else if (a.xout) {
        for (int c = 0; c < nc; c++)
            for (int q = tid; q < nq; q += MV_THREADS)
                if ((int) (q % gridDim.x) == (int) blockIdx.x)
                    ((float4 *) (a.xout + (size_t) c * a.x_stride))[q] = ((const float4 *) (vb + c * VL))[q];
    }
    // h = norm(x) * w_pre (imi_norm_mul, vec.h:36-39), cut where it is made
    if (warp < nc) {
        const float sc = warp_rms_scale(vb + warp * VL, E, a.eps);
        if ((tid & 31) == 0) red[32 + warp] = sc;
    }
    __syncthreads();
    for (int c = 0; c < nc; c++) {
        const float sc = red[32 + c];
        const float4 *v4 = (const float4 *) (vb + c * VL);
        float *hid = PRO == P_FINAL ? a.cols_d[c].hid_out : nullptr;
#pragma unroll
        for (int k = 0; k < PQ; k++) {
            if (k * MV_THREADS >= nq) break;   // CTA-uniform
            const int q = tid + k * MV_THREADS;
            const bool act = q < nq;
            const float4 h = act ? mul4(scl4(v4[q], sc), pr.wpr[k]) : make_float4(0, 0, 0, 0);
            if (hid && act && (int) (q % gridDim.x) == (int) blockIdx.x) ((float4 *) hid)[q] = h;
            cut_chunk(h, act, q, xq + c * K, xd + c * nb, xs + c * nb);
        }
    }
    // conv memory of a prefill chunk: the slot of each column's position takes b*x (seoul.cpp:419-423); written one
    // launch after the conv read it, so no CTA of the reading launch can see it early; spread over the CTAs
    if (a.ring_layer >= 0) {
        const int R = a.d_conv + 1;
        for (int c = 0; c < nc; c++) {
            const Col &col = a.cols_d[c];
            const int p = col.s->pos + col.off;
            const float *bcx = a.ring_src + (size_t) c * a.ring_src_stride;
            float4 *slot = (float4 *) (col.ring + ((size_t) a.ring_layer * R + p % R) * E);
            for (int q = blockIdx.x * MV_THREADS + tid; q < nq; q += gridDim.x * MV_THREADS)
                slot[q] = mul4(((const float4 *) bcx)[q], ((const float4 *) (bcx + 2 * E))[q]);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ int dot_block(const uint4 c, const int *x) {
    const int l0 = (int) (c.x & 0x0f0f0f0fu), l1 = (int) (c.y & 0x0f0f0f0fu), l2 = (int) (c.z & 0x0f0f0f0fu),
              l3 = (int) (c.w & 0x0f0f0f0fu);
    const int h0 = (int) ((c.x >> 4) & 0x0f0f0f0fu), h1 = (int) ((c.y >> 4) & 0x0f0f0f0fu),
              h2 = (int) ((c.z >> 4) & 0x0f0f0f0fu), h3 = (int) ((c.w >> 4) & 0x0f0f0f0fu);
    int s = __dp4a(l0, x[0], 0);
    s = __dp4a(l1, x[1], s);
    s = __dp4a(l2, x[2], s);
    s = __dp4a(l3, x[3], s);
    s = __dp4a(h0, x[4], s);
    s = __dp4a(h1, x[5], s);
    s = __dp4a(h2, x[6], s);
    s = __dp4a(h3, x[7], s);
    return s;
}

__device__ __forceinline__ unsigned long long amax_key(float v, int idx) {
    v = v + 0.0f;   // -0 -> +0: equal values compare equal and the lowest id wins
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long) o << 32) | (unsigned long long) (0xffffffffu - (uint32_t) idx);
}
__device__ __forceinline__ float amax_val(unsigned long long k) {
    const uint32_t o = (uint32_t) (k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

// the two fma chains of one (input, row), blocks in order (group_avx2<false>, tables.cpp:134-142); the next 8
// blocks' operands load while these 8 blocks run (nb is a multiple of 8)
__device__ __forceinline__ float row_chain(const float *f, const uint16_t *d, const float *xdc, const float *xsc,
                                           int nb) {
    float acc = 0.0f, cor = 0.0f;
    float4 fv[2], xv[2], sv[2];
    uint2 dv[2];
#pragma unroll
    for (int g = 0; g < 2; g++) {
        fv[g] = *(const float4 *) (f + 4 * g);
        xv[g] = *(const float4 *) (xdc + 4 * g);
        sv[g] = *(const float4 *) (xsc + 4 * g);
        dv[g] = *(const uint2 *) (d + 4 * g);
    }
    for (int j = 0; j < nb; j += 8) {
        const int jn = j + 8 < nb ? j + 8 : j;   // the last round reloads its own blocks (in bounds, unused)
        float4 fn[2], xn[2], sn[2];
        uint2 dn[2];
#pragma unroll
        for (int g = 0; g < 2; g++) {
            fn[g] = *(const float4 *) (f + jn + 4 * g);
            xn[g] = *(const float4 *) (xdc + jn + 4 * g);
            sn[g] = *(const float4 *) (xsc + jn + 4 * g);
            dn[g] = *(const uint2 *) (d + jn + 4 * g);
        }
#pragma unroll
        for (int g = 0; g < 2; g++) {
            const float d0 = h2f((uint16_t) (dv[g].x & 0xffff)), d1 = h2f((uint16_t) (dv[g].x >> 16)),
                        d2 = h2f((uint16_t) (dv[g].y & 0xffff)), d3 = h2f((uint16_t) (dv[g].y >> 16));
            acc = __fmaf_rn(fv[g].x, __fmul_rn(d0, xv[g].x), acc);
            cor = __fmaf_rn(d0, sv[g].x, cor);
            acc = __fmaf_rn(fv[g].y, __fmul_rn(d1, xv[g].y), acc);
            cor = __fmaf_rn(d1, sv[g].y, cor);
            acc = __fmaf_rn(fv[g].z, __fmul_rn(d2, xv[g].z), acc);
            cor = __fmaf_rn(d2, sv[g].z, cor);
            acc = __fmaf_rn(fv[g].w, __fmul_rn(d3, xv[g].w), acc);
            cor = __fmaf_rn(d3, sv[g].w, cor);
        }
#pragma unroll
        for (int g = 0; g < 2; g++) {
            fv[g] = fn[g];
            xv[g] = xn[g];
            sv[g] = sn[g];
            dv[g] = dn[g];
        }
    }
    return __fmaf_rn(-8.0f, cor, acc);
}

// the Q4_1 chains of one (input, row) (group_avx2<true>, tables.cpp:127-143): acc as for Q4_0, cor = fma(m_j, s_j,
// cor) over the blocks' minimums, result acc + cor with one rounding; blocks in order
__device__ __noinline__ float row_chain_m(const float *f, const uint16_t *d, const uint16_t *mn, const float *xdc,
                                          const float *xsc, int nb) {
    float acc = 0.0f, cor = 0.0f;
#pragma unroll 4
    for (int j = 0; j < nb; j += 4) {
        const float4 fv = *(const float4 *) (f + j), xv = *(const float4 *) (xdc + j), sv = *(const float4 *) (xsc + j);
        const uint2 dv = *(const uint2 *) (d + j), mv = *(const uint2 *) (mn + j);
        const float d0 = h2f((uint16_t) (dv.x & 0xffff)), d1 = h2f((uint16_t) (dv.x >> 16)),
                    d2 = h2f((uint16_t) (dv.y & 0xffff)), d3 = h2f((uint16_t) (dv.y >> 16));
        const float m0 = h2f((uint16_t) (mv.x & 0xffff)), m1 = h2f((uint16_t) (mv.x >> 16)),
                    m2 = h2f((uint16_t) (mv.y & 0xffff)), m3 = h2f((uint16_t) (mv.y >> 16));
        acc = __fmaf_rn(fv.x, __fmul_rn(d0, xv.x), acc);
        cor = __fmaf_rn(m0, sv.x, cor);
        acc = __fmaf_rn(fv.y, __fmul_rn(d1, xv.y), acc);
        cor = __fmaf_rn(m1, sv.y, cor);
        acc = __fmaf_rn(fv.z, __fmul_rn(d2, xv.z), acc);
        cor = __fmaf_rn(m2, sv.z, cor);
        acc = __fmaf_rn(fv.w, __fmul_rn(d3, xv.w), acc);
        cor = __fmaf_rn(m3, sv.w, cor);
    }
    return __fadd_rn(acc, cor);
}

// HM: Q4_1 rows (minimums beside the scales); a compile-time switch, so the Q4_0 instances carry none of it
template <int PRO, int EPI, int NC, int HM>
__global__ void __launch_bounds__(MV_THREADS, 1) k_table(const __grid_constant__ MvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ int abort_flag, last_cta;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, K = a.cols, nb = K / 32, ld = nb + 4,
              nc = a.ncol, sr = a.sr;
    const int NS = a.nstage;
    const MvPlan P = mv_plan(K, sr, NC, mv_vb_len(PRO, K, a.n_embd, NC, a.d_conv), a.ab_len, NS, HM);
    uint8_t *stage = sm + P.stage;
    uint64_t *bar = (uint64_t *) (sm + P.bar);
    const int8_t *xq = (const int8_t *) (sm + P.xq);
    const float *xd = (const float *) (sm + P.xd), *xs = (const float *) (sm + P.xs);
    float *fs = (float *) (sm + P.fs), *red = (float *) (sm + P.red), *ab = (float *) (sm + P.ab);
    uint16_t *dd = (uint16_t *) (sm + P.dd);

    const int units = a.rows / a.unit;
    const int u0 = (int) ((long long) units * blockIdx.x / gridDim.x),
              u1 = (int) ((long long) units * (blockIdx.x + 1) / gridDim.x);
    const int r0 = u0 * a.unit, nrows = (u1 - u0) * a.unit;
    const int nst = (nrows + sr - 1) / sr;

    {   // later phases read the parameter block piecemeal; reading every word of it once now, before the dependency
        // wait, brings it on chip while nothing waits on it
        __shared__ volatile int pwarm[(sizeof(MvArgs) + 3) / 4];
        if (tid < (int) (sizeof(MvArgs) / 4)) pwarm[tid] = reinterpret_cast<const int *>(&a)[tid];
    }
    unsigned long long *trace = a.trace ? a.trace + (size_t) blockIdx.x * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    if (tid == 0) {
        for (int b = 0; b < NS; b++) mbar_init(&bar[b], 1);
        fence_barrier_init();
        abort_flag = 0;
    }
    __syncthreads();
    auto issue = [&](int st) {
        const int rr = st * sr, n = min(sr, nrows - rr);
        const uint32_t bytes = (uint32_t) n * (uint32_t) a.row_bytes;
        uint64_t *b = &bar[st % NS];
        mbar_expect_tx(b, bytes);
        bulk_g2s(stage + (st % NS) * P.sstride, a.W + (size_t) (r0 + rr) * a.row_bytes, bytes, b);
    };
    constexpr bool late = PRO == P_RESID_NORM || PRO == P_FINAL;
    // by one thread: the first stages (later ones are issued as their slots free up; an L2 bulk prefetch of the rest
    // of the slice here made the batch-1 step 1.5% slower). The norm/residual reads take only the first stage with
    // their activations and the rest once the input preparation is done: copies landing in shared memory during the
    // preparation slowed it more than the early bytes gained (riding step 2.6% faster this way)
    const int nfirst = min(late ? 1 : NS, nst);
    auto issue_weights = [&]() {
        for (int st = 0; st < nfirst; st++) issue(st);
    };
    // the weights do not depend on the previous launch: start them before waiting on it
    if (!late && tid == 0) issue_weights();
    pdl_trigger();
    PreRegs pr;
    table_preload<PRO, NC>(a, P, sm, pr);
    if (trace && tid == 0) trace[15] = global_ns();
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    // norm/residual reads: issued once the activations are in, by a lane of the last warp, which holds the fewest
    // chunks of the input preparation (none while n_embd / 4 <= MV_THREADS - 32)
    table_prologue<PRO, NC>(a, P, sm, pr, [&]() { if (late && tid == MV_THREADS - 32) issue_weights(); });
    if (late && tid == MV_THREADS - 32)
        for (int st = nfirst; st < min(NS, nst); st++) issue(st);
    if (trace && tid == 0) trace[2] = global_ns();

    if (warp < MV_IWARPS) {
        // ---------------- integer warps ----------------
        const int it = tid;
        const bool fixed_j = (MV_ITHREADS % nb) == 0;   // nb divides 256: each thread keeps one block column
        const int j0 = fixed_j ? it % nb : 0, rstep = fixed_j ? MV_ITHREADS / nb : 0;
        constexpr int NX = NC <= 2 ? NC : 1;
        int xw[NX][8];
        if (NC <= 2 && fixed_j) {
#pragma unroll
            for (int c = 0; c < NX; c++) {
                const int4 *xp = (const int4 *) (xq + c * K + 32 * j0);
                const int4 x0 = xp[0], x1 = xp[1];
                xw[c][0] = x0.x; xw[c][1] = x0.y; xw[c][2] = x0.z; xw[c][3] = x0.w;
                xw[c][4] = x1.x; xw[c][5] = x1.y; xw[c][6] = x1.z; xw[c][7] = x1.w;
            }
        }
        const int nchunk = nb / 4;   // 8-byte chunks of a row's scales (scale rows are nb + 4 halfs: 8-byte aligned)
        for (int st = 0; st < nst; st++) {
            const int b = st % MV_NBUF;
            // each thread waits on the stage itself (a phase completes for all at once); a wait that gives up marks
            // the CTA aborted before this thread's READY arrival, which the chain warp's sync orders after it
            const bool ok = mbar_wait(&bar[st % NS], (uint32_t) ((st / NS) & 1));
            if (!ok) {
                abort_flag = 1;
                atomicExch(a.err, 7);
            }
            if (st >= MV_NBUF) nbar_sync(NB_FREE + b, NB_PAIR);   // chain warp b is done with buffer b
            if (ok) {
                const int rb = st * sr, nr = min(sr, nrows - rb);
                const uint8_t *sb = stage + (st % NS) * P.sstride;
                float *f = fs + b * NC * sr * ld;
                uint16_t *dq = dd + b * sr * ld;
                for (int idx = it; idx < nr * nchunk; idx += MV_ITHREADS) {   // the rows' scales
                    const int r = idx / nchunk, k = idx - r * nchunk;
                    *(uint2 *) (dq + r * ld + 4 * k) = *(const uint2 *) (sb + (size_t) r * a.row_bytes + K / 2 + 8 * k);
                }
                if (HM) {   // Q4_1: the rows' minimums, after the scales in the row and in the second half here
                    uint16_t *mq = dq + MV_NBUF * sr * ld;
                    for (int idx = it; idx < nr * nchunk; idx += MV_ITHREADS) {
                        const int r = idx / nchunk, k = idx - r * nchunk;
                        *(uint2 *) (mq + r * ld + 4 * k) =
                            *(const uint2 *) (sb + (size_t) r * a.row_bytes + K / 2 + 2 * nb + 8 * k);
                    }
                }
                auto one = [&](int r, int j, bool cached) {
                    const uint4 code = *(const uint4 *) (sb + (size_t) r * a.row_bytes + 16 * j);
#pragma unroll
                    for (int c = 0; c < NC; c++) {
                        if (c < nc) {
                            int s;
                            if (NC <= 2 && cached) {
                                s = dot_block(code, xw[c < NX ? c : 0]);
                            } else {
                                const int4 *xp = (const int4 *) (xq + c * K + 32 * j);
                                const int4 x0 = xp[0], x1 = xp[1];
                                const int x8[8] = { x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w };
                                s = dot_block(code, x8);
                            }
                            f[(c * sr + r) * ld + j] = __int2float_rn(s);
                            if (c == 0 && a.dots) a.dots[(size_t) (r0 + rb + r) * nb + j] = s;
                        }
                    }
                };
                if (fixed_j) {   // rows it/nb + k*rstep, 4 at a time with their code loads first
                    for (int rr = it / nb; rr < nr; rr += 4 * rstep) {
                        uint4 code[4];
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            if (rr + u * rstep < nr)
                                code[u] = *(const uint4 *) (sb + (size_t) (rr + u * rstep) * a.row_bytes + 16 * j0);
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const int r = rr + u * rstep;
                            if (r >= nr) break;
#pragma unroll
                            for (int c = 0; c < NC; c++) {
                                if (c < nc) {
                                    int s;
                                    if (NC <= 2) {
                                        s = dot_block(code[u], xw[c < NX ? c : 0]);
                                    } else {
                                        const int4 *xp = (const int4 *) (xq + c * K + 32 * j0);
                                        const int4 x0 = xp[0], x1 = xp[1];
                                        const int x8[8] = { x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w };
                                        s = dot_block(code[u], x8);
                                    }
                                    f[(c * sr + r) * ld + j0] = __int2float_rn(s);
                                    if (c == 0 && a.dots) a.dots[(size_t) (r0 + rb + r) * nb + j0] = s;
                                }
                            }
                        }
                    }
                } else {
                    for (int idx = it; idx < nr * nb; idx += MV_ITHREADS) one(idx / nb, idx % nb, false);
                }
            }
            if (st + NS < nst) {   // the slot is refilled: every integer thread must be done with it first
                nbar_sync(NB_INT, MV_ITHREADS);
                if (it == 0 && ok) {
                    fence_proxy_async();
                    issue(st + NS);
                }
            }
            if (trace && it == 0 && st < 11) trace[3 + st] = global_ns();
            nbar_arrive(NB_READY + b, NB_PAIR);
        }
        for (int st = max(nst - MV_NBUF, 0); st < nst; st++) nbar_sync(NB_FREE + st % MV_NBUF, NB_PAIR);
        return;
    }

    // ---------------- chain warps: warp cw takes stages cw, cw + MV_NBUF, ...; one lane per (input, row) ----------------
    const int ct = tid - MV_ITHREADS, cw = ct >> 5;
    unsigned long long best[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) best[c] = 0ull;
    for (int st = cw; st < nst; st += MV_NBUF) {
        const int b = cw;
        nbar_sync(NB_READY + b, NB_PAIR);
        const bool ok = abort_flag == 0;
        const int rb = st * sr, nr = min(sr, nrows - rb);
        const float *f = fs + b * NC * sr * ld;
        const uint16_t *dq = dd + b * sr * ld;
        if (ok) {
            for (int base = 0; base < nc * nr; base += 32) {   // warp-uniform trip count
                const int t = base + lane;
                const bool act = t < nc * nr;
                const int c = act ? t / nr : 0, r = act ? t - c * nr : 0;
                float v = 0.0f;
                if (act)
                    v = HM ? row_chain_m(f + (c * sr + r) * ld, dq + r * ld, dq + MV_NBUF * sr * ld + r * ld,
                                              xd + c * nb, xs + c * nb, nb)
                                : row_chain(f + (c * sr + r) * ld, dq + r * ld, xd + c * nb, xs + c * nb, nb);
                if (EPI == E_STORE) {
                    if (act) a.out[(size_t) c * a.out_stride + r0 + rb + r] = v;
                } else if (EPI == E_SILU) {   // rows (2i, 2i+1) are (gate_i, up_i): act_i = silu(gate) * up (seoul.cpp:384-391)
                    const float u = __shfl_down_sync(0xffffffffu, v, 1);
                    if (act && (r & 1) == 0) {
                        const float sl = __fdiv_rn(v, __fadd_rn(1.0f, exp_cr(-v)));
                        const float y = __fmul_rn(sl, u);
                        a.out[(size_t) c * a.out_stride + (r0 + rb + r) / 2] = y;
                        if (a.q8o_q) ab[c * a.ab_len + (rb + r) / 2] = y;
                    }
                } else if (act) {   // E_HEAD: word scores and the running first maximum
                    const int row = r0 + rb + r;
                    float *lg = a.cols_d[c].logits;
                    if (lg) lg[row] = v;
#pragma unroll
                    for (int cc = 0; cc < NC; cc++)
                        if (cc == c) {
                            const unsigned long long k = amax_key(v, row);
                            best[cc] = k > best[cc] ? k : best[cc];
                        }
                }
            }
        }
        nbar_arrive(NB_FREE + b, NB_PAIR);
    }
    if (trace && lane == 0) atomicMax(&trace[14], global_ns());
    if (EPI == E_SILU && a.q8o_q && abort_flag == 0) {   // the cut of this CTA's whole 32-value blocks (imi_cut32)
        nbar_sync(NB_TAIL, MV_CTHREADS);
        const int nch = nrows / 8, half = a.rows / 2;   // float4 chunks of produced values per column
        for (int b0 = 0; b0 < nc * nch; b0 += MV_CTHREADS) {   // 8 lanes per block; a column has whole blocks
            const int t = b0 + ct;
            const bool act = t < nc * nch;
            const int c = act ? t / nch : 0, q = act ? t - c * nch : 0;
            const float4 v = act ? *(const float4 *) (ab + c * a.ab_len + 4 * q) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            cut_chunk(v, act, q, a.q8o_q + (size_t) c * half + r0 / 2, a.q8o_d + (size_t) c * (half / 32) + r0 / 64,
                      a.q8o_s + (size_t) c * (half / 32) + r0 / 64);
        }
    }

    if (EPI == E_HEAD) {   // the step ends here: pick, position, counters (one CTA, the last to finish)
        unsigned long long *wbest = (unsigned long long *) (red + 64);
#pragma unroll
        for (int c = 0; c < NC; c++) {
            unsigned long long k = best[c];
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const unsigned long long u = __shfl_xor_sync(0xffffffffu, k, o);
                k = u > k ? u : k;
            }
            if (lane == 0) wbest[c * MV_CWARPS + cw] = k;
        }
        nbar_sync(NB_TAIL, MV_CTHREADS);
        if (ct < nc && abort_flag == 0) {
            unsigned long long k = 0;
            for (int w = 0; w < MV_CWARPS; w++) k = wbest[ct * MV_CWARPS + w] > k ? wbest[ct * MV_CWARPS + w] : k;
            atomicMax(&a.cols_d[ct].s->amax, k);
        }
        __threadfence();
        nbar_sync(NB_TAIL, MV_CTHREADS);
        if (ct == 0) last_cta = atomicAdd(a.done, 1u) == gridDim.x - 1;
        nbar_sync(NB_TAIL, MV_CTHREADS);
        if (last_cta && ct < nc) {
            __threadfence();
            const Col col = a.cols_d[ct];
            const unsigned long long k = atomicExch(&col.s->amax, 0ull);
            const int id = (int) (0xffffffffu - (uint32_t) (k & 0xffffffffu));
            col.s->next_token = id;
            col.s->amax_val = amax_val(k);
            if (col.picks) col.picks[col.s->pos + col.off] = id;
            if (col.pos_inc) atomicAdd(&col.s->pos, col.pos_inc);
        }
        if (last_cta && ct == 0) *a.done = 0;
    }
}

}  // namespace imi

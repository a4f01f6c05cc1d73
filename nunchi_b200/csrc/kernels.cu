// sm_100a kernels of the decode engine.
//
// k_table: one 4-bit table times up to 8 inputs ("columns"), the replacement of imi_q4_group / imi_q4_group2 /
//   imi_q4_group_batch (imi/core/tables.cpp:127-177,419-477) together with the small math that imi's threads repeat
//   before every table read (norms, residual adds, the short conv, the 8-bit cut; seoul.cpp:402-474). Each CTA owns a
//   contiguous slice of rows; its weights arrive by TMA bulk copies into shared memory, issued before the kernel waits
//   on its predecessor (programmatic dependent launch), so the weight stream of step k+1 overlaps the tail of step k.
//   Every CTA recomputes the (tiny) input preparation itself, as every imi thread does.
//   Per row, the float result is the exact order of group_avx2<false> (tables.cpp:127-143):
//       acc = fma(float(dot_j), d_j * dx_j, acc);  cor = fma(d_j, sx_j, cor)   for blocks j in order
//       out = acc - 8 * cor (one rounding)
//   where dot_j is the integer dot of 32 4-bit codes with 32 8-bit input codes (exact, computed with dp4a).
// k_attn: decode attention for one (column, kv head): q/k RMSNorm, NEOX rotation, fp16 K/V write, scores, softmax,
//   P.V and the sigmoid gate, in the float order of seoul.cpp:425-453.
#include "common.cuh"

namespace imi {

// ---------------------------------------------------------------------------------------------------------------
// input preparation (prologues)
// ---------------------------------------------------------------------------------------------------------------

// cut `get(i)` (i < n) into 8-bit codes per 32 values; warps take blocks in turn
template <class Get>
__device__ __forceinline__ void cut_into(Get get, int n, int8_t *xq, float *xd, float *xs) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    for (int j = warp; j < n / 32; j += nw) {
        float d;
        int sum;
        const int q = warp_cut32(get(32 * j + lane), d, sum);
        xq[32 * j + lane] = (int8_t) q;
        if (lane == 0) {
            xd[j] = d;
            xs[j] = __fmul_rn(d, (float) sum);
        }
    }
}

// the word table row of `tok` as floats: d * (code - 8); codes of block j at bytes 16j.., scales after the codes
__device__ __forceinline__ float word_value(const uint8_t *row, int cols, int i) {
    const int j = i >> 5, k = i & 31;
    const uint8_t b = row[16 * j + (k & 15)];
    const int code = k < 16 ? (b & 15) : (b >> 4);
    const uint16_t dh = *(const uint16_t *) (row + cols / 2 + 2 * j);
    return __fmul_rn(h2f(dh), (float) (code - 8));
}

// x_new = x + norm(r) * w_post (imi_norm_mul_add, vec.h:41-44) into vb; r is staged in vb first
__device__ __forceinline__ void resid_add(float *vb, const float *r, const float *x, const float *wpost, int n,
                                          float eps, float *red, int c) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) vb[i] = r[i];
    __syncthreads();
    if ((threadIdx.x >> 5) == 0) {
        const float sc = warp_rms_scale(vb, n, eps);
        if (threadIdx.x == 0) red[c] = sc;
    }
    __syncthreads();
    const float sc = red[c];
    for (int i = threadIdx.x; i < n; i += blockDim.x) vb[i] = __fadd_rn(x[i], __fmul_rn(__fmul_rn(vb[i], sc), wpost[i]));
    __syncthreads();
}

template <int PRO, int NC>
__device__ void prologue(const MvArgs &a, const MvPlan &P, uint8_t *sm) {
    int8_t *xq = (int8_t *) (sm + P.xq);
    float *xd = (float *) (sm + P.xd), *xs = (float *) (sm + P.xs), *vb = (float *) (sm + P.vb);
    float *red = (float *) (sm + P.red);
    const int K = a.cols, nb = K / 32;
    const bool lead = blockIdx.x == 0;
    for (int c = 0; c < a.ncol; c++) {
        const Col col = a.cols_d[c];
        int8_t *q = xq + c * K;
        float *d = xd + c * nb, *s = xs + c * nb;
        float *v = vb + c * a.n_embd;
        if (PRO == P_CUT) {
            const float *in = a.in + (size_t) c * a.in_stride;
            cut_into([&](int i) { return in[i]; }, K, q, d, s);
        } else if (PRO == P_Q8IN) {
            for (int i = threadIdx.x; i < K; i += blockDim.x) q[i] = a.q8_q[(size_t) c * K + i];
            for (int j = threadIdx.x; j < nb; j += blockDim.x) {
                d[j] = a.q8_d[(size_t) c * nb + j];
                s[j] = a.q8_s[(size_t) c * nb + j];
            }
        } else if (PRO == P_CONV) {
            // seoul.cpp:410-414 (run) and 566-576 (run_batch): u = c * (b*x*w[d_conv] + sum_k st_k * w_k), st_k the
            // b*x of position p - d_conv + k: from this step's earlier columns of the same conversation when that
            // position is in this step, else from the conv memory ring.
            const int E = a.n_embd, R = a.d_conv + 1;
            const float *bcx = a.in + (size_t) c * a.in_stride;
            const int p = col.s->pos + col.off;
            const float *ring = col.ring + (size_t) a.conv_layer * R * E;
            for (int e = threadIdx.x; e < E; e += blockDim.x) {
                float u = __fmul_rn(__fmul_rn(bcx[e], bcx[2 * E + e]), a.conv_w[(size_t) a.d_conv * E + e]);
                for (int k = 0; k < a.d_conv; k++) {
                    const int qp = p - a.d_conv + k;
                    float st;
                    if (qp >= p - col.off) {
                        const float *ob = a.in + (size_t) (c - a.d_conv + k) * a.in_stride;
                        st = __fmul_rn(ob[e], ob[2 * E + e]);
                    } else {
                        st = ring[(size_t) (((qp % R) + R) % R) * E + e];
                    }
                    u = __fadd_rn(u, __fmul_rn(st, a.conv_w[(size_t) k * E + e]));
                }
                v[e] = __fmul_rn(u, bcx[E + e]);
            }
            __syncthreads();
            cut_into([&](int i) { return v[i]; }, K, q, d, s);
        } else {
            const int E = a.n_embd;
            if (PRO == P_EMBED_NORM) {
                int tok = col.token;
                if (tok == -2) tok = col.s->next_token;
                if (tok >= 0) {
                    const uint8_t *row = a.emb + (size_t) tok * a.emb_row_bytes;
                    for (int i = threadIdx.x; i < E; i += blockDim.x) v[i] = word_value(row, E, i);
                } else {
                    for (int i = threadIdx.x; i < E; i += blockDim.x) v[i] = col.embd[i];
                }
                __syncthreads();
            } else {   // P_RESID_NORM, P_FINAL
                resid_add(v, a.in + (size_t) c * a.in_stride, a.xin + (size_t) c * a.x_stride, a.wpost, E, a.eps, red,
                          c);
            }
            if (lead && a.xout)
                for (int i = threadIdx.x; i < E; i += blockDim.x) a.xout[(size_t) c * a.x_stride + i] = v[i];
            if ((threadIdx.x >> 5) == 0) {
                const float sc = warp_rms_scale(v, E, a.eps);
                if (threadIdx.x == 0) red[32 + c] = sc;
            }
            __syncthreads();
            const float sc = red[32 + c];
            const float *w = a.wpre;
            float *hid = (PRO == P_FINAL && lead) ? col.hid_out : nullptr;
            cut_into(
                [&](int i) {
                    const float h = __fmul_rn(__fmul_rn(v[i], sc), w[i]);
                    if (hid) hid[i] = h;
                    return h;
                },
                K, q, d, s);
        }
        __syncthreads();
    }
    // conv memory: the slot of each column's position takes b*x (seoul.cpp:419-423); written one launch after the
    // conv read it, so no CTA of the reading launch can see it early
    if (a.ring_layer >= 0 && lead) {
        const int E = a.n_embd, R = a.d_conv + 1;
        for (int c = 0; c < a.ncol; c++) {
            const Col col = a.cols_d[c];
            const int p = col.s->pos + col.off;
            const float *bcx = a.ring_src + (size_t) c * a.ring_src_stride;
            float *slot = col.ring + ((size_t) a.ring_layer * R + p % R) * E;
            for (int e = threadIdx.x; e < E; e += blockDim.x) slot[e] = __fmul_rn(bcx[e], bcx[2 * E + e]);
        }
    }
}

// ---------------------------------------------------------------------------------------------------------------
// k_table
// ---------------------------------------------------------------------------------------------------------------

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
    v = v + 0.0f;   // -0 -> +0: equal values compare equal, the lowest id wins
    const uint32_t b = __float_as_uint(v);
    const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long) o << 32) | (unsigned long long) (0xffffffffu - (uint32_t) idx);
}
__device__ __forceinline__ float amax_val(unsigned long long k) {
    const uint32_t o = (uint32_t) (k >> 32);
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}

template <int PRO, int EPI, int NC>
__global__ void __launch_bounds__(MV_THREADS, 1) k_table(const __grid_constant__ MvArgs a) {
    extern __shared__ __align__(128) uint8_t sm[];
    const int tid = threadIdx.x, K = a.cols, nb = K / 32, ld = nb + 1;
    const MvPlan P = mv_plan(K, a.sr, NC, (PRO == P_EMBED_NORM || PRO == P_RESID_NORM || PRO == P_FINAL ||
                                           PRO == P_CONV) ? a.n_embd : 0);
    uint8_t *stage = sm + P.stage;
    uint64_t *bar = (uint64_t *) (sm + P.bar);
    const int8_t *xq = (const int8_t *) (sm + P.xq);
    const float *xd = (const float *) (sm + P.xd), *xs = (const float *) (sm + P.xs);
    float *fs = (float *) (sm + P.fs), *dd = (float *) (sm + P.dd), *vo = (float *) (sm + P.vo);
    float *red = (float *) (sm + P.red);

    // rows of this CTA: whole units, split as evenly as the units allow
    const int units = a.rows / a.unit;
    const int u0 = (int) ((long long) units * blockIdx.x / gridDim.x),
              u1 = (int) ((long long) units * (blockIdx.x + 1) / gridDim.x);
    const int r0 = u0 * a.unit, nrows = (u1 - u0) * a.unit;
    const int nst = (nrows + a.sr - 1) / a.sr;

    if (tid == 0) {
        for (int b = 0; b < MV_STAGES; b++) mbar_init(&bar[b], 1);
        fence_barrier_init();
    }
    __syncthreads();
    auto issue = [&](int st) {
        const int rr = st * a.sr, n = min(a.sr, nrows - rr);
        const uint32_t bytes = (uint32_t) n * (uint32_t) a.row_bytes;
        uint64_t *b = &bar[st % MV_STAGES];
        mbar_expect_tx(b, bytes);
        bulk_g2s(stage + (st % MV_STAGES) * MV_STAGE_BYTES, a.W + (size_t) (r0 + rr) * a.row_bytes, bytes, b);
    };
    // weights do not depend on the previous launch: start them before waiting on it
    if (tid == 0)
        for (int st = 0; st < min(MV_STAGES, nst); st++) issue(st);
    pdl_trigger();
    pdl_wait();

    prologue<PRO, NC>(a, P, sm);

    // per-thread argmax of the word scores, per column
    unsigned long long best[NC];
#pragma unroll
    for (int c = 0; c < NC; c++) best[c] = 0ull;

    for (int st = 0; st < nst; st++) {
        const int buf = st % MV_STAGES;
        const bool ok = mbar_wait(&bar[buf], (uint32_t) ((st / MV_STAGES) & 1));
        if (!__syncthreads_and(ok)) {
            if (tid == 0) atomicExch(a.err, (int) 7);
            return;
        }
        const int rb = st * a.sr, nr = min(a.sr, nrows - rb);
        const uint8_t *sb = stage + buf * MV_STAGE_BYTES;
        // integer block dots of every (row, block) pair, all inputs; block scales as floats
        {
            int jc = -1;
            int xw[NC][8];
            for (int idx = tid; idx < nr * nb; idx += MV_THREADS) {
                const int r = idx / nb, j = idx - r * nb;
                if (j != jc) {
                    jc = j;
#pragma unroll
                    for (int c = 0; c < NC; c++) {
                        const int4 *xp = (const int4 *) (xq + c * K + 32 * j);
                        const int4 x0 = xp[0], x1 = xp[1];
                        xw[c][0] = x0.x; xw[c][1] = x0.y; xw[c][2] = x0.z; xw[c][3] = x0.w;
                        xw[c][4] = x1.x; xw[c][5] = x1.y; xw[c][6] = x1.z; xw[c][7] = x1.w;
                    }
                }
                const uint8_t *row = sb + (size_t) r * a.row_bytes;
                const uint4 code = *(const uint4 *) (row + 16 * j);
                dd[r * ld + j] = h2f(*(const uint16_t *) (row + K / 2 + 2 * j));
#pragma unroll
                for (int c = 0; c < NC; c++) {
                    if (c < a.ncol) {
                        const int s = dot_block(code, xw[c]);
                        fs[(c * a.sr + r) * ld + j] = __int2float_rn(s);
                        if (c == 0 && a.dots) a.dots[(size_t) (r0 + rb + r) * nb + j] = s;
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && st + MV_STAGES < nst) {   // every thread is done with this buffer
            fence_proxy_async();
            issue(st + MV_STAGES);
        }
        // the two fma chains per (input, row), blocks in order
        for (int t = tid; t < a.ncol * nr; t += MV_THREADS) {
            const int c = t / nr, r = t - c * nr;
            const float *f = fs + (c * a.sr + r) * ld, *dr = dd + r * ld, *xdc = xd + c * nb, *xsc = xs + c * nb;
            float acc = 0.0f, cor = 0.0f;
            for (int j = 0; j < nb; j++) {
                acc = __fmaf_rn(f[j], __fmul_rn(dr[j], xdc[j]), acc);
                cor = __fmaf_rn(dr[j], xsc[j], cor);
            }
            vo[c * a.sr + r] = __fmaf_rn(-8.0f, cor, acc);
        }
        __syncthreads();
        // epilogue
        if (EPI == E_STORE) {
            for (int t = tid; t < a.ncol * nr; t += MV_THREADS) {
                const int c = t / nr, r = t - c * nr;
                a.out[(size_t) c * a.out_stride + r0 + rb + r] = vo[c * a.sr + r];
            }
        } else if (EPI == E_SILU) {   // rows (2i, 2i+1) are (gate_i, up_i): act_i = silu(gate) * up (seoul.cpp:384-391)
            const int np = nr / 2;
            for (int t = tid; t < a.ncol * np; t += MV_THREADS) {
                const int c = t / np, i = t - c * np;
                const float g = vo[c * a.sr + 2 * i], u = vo[c * a.sr + 2 * i + 1];
                const float sl = __fdiv_rn(g, __fadd_rn(1.0f, exp_cr(-g)));
                a.out[(size_t) c * a.out_stride + (r0 + rb) / 2 + i] = __fmul_rn(sl, u);
            }
        } else {   // E_HEAD: word scores and the running first-maximum
            for (int t = tid; t < a.ncol * nr; t += MV_THREADS) {
                const int c = t / nr, r = t - c * nr;
                const float v = vo[c * a.sr + r];
                const int row = r0 + rb + r;
                float *lg = a.cols_d[c].logits;
                if (lg) lg[row] = v;
#pragma unroll
                for (int cc = 0; cc < NC; cc++)
                    if (cc == c) { const unsigned long long k = amax_key(v, row); best[cc] = k > best[cc] ? k : best[cc]; }
            }
        }
        // the next stage's integer phase rewrites fs/dd and the chain rewrites vo only after the sync above and the
        // one after its integer phase
    }

    if (EPI == E_HEAD) {
        unsigned long long *wbest = (unsigned long long *) (red + 64);
        const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
        for (int c = 0; c < NC; c++) {
            unsigned long long k = best[c];
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const unsigned long long v = __shfl_xor_sync(0xffffffffu, k, o);
                k = v > k ? v : k;
            }
            if (lane == 0) wbest[c * (MV_THREADS / 32) + warp] = k;
        }
        __syncthreads();
        if (tid < a.ncol) {
            unsigned long long k = 0;
            for (int w = 0; w < MV_THREADS / 32; w++) {
                const unsigned long long v = wbest[tid * (MV_THREADS / 32) + w];
                k = v > k ? v : k;
            }
            atomicMax(&a.cols_d[tid].s->amax, k);
        }
        __threadfence();
        __syncthreads();
        __shared__ int last;
        if (tid == 0) last = atomicAdd(a.done, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last && tid < a.ncol) {   // the step's end: the pick, the new position, counters reset
            __threadfence();
            const Col col = a.cols_d[tid];
            const unsigned long long k = atomicExch(&col.s->amax, 0ull);
            const int id = (int) (0xffffffffu - (uint32_t) (k & 0xffffffffu));
            col.s->next_token = id;
            col.s->amax_val = amax_val(k);
            if (col.picks) col.picks[col.s->pos + col.off] = id;
            col.s->pos += col.pos_inc;
        }
        if (last && tid == 0) *a.done = 0;
    }
}

// ---------------------------------------------------------------------------------------------------------------
// k_final: the last post-norm and the output norm without word scores (seoul.cpp:473-477), one CTA per column;
// ends the step (position update)
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_final(const __grid_constant__ FinalArgs a) {
    extern __shared__ __align__(16) uint8_t smf[];
    float *v = (float *) smf, *red = v + a.n_embd;
    pdl_trigger();
    pdl_wait();
    const int c = blockIdx.x, E = a.n_embd;
    const Col col = a.cols_d[c];
    resid_add(v, a.in + (size_t) c * a.in_stride, a.xin + (size_t) c * a.x_stride, a.wpost, E, a.eps, red, 0);
    if ((threadIdx.x >> 5) == 0) {
        const float sc = warp_rms_scale(v, E, a.eps);
        if (threadIdx.x == 0) red[1] = sc;
    }
    __syncthreads();
    const float sc = red[1];
    if (col.hid_out)
        for (int i = threadIdx.x; i < E; i += blockDim.x) col.hid_out[i] = __fmul_rn(__fmul_rn(v[i], sc), a.out_norm[i]);
    __syncthreads();
    if (threadIdx.x == 0) col.s->pos += col.pos_inc;
}

// ---------------------------------------------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------------------------------------------

// k RMSNorm + NEOX rotation of one head vector held in shared memory (seoul.cpp:19-28,435-436 / 442-443), in place
template <int D>
__device__ __forceinline__ void norm_rope(float *x, const float *w, const float *cs, const float *sn, float eps,
                                          float *tmp) {
    // executed by one warp
    const float sc = warp_rms_scale(x, D, eps);
    const int L = threadIdx.x & 31;
    for (int i = L; i < D; i += 32) tmp[i] = __fmul_rn(__fmul_rn(x[i], sc), w[i]);
    __syncwarp();
    for (int i = L; i < D / 2; i += 32) {
        const float x0 = tmp[i], x1 = tmp[i + D / 2];
        x[i] = __fsub_rn(__fmul_rn(x0, cs[i]), __fmul_rn(x1, sn[i]));
        x[i + D / 2] = __fadd_rn(__fmul_rn(x0, sn[i]), __fmul_rn(x1, cs[i]));
    }
    __syncwarp();
}

// fp16 K and V of one position for kv head g (written to the caches)
template <int D>
__device__ __forceinline__ void kv_make(const AttnArgs &a, const float *qkv, int g, int p, float *ktmp, float *tmp,
                                        uint16_t *kh, uint16_t *vh) {
    const int H = a.n_head, kvd = a.n_head_kv * D;
    if ((threadIdx.x >> 5) == 0) {
        for (int i = threadIdx.x; i < D; i += 32) ktmp[i] = qkv[H * D + g * D + i];
        __syncwarp();
        norm_rope<D>(ktmp, a.k_norm, a.rope_cs + (size_t) p * (D / 2), a.rope_sn + (size_t) p * (D / 2), a.eps, tmp);
        for (int i = threadIdx.x; i < D; i += 32) {
            kh[i] = f2h(ktmp[i]);
            vh[i] = f2h(qkv[H * D + kvd + g * D + i]);
        }
    }
}

// K/V of every column's position, before a chunk's attention reads them (prefill: run_batch, seoul.cpp:592-600)
template <int D>
__global__ void __launch_bounds__(32) k_kvwrite(const __grid_constant__ AttnArgs a) {
    __shared__ float ktmp[D], tmp[D];
    __shared__ uint16_t kh[D], vh[D];
    pdl_trigger();
    pdl_wait();
    const int g = blockIdx.x, c = blockIdx.y, kvd = a.n_head_kv * D;
    const Col col = a.cols_d[c];
    const int p = col.s->pos + col.off;
    kv_make<D>(a, a.qkv + (size_t) c * a.qkv_stride, g, p, ktmp, tmp, kh, vh);
    __syncwarp();
    const size_t o = ((size_t) a.ai * a.n_ctx + p) * kvd + g * D;
    for (int i = threadIdx.x; i < D; i += 32) {
        ((uint16_t *) col.kc)[o + i] = kh[i];
        ((uint16_t *) col.vc)[o + i] = vh[i];
    }
}

// one CTA per (kv head g, column): the GRP query heads of the group, GRP*D threads
template <int D, int GRP>
__global__ void __launch_bounds__(GRP *D) k_attn(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) uint8_t sma[];
    float *q = (float *) sma;                    // [GRP][D]
    float *ktmp = q + GRP * D, *tmp = ktmp + D;  // [D], [D]
    float *mx = tmp + D;                         // [GRP]
    float *inv = mx + GRP;                       // [GRP]
    double *dsum = (double *) (inv + GRP + (GRP & 1 ? 1 : 0));   // [GRP][nwarps]
    float *wmax = (float *) (dsum + GRP * (GRP * D / 32));     // [GRP][nwarps]
    uint16_t *kh = (uint16_t *) (wmax + GRP * (GRP * D / 32)); // [D]
    uint16_t *vh = kh + D;                                      // [D]
    float *sc = (float *) (vh + D + (D & 1 ? 1 : 0));            // [GRP][n_ctx]
    constexpr int NT = GRP * D, NW = NT / 32;

    pdl_trigger();
    pdl_wait();
    const int g = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = a.n_head, kvd = a.n_head_kv * D;
    const Col col = a.cols_d[c];
    const int p = col.s->pos + col.off;
    const float *qkv = a.qkv + (size_t) c * a.qkv_stride;
    const float *cs = a.rope_cs + (size_t) p * (D / 2), *sn = a.rope_sn + (size_t) p * (D / 2);
    const uint16_t *kc = (const uint16_t *) col.kc + (size_t) a.ai * a.n_ctx * kvd + g * D;
    const uint16_t *vc = (const uint16_t *) col.vc + (size_t) a.ai * a.n_ctx * kvd + g * D;

    // this position's K and V (written to the caches here when fused)
    if (a.kv_fused) {
        kv_make<D>(a, qkv, g, p, ktmp, tmp, kh, vh);
        __syncthreads();
        if (tid < D) {
            ((uint16_t *) kc)[(size_t) p * kvd + tid] = kh[tid];
            ((uint16_t *) vc)[(size_t) p * kvd + tid] = vh[tid];
        }
    }
    // the group's queries: RMSNorm + rotation, one warp per head (seoul.cpp:442-443)
    for (int hh = warp; hh < GRP; hh += NW) {
        float *qh = q + hh * D;
        const int h = g * GRP + hh;
        for (int i = lane; i < D; i += 32) qh[i] = qkv[h * D + i];
        __syncwarp();
        float *t2 = (float *) (sc + (size_t) hh * a.n_ctx);   // scratch: the head's score row is free yet
        norm_rope<D>(qh, a.q_norm, cs, sn, a.eps, t2);
    }
    __syncthreads();

    const int s0 = a.window > 0 ? max(0, p - a.window + 1) : 0, nk = p - s0 + 1;
    // scores (seoul.cpp:445): one thread per position, all GRP heads
    float lmax[GRP];
#pragma unroll
    for (int hh = 0; hh < GRP; hh++) lmax[hh] = -INFINITY;
    for (int t = tid; t < nk; t += NT) {
        const int pt = s0 + t;
        uint4 kr[D / 8];
        if (a.kv_fused && pt == p) {
#pragma unroll
            for (int w = 0; w < D / 8; w++) kr[w] = ((const uint4 *) kh)[w];
        } else {
            const uint4 *src = (const uint4 *) (kc + (size_t) pt * kvd);
#pragma unroll
            for (int w = 0; w < D / 8; w++) kr[w] = src[w];
        }
#pragma unroll
        for (int hh = 0; hh < GRP; hh++) {
            const float s = __fmul_rn(dot_h8<D>(q + hh * D, kr), a.scale);
            sc[(size_t) hh * a.n_ctx + t] = s;
            lmax[hh] = lmax[hh] < s ? s : lmax[hh];
        }
    }
#pragma unroll
    for (int hh = 0; hh < GRP; hh++) {
        float m = lmax[hh];
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[hh * NW + warp] = m;
    }
    __syncthreads();
    if (tid < GRP) {
        float m = -INFINITY;
        for (int w = 0; w < NW; w++) m = fmaxf(m, wmax[tid * NW + w]);
        mx[tid] = m;
    }
    __syncthreads();
    // exp and the double sum (seoul.cpp:446-448)
    double lsum[GRP];
#pragma unroll
    for (int hh = 0; hh < GRP; hh++) lsum[hh] = 0.0;
    for (int t = tid; t < nk; t += NT) {
#pragma unroll
        for (int hh = 0; hh < GRP; hh++) {
            float *sp = sc + (size_t) hh * a.n_ctx + t;
            const float e = exp_cr(__fsub_rn(*sp, mx[hh]));
            *sp = e;
            lsum[hh] += (double) e;
        }
    }
#pragma unroll
    for (int hh = 0; hh < GRP; hh++) {
        double s = lsum[hh];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) dsum[hh * NW + warp] = s;
    }
    __syncthreads();
    if (tid < GRP) {
        double s = 0.0;
        for (int w = 0; w < NW; w++) s += dsum[tid * NW + w];
        inv[tid] = __double2float_rn(1.0 / s);
    }
    __syncthreads();
    for (int t = tid; t < nk; t += NT) {
#pragma unroll
        for (int hh = 0; hh < GRP; hh++) {
            float *sp = sc + (size_t) hh * a.n_ctx + t;
            *sp = __fmul_rn(*sp, inv[hh]);
        }
    }
    __syncthreads();
    // P.V (seoul.cpp:449-450): o_i = fma(p_t, v_t,i, o_i) over positions in order; thread (head, i)
    {
        const int hh = tid / D, i = tid - hh * D;
        const float *pr = sc + (size_t) hh * a.n_ctx;
        const int ng = (a.kv_fused && s0 + nk - 1 == p) ? nk - 1 : nk;   // positions read from the cache
        const uint16_t *vp = vc + (size_t) s0 * kvd + i;
        float o = 0.0f;
        int t = 0;
        for (; t + 8 <= ng; t += 8) {
            uint16_t v8[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v8[u] = vp[(size_t) (t + u) * kvd];
#pragma unroll
            for (int u = 0; u < 8; u++) o = __fmaf_rn(pr[t + u], h2f(v8[u]), o);
        }
        for (; t < ng; t++) o = __fmaf_rn(pr[t], h2f(vp[(size_t) t * kvd]), o);
        if (ng < nk) o = __fmaf_rn(pr[nk - 1], h2f(vh[i]), o);
        const int h = g * GRP + hh;
        const float gv = qkv[H * D + 2 * kvd + h];
        const float gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-gv)));   // seoul.cpp:451
        a.att[(size_t) c * a.att_stride + h * D + i] = __fmul_rn(o, gate);
    }
}

__host__ __device__ inline size_t attn_smem_bytes(int D, int GRP, int n_ctx) {
    const int NW = GRP * D / 32;
    size_t o = 4 * (size_t) (GRP * D + 2 * D + 2 * GRP + (GRP & 1 ? 1 : 0));
    o += 8 * (size_t) GRP * NW + 4 * (size_t) GRP * NW + 2 * (size_t) (2 * D + (D & 1 ? 1 : 0));
    o = (o + 15) / 16 * 16;
    o += 4 * (size_t) GRP * n_ctx;
    return o;
}

// ---------------------------------------------------------------------------------------------------------------
// known-answer helper: the 8-bit cut of a vector
// ---------------------------------------------------------------------------------------------------------------
__global__ void k_q8_cut(const float *x, int n, int8_t *q, float *d, float *s) {
    const int lane = threadIdx.x & 31, j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (j >= n / 32) return;   // whole warps only: n / 32 blocks, warp-uniform
    float dd;
    int sum;
    const int qq = warp_cut32(x[32 * j + lane], dd, sum);
    q[32 * j + lane] = (int8_t) qq;
    if (lane == 0) {
        d[j] = dd;
        s[j] = __fmul_rn(dd, (float) sum);
    }
}

}  // namespace imi

#include "launch.inc"

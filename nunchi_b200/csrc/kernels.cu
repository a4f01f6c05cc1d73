// sm_100a kernels of the decode engine.
//
// k_table (table.cuh): the 4-bit table reads with the small math of imi's step folded in.
// k_attn: decode attention for one (column, kv head): q/k RMSNorm, NEOX rotation, fp16 K/V write, scores, softmax,
//   P.V and the sigmoid gate, in the float order of seoul.cpp:425-453.
#include "common.cuh"
#include "table.cuh"

namespace imi {

// ---------------------------------------------------------------------------------------------------------------
// input preparation (prologues)
// ---------------------------------------------------------------------------------------------------------------

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

// ---------------------------------------------------------------------------------------------------------------
// k_final: the last post-norm and the output norm without word scores (seoul.cpp:473-477), one CTA per column;
// ends the step (position update)
// ---------------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_final(const __grid_constant__ FinalArgs a) {
    extern __shared__ __align__(16) uint8_t smf[];
    float *v = (float *) smf, *red = v + a.n_embd;
    unsigned long long *trace = a.trace ? a.trace + (size_t) blockIdx.x * MV_TRACE : nullptr;
    if (trace && threadIdx.x == 0) trace[0] = global_ns();
    pdl_trigger();
    pdl_wait();
    if (trace && threadIdx.x == 0) trace[1] = global_ns();
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
    if (threadIdx.x == 0 && col.pos_inc) atomicAdd(&col.s->pos, col.pos_inc);   // several columns may share a conversation
    if (trace && threadIdx.x == 0) trace[14] = global_ns();
}

// ---------------------------------------------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------------------------------------------

// shared-memory plan of k_attn (host and device agree on it); every region 16-byte aligned
struct AttnPlan {
    size_t q, qtmp, ktmp, tmp, mx, inv, dsum, wmax, kh, vh, sc, total;
};
__host__ __device__ inline AttnPlan attn_plan(int D, int GRP, int n_ctx) {
    AttnPlan p;
    const int NW = GRP * D / 32;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 15) / 16 * 16; return r; };
    p.q = take(4 * (size_t) GRP * D);
    p.qtmp = take(4 * (size_t) GRP * D);
    p.ktmp = take(4 * (size_t) D);
    p.tmp = take(4 * (size_t) D);
    p.mx = take(4 * (size_t) GRP);
    p.inv = take(4 * (size_t) GRP);
    p.dsum = take(8 * (size_t) GRP * NW);
    p.wmax = take(4 * (size_t) GRP * NW);
    p.kh = take(2 * (size_t) D);
    p.vh = take(2 * (size_t) D);
    p.sc = take(4 * (size_t) GRP * n_ctx);
    p.total = o;
    return p;
}

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
    constexpr int NT = GRP * D, NW = NT / 32;
    const AttnPlan L = attn_plan(D, GRP, a.n_ctx);
    unsigned long long *trace = a.trace ? a.trace + (size_t) (blockIdx.y * gridDim.x + blockIdx.x) * MV_TRACE : nullptr;
    if (trace && threadIdx.x == 0) trace[0] = global_ns();
    float *q = (float *) (sma + L.q);          // [GRP][D] rotated queries
    float *qtmp = (float *) (sma + L.qtmp);    // [GRP][D] norm scratch per head
    float *ktmp = (float *) (sma + L.ktmp), *tmp = (float *) (sma + L.tmp);   // [D], [D]
    float *mx = (float *) (sma + L.mx), *inv = (float *) (sma + L.inv);       // [GRP]
    double *dsum = (double *) (sma + L.dsum);  // [GRP][NW]
    float *wmax = (float *) (sma + L.wmax);    // [GRP][NW]
    uint16_t *kh = (uint16_t *) (sma + L.kh), *vh = (uint16_t *) (sma + L.vh);   // [D] fp16 (16-byte aligned)
    float *sc = (float *) (sma + L.sc);        // [GRP][n_ctx] scores, then probabilities

    pdl_trigger();
    pdl_wait();
    const int g = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (trace && tid == 0) trace[1] = global_ns();
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
        norm_rope<D>(qh, a.q_norm, cs, sn, a.eps, qtmp + hh * D);
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
        const float y = __fmul_rn(o, gate);
        a.att[(size_t) c * a.att_stride + h * D + i] = y;
        qtmp[hh * D + i] = y;
    }
    // the 8-bit cut of this group's output blocks (imi_cut32 of seoul.cpp:457), so the o table only loads codes
    if (trace && tid == 0) trace[13] = global_ns();
    if (a.q8o_q) {
        __syncthreads();
        const int HD = H * D;
        for (int t = tid; t < GRP * D / 32; t += NT) {
            float v[32];
            load32(qtmp + 32 * t, v);
            const int blk = g * GRP * D / 32 + t;
            cut32(v, a.q8o_q + (size_t) c * HD + 32 * blk, a.q8o_d + (size_t) c * (HD / 32) + blk,
                  a.q8o_s + (size_t) c * (HD / 32) + blk);
        }
    }
    if (trace && tid == 0) trace[14] = global_ns();
}

__host__ __device__ inline size_t attn_smem_bytes(int D, int GRP, int n_ctx) { return attn_plan(D, GRP, n_ctx).total; }

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

// GGUF Q4_0 rows (blocks of 18 bytes: fp16 scale, then 16 code bytes) into the table kernel's row layout
// [cols/2 code bytes | cols/32 fp16 scales]; one thread per block, byte copies (GGUF blocks are only 2-byte aligned)
__global__ void k_q4_repack(const uint8_t *src, int rows, int nb, uint8_t *dst) {
    const size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t) rows * nb) return;
    const size_t r = i / nb;
    const int j = (int) (i - r * nb);
    const uint8_t *b = src + i * 18;
    uint8_t *row = dst + r * (size_t) nb * 18;
#pragma unroll
    for (int k = 0; k < 16; k++) row[16 * j + k] = b[2 + k];
    row[(size_t) nb * 16 + 2 * j] = b[0];
    row[(size_t) nb * 16 + 2 * j + 1] = b[1];
}

}  // namespace imi

#include "launch.inc"

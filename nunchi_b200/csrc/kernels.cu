// sm_100a kernels of the decode engine.
//
// k_table (table.cuh): the 4-bit table reads with the small math of imi's step folded in.
// k_attn: decode attention for one (query head, column): q/k RMSNorm, NEOX rotation, fp16 K/V write, scores,
//   softmax, P.V and the sigmoid gate, in the float order of seoul.cpp:425-453.
#define IMI_KERNELS 1
#include <cuda.h>

#include "common.cuh"
#include "table.cuh"
#include "tc_table.cuh"
#include "tc_prep.cuh"

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

// imi_q8k::from of one 256-value block by one warp (lane L: values 8L..8L+7): amax, d = amax/127, id = d ? 1/d : 0,
// codes round-half-even(x * id), the code sum of every 16 values (tables.cpp:200-213)
__device__ __forceinline__ void q8k_block(const float *x, int lane, int8_t *q, float *d, int16_t *bsums) {
    const float *v = x + 8 * lane;
    float a[8], amax = 0.0f;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        a[u] = v[u];
        amax = fmaxf(amax, fabsf(a[u]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = __fdiv_rn(amax, 127.0f), id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    int s = 0;
#pragma unroll
    for (int u = 0; u < 8; u++) {
        const int c = __float2int_rn(__fmul_rn(a[u], id));
        q[8 * lane + u] = (int8_t) c;
        s += c;
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);   // lanes 2m, 2m+1 hold the 16 values of sum m
    if ((lane & 1) == 0) bsums[lane / 2] = (int16_t) s;
    if (lane == 0) *d = dd;
}

// k_final: the last post-norm and the output norm without word scores (seoul.cpp:473-477), one CTA per column;
// ends the step (position update). With a Q6_K word table it also cuts the hidden state per 256 values for the
// word-score launch that follows (k_q6k_head), which then ends the step.
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
    if (a.q8k_q) {   // Q6_K word table: keep the hidden state, cut it per 256 values (one warp per block)
        __syncthreads();
        for (int i = threadIdx.x; i < E; i += blockDim.x) {
            v[i] = __fmul_rn(__fmul_rn(v[i], sc), a.out_norm[i]);
            if (col.hid_out) col.hid_out[i] = v[i];
        }
        __syncthreads();
        const int lane = threadIdx.x & 31;
        for (int j = threadIdx.x >> 5; j < E / 256; j += blockDim.x >> 5)
            q8k_block(v + 256 * j, lane, a.q8k_q + (size_t) c * E + 256 * j, a.q8k_d + (size_t) c * (E / 256) + j,
                      a.q8k_b + (size_t) c * (E / 16) + 16 * j);
        if (trace && threadIdx.x == 0) trace[14] = global_ns();
        return;   // the word-score launch advances the position after its pick
    }
    if (col.hid_out)
        for (int i = threadIdx.x; i < E; i += blockDim.x) col.hid_out[i] = __fmul_rn(__fmul_rn(v[i], sc), a.out_norm[i]);
    __syncthreads();
    if (threadIdx.x == 0 && col.pos_inc) atomicAdd(&col.s->pos, col.pos_inc);   // several columns may share a conversation
    if (trace && threadIdx.x == 0) trace[14] = global_ns();
}

// ---------------------------------------------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------------------------------------------

// k_attn: one CTA of ATT_NT threads per (query head, column). The cached V rows the P.V chain reads arrive in shared
// memory in tiles of 64 KB (two in flight, cp.async), issued before the scores so the copies overlap them.
constexpr int ATT_NT = 128, ATT_NW = ATT_NT / 32;
__host__ __device__ inline int attn_vtile(int D) { return 32768 / D; }   // positions per V tile (64 KB of fp16)
// shared-memory plan of k_attn (host and device agree on it); every region 16-byte aligned
struct AttnPlan {
    size_t q, ktmp, tmp, y, kh, vh, rcs, rsn, red, vt, sc, total;
};
__host__ __device__ inline AttnPlan attn_plan(int D, int n_ctx) {
    AttnPlan p;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 15) / 16 * 16; return r; };
    p.q = take(4 * (size_t) D);
    p.ktmp = take(4 * (size_t) D);
    p.tmp = take(4 * (size_t) D);
    p.y = take(4 * (size_t) D);
    p.kh = take(2 * (size_t) D);
    p.vh = take(2 * (size_t) D);
    p.rcs = take(4 * (size_t) D / 2);
    p.rsn = take(4 * (size_t) D / 2);
    p.red = take(8 * ATT_NW + 4 * ATT_NW + 16);
    p.vt = take(2 * (size_t) attn_vtile(D) * D * 2);
    p.sc = take(4 * (size_t) n_ctx);
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
    const int g = blockIdx.x, c = blockIdx.y;
    const Col col = a.cols_d[c];
    const int p = col.s->pos + col.off;
    kv_make<D>(a, a.qkv + (size_t) c * a.qkv_stride, g, p, ktmp, tmp, kh, vh);
    __syncwarp();
    const size_t o = (((size_t) a.ai * a.n_head_kv + g) * a.n_ctx + p) * D;   // caches [layer][kv head][position][D]
    for (int i = threadIdx.x; i < D; i += 32) {
        ((uint16_t *) col.kc)[o + i] = kh[i];
        ((uint16_t *) col.vc)[o + i] = vh[i];
    }
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait_group() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// decode / prefill attention of query head h for column c (seoul.cpp:425-453 and 589-621): q RMSNorm + rotation,
// this position's K/V (decode: made here and written to the caches by the group's first head), scores by dot_h,
// softmax with a double sum, the serial P.V chain over positions in order, the sigmoid gate, and the 8-bit cut of
// the head's output blocks for the o table.
template <int D>
__global__ void __launch_bounds__(ATT_NT) k_attn(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(16) uint8_t sma[];
    const AttnPlan L = attn_plan(D, a.n_ctx);
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *trace = a.trace ? a.trace + (size_t) (blockIdx.y * gridDim.x + blockIdx.x) * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    float *q = (float *) (sma + L.q), *ktmp = (float *) (sma + L.ktmp), *tmp = (float *) (sma + L.tmp);
    float *y = (float *) (sma + L.y), *sc = (float *) (sma + L.sc);
    uint16_t *kh = (uint16_t *) (sma + L.kh), *vh = (uint16_t *) (sma + L.vh), *vt = (uint16_t *) (sma + L.vt);
    double *dsum = (double *) (sma + L.red);
    float *wmax = (float *) (sma + L.red + 8 * ATT_NW), *mx = wmax + ATT_NW, *inv = mx + 1;

    float *rcs = (float *) (sma + L.rcs), *rsn = (float *) (sma + L.rsn);
    pdl_trigger();
    const int H = a.n_head, grp = H / a.n_head_kv, g = h / grp, kvd = a.n_head_kv * D;
    const Col col = a.cols_d[c];
    // the rotary rows of the position read now (it changes only at the end of a step; checked again after the wait)
    const int pspec = ld_relaxed(&col.s->pos) + col.off;
    for (int i = tid; i < D / 2; i += ATT_NT) {
        rcs[i] = a.rope_cs[(size_t) pspec * (D / 2) + i];
        rsn[i] = a.rope_sn[(size_t) pspec * (D / 2) + i];
    }
    if (tid == 0) {   // before the wait: this CTA's share of its kv head's cached K and V rows into L2 (a hint only:
                      // the position read here may be one behind; the rows before it are final)
        const int pp = ld_relaxed(&col.s->pos) + col.off, ps = a.window > 0 ? max(0, pp - a.window + 1) : 0;
        const size_t row = (size_t) D * 2, bytes = (size_t) max(pp - ps, 0) * row, hb = ((size_t) a.ai * a.n_head_kv + g) * a.n_ctx;
        const size_t share = (bytes / grp + 15) / 16 * 16, b0 = (size_t) (h % grp) * share, b1 = min(b0 + share, bytes);
        const uint8_t *kb = (const uint8_t *) col.kc + (hb + ps) * row;
        const uint8_t *vb0 = (const uint8_t *) col.vc + (hb + ps) * row;
        for (size_t o = b0; o < b1; o += 65536) {
            const uint32_t n = (uint32_t) min((size_t) 65536, b1 - o);
            prefetch_l2(kb + o, n);
            prefetch_l2(vb0 + o, n);
        }
    }
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    const int p = ld_relaxed(&col.s->pos) + col.off;
    const float *qkv = a.qkv + (size_t) c * a.qkv_stride;
    const float *cs = rcs, *sn = rsn;
    if (p != pspec) {   // the position moved since the rows were read: the table rows themselves
        cs = a.rope_cs + (size_t) p * (D / 2);
        sn = a.rope_sn + (size_t) p * (D / 2);
    }
    // this kv head's rows of the layer: [position][D] (caches [layer][kv head][position][D])
    uint16_t *kc = (uint16_t *) col.kc + ((size_t) a.ai * a.n_head_kv + g) * a.n_ctx * D;
    uint16_t *vc = (uint16_t *) col.vc + ((size_t) a.ai * a.n_head_kv + g) * a.n_ctx * D;
    const int s0 = a.window > 0 ? max(0, p - a.window + 1) : 0, nk = p - s0 + 1;
    const int ng = a.kv_fused ? nk - 1 : nk;   // positions whose V is read from the cache
    const int VT = attn_vtile(D), ntile = (ng + VT - 1) / VT;
    auto load_tile = [&](int k) {   // by warps 2.., idle while warps 0 and 1 make this position's K, V and query
        if (warp < 2) return;
        uint16_t *dst = vt + (size_t) (k & 1) * VT * D;
        const int t0 = k * VT, n = min(VT, ng - t0);
        for (int i = tid - 64; i < n * (D / 8); i += ATT_NT - 64) {
            const int t = i / (D / 8), ch = i - t * (D / 8);
            cp16(dst + (size_t) t * D + 8 * ch, vc + (size_t) (s0 + t0 + t) * D + 8 * ch);
        }
        cp_commit();
    };
    __syncthreads();   // the rotary rows are in shared memory
    // the cached V rows into shared memory while the rest of the setup and the scores run
    if (ntile > 0) load_tile(0);
    if (ntile > 1) load_tile(1);

    // this position's K and V (warp 0) and the rotated query (warp 1)
    if (a.kv_fused) kv_make<D>(a, qkv, g, p, ktmp, tmp, kh, vh);
    if (warp == 1) {
        for (int i = lane; i < D; i += 32) q[i] = qkv[h * D + i];
        __syncwarp();
        norm_rope<D>(q, a.q_norm, cs, sn, a.eps, y);
    }
    __syncthreads();
    if (a.kv_fused && h % grp == 0 && tid < D) {
        kc[(size_t) p * D + tid] = kh[tid];
        vc[(size_t) p * D + tid] = vh[tid];
    }

    // scores (seoul.cpp:445): one thread per position
    float lmax = -INFINITY;
    constexpr int SB = D == 64 ? 4 : 2;   // positions per thread whose K rows are loaded together
    for (int t0 = tid; t0 < nk; t0 += SB * ATT_NT) {
        uint4 kr[SB][D / 8];
#pragma unroll
        for (int u = 0; u < SB; u++) {
            const int t = t0 + u * ATT_NT, pt = s0 + t;
            if (t < nk) {
                const uint4 *src = (a.kv_fused && pt == p) ? (const uint4 *) kh : (const uint4 *) (kc + (size_t) pt * D);
#pragma unroll
                for (int w = 0; w < D / 8; w++) kr[u][w] = src[w];
            }
        }
#pragma unroll
        for (int u = 0; u < SB; u++) {
            const int t = t0 + u * ATT_NT;
            if (t < nk) {
                const float v = __fmul_rn(dot_h8<D>(q, kr[u]), a.scale);
                sc[t] = v;
                lmax = lmax < v ? v : lmax;
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) wmax[warp] = lmax;
    __syncthreads();
    float m = wmax[0];
    for (int w = 1; w < ATT_NW; w++) m = fmaxf(m, wmax[w]);
    // exp and the double sum (seoul.cpp:446-448)
    double ls = 0.0;
    for (int t = tid; t < nk; t += ATT_NT) {
        const float e = exp_cr(__fsub_rn(sc[t], m));
        sc[t] = e;
        ls += (double) e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane == 0) dsum[warp] = ls;
    __syncthreads();
    if (tid == 0) {
        double t = 0.0;
        for (int w = 0; w < ATT_NW; w++) t += dsum[w];
        *inv = __double2float_rn(1.0 / t);
    }
    __syncthreads();
    const float iv = *inv;
    for (int t = tid; t < nk; t += ATT_NT) sc[t] = __fmul_rn(sc[t], iv);

    // P.V (seoul.cpp:449-450): o_i = fma(p_t, v_t,i, o_i) over positions in order; thread i < D owns dimension i
    float o = 0.0f;
    for (int k = 0; k < ntile; k++) {
        if (k + 1 < ntile) cp_wait_group<1>();
        else cp_wait_group<0>();
        __syncthreads();
        if (tid < D) {
            const uint16_t *vb = vt + (size_t) (k & 1) * VT * D + tid;
            const float *pr = sc + (size_t) k * VT;
            const int n = min(VT, ng - k * VT);
            int t = 0;
#pragma unroll 4
            for (; t + 8 <= n; t += 8) {
                uint16_t v8[8];
#pragma unroll
                for (int u = 0; u < 8; u++) v8[u] = vb[(size_t) (t + u) * D];
                const float4 p0 = *(const float4 *) (pr + t), p1 = *(const float4 *) (pr + t + 4);
                o = __fmaf_rn(p0.x, h2f(v8[0]), o);
                o = __fmaf_rn(p0.y, h2f(v8[1]), o);
                o = __fmaf_rn(p0.z, h2f(v8[2]), o);
                o = __fmaf_rn(p0.w, h2f(v8[3]), o);
                o = __fmaf_rn(p1.x, h2f(v8[4]), o);
                o = __fmaf_rn(p1.y, h2f(v8[5]), o);
                o = __fmaf_rn(p1.z, h2f(v8[6]), o);
                o = __fmaf_rn(p1.w, h2f(v8[7]), o);
            }
            for (; t < n; t++) o = __fmaf_rn(pr[t], h2f(vb[(size_t) t * D]), o);
        }
        __syncthreads();
        if (k + 2 < ntile) load_tile(k + 2);
    }
    if (tid < D) {
        if (ng < nk) o = __fmaf_rn(sc[nk - 1], h2f(vh[tid]), o);   // this position's own V
        const float gv = qkv[H * D + 2 * kvd + h];
        const float gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-gv)));   // seoul.cpp:451
        const float yv = __fmul_rn(o, gate);
        a.att[(size_t) c * a.att_stride + h * D + tid] = yv;
        y[tid] = yv;
    }
    __syncthreads();
    // the 8-bit cut of this head's output blocks (imi_cut32 of seoul.cpp:457), so the o table only loads codes
    if (a.q8o_q && warp == 0) {
        const int HD = H * D;
        for (int q0 = 0; q0 < D / 4; q0 += 32) {
            const int qi = q0 + lane;
            const bool act = qi < D / 4;
            const float4 v = act ? ((const float4 *) y)[qi] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            cut_chunk(v, act, qi, a.q8o_q + (size_t) c * HD + h * D, a.q8o_d + (size_t) c * (HD / 32) + h * D / 32,
                      a.q8o_s + (size_t) c * (HD / 32) + h * D / 32);
        }
    }
    if (trace && tid == 0) trace[14] = global_ns();
}

__host__ __device__ inline size_t attn_smem_bytes(int D, int n_ctx) { return attn_plan(D, n_ctx).total; }

// k_attn_tma: the same attention (one CTA per query head and column, k_attn's float order) at head_dim 64, with the
// head's cached K and V streamed into shared memory by the copy engine instead of per-thread loads (the caches are
// head-major, so a head's rows are contiguous). One ring of ns slots of ATK_T positions (32 KB) carries the head's K
// tiles and then its V tiles: tile i sits in slot i % ns, the first ns tiles are issued at once and tile i + ns as
// soon as tile i is consumed, so at the lengths decode runs at the whole K and most of V are in flight from the start.
// Large copies matter: a CTA completes about one copy every 0.28 us whatever its size up to 32 KB.
// Both come by 2D tensor copies with the 128-byte swizzle (chunk w of row r lands at chunk position w ^ (r & 7), so
// one thread per position reading chunk w of its row hits distinct banks; the P.V threads read V by the same rule).
// The session's K and V tensor maps sit ATK_TMAP_OFF bytes into its device record (written when the conversation is
// made).
struct AttkPlan {
    size_t q, kf, vf, tq, tk, wq, wk, y, kh, vh, rcs, rsn, red, bar, sc, total;
    int ns;   // ring slots (the ring starts at the 1024-byte aligned base)
};
__host__ __device__ inline AttkPlan attk_layout(int n_ctx, int ns) {
    AttkPlan p;
    p.ns = ns;
    size_t o = (size_t) ns * ATK_TILE;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 15) / 16 * 16; return r; };
    p.q = take(4 * ATK_D);
    p.kf = take(4 * ATK_D);
    p.vf = take(4 * ATK_D);
    p.tq = take(4 * ATK_D);
    p.tk = take(4 * ATK_D);
    p.wq = take(4 * ATK_D);
    p.wk = take(4 * ATK_D);
    p.y = take(4 * ATK_D);
    p.kh = take(2 * ATK_D);
    p.vh = take(2 * ATK_D);
    p.rcs = take(4 * ATK_D / 2);
    p.rsn = take(4 * ATK_D / 2);
    p.red = take(8 * ATK_NW + 4 * ATK_NW + 16);
    p.bar = take(8 * ATK_NSMAX);
    p.sc = take(4 * (size_t) n_ctx);
    p.total = o + 1024;   // + slack to align the base to 1024 bytes (the swizzle's period)
    return p;
}
__host__ __device__ inline AttkPlan attk_plan(int n_ctx) {
    const long room = (long) ATK_SMEM - (long) attk_layout(n_ctx, 0).total;
    const long ns = room > 0 ? room / ATK_TILE : 0;
    return attk_layout(n_ctx, (int) (ns < ATK_NSMAX ? ns : ATK_NSMAX));
}

// one full V tile of the P.V chain for one dimension (o_i = fma(p_t, v_t,i, o_i) over its ATK_T positions in order),
// the next 16 positions' values and probabilities loaded while these 16 go through the chain. The tile is swizzled:
// the dimension's value of row r sits at r * 128 + off[r & 7].
__device__ __forceinline__ float pv_tile(const uint8_t *vt, const uint32_t (&off)[8], const float *pr, float o) {
    constexpr int G = 16;
    uint16_t v[G];
    float4 pp[G / 4];
#pragma unroll
    for (int u = 0; u < G; u++) v[u] = *(const uint16_t *) (vt + u * 128 + off[u & 7]);
#pragma unroll
    for (int u = 0; u < G / 4; u++) pp[u] = ((const float4 *) pr)[u];
#pragma unroll
    for (int gi = 0; gi < ATK_T / G; gi++) {
        uint16_t vn[G];
        float4 pn[G / 4];
        if (gi + 1 < ATK_T / G) {
#pragma unroll
            for (int u = 0; u < G; u++) vn[u] = *(const uint16_t *) (vt + ((gi + 1) * G + u) * 128 + off[u & 7]);
#pragma unroll
            for (int u = 0; u < G / 4; u++) pn[u] = ((const float4 *) (pr + (gi + 1) * G))[u];
        }
#pragma unroll
        for (int u = 0; u < G / 4; u++) {
            o = __fmaf_rn(pp[u].x, h2f(v[4 * u]), o);
            o = __fmaf_rn(pp[u].y, h2f(v[4 * u + 1]), o);
            o = __fmaf_rn(pp[u].z, h2f(v[4 * u + 2]), o);
            o = __fmaf_rn(pp[u].w, h2f(v[4 * u + 3]), o);
        }
        if (gi + 1 < ATK_T / G) {
#pragma unroll
            for (int u = 0; u < G; u++) v[u] = vn[u];
#pragma unroll
            for (int u = 0; u < G / 4; u++) pp[u] = pn[u];
        }
    }
    return o;
}

__global__ void __launch_bounds__(ATK_NT) k_attn_tma(const __grid_constant__ AttnArgs a) {
    constexpr int D = ATK_D, T = ATK_T;
    extern __shared__ __align__(128) uint8_t smk[];
    uint8_t *sm = smk + ((1024 - (smem_u32(smk) & 1023)) & 1023);
    const AttkPlan L = attk_plan(a.n_ctx);
    const int NS = L.ns;
    const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *trace = a.trace ? a.trace + (size_t) (blockIdx.y * gridDim.x + blockIdx.x) * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    float *q = (float *) (sm + L.q), *kf = (float *) (sm + L.kf), *vf = (float *) (sm + L.vf);
    float *tq = (float *) (sm + L.tq), *tk = (float *) (sm + L.tk), *wq = (float *) (sm + L.wq);
    float *wk = (float *) (sm + L.wk), *y = (float *) (sm + L.y), *sc = (float *) (sm + L.sc);
    uint16_t *kh = (uint16_t *) (sm + L.kh), *vh = (uint16_t *) (sm + L.vh);
    double *dsum = (double *) (sm + L.red);
    float *wmax = (float *) (sm + L.red + 8 * ATK_NW);
    float *rcs = (float *) (sm + L.rcs), *rsn = (float *) (sm + L.rsn);
    uint64_t *full = (uint64_t *) (sm + L.bar);
    if (tid == 0) {
        for (int i = 0; i < NS; i++) mbar_init(&full[i], 1);
        fence_barrier_init();
    }
    pdl_trigger();
    const int H = a.n_head, grp = H / a.n_head_kv, g = h / grp, kvd = a.n_head_kv * D;
    const Col col = a.cols_d[c];
    // before the wait (none of it is written by the previous kernel): the rotary rows of the position read now and
    // both norm weights
    const int pspec = ld_relaxed(&col.s->pos) + col.off;
    const CUtensorMap *tmk = (const CUtensorMap *) ((const uint8_t *) col.s + ATK_TMAP_OFF);
    if (tid == ATK_NT - 1) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(tmk) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(tmk + 1) : "memory");
    }
    if (tid < D) {
        wq[tid] = a.q_norm[tid];
        wk[tid] = a.k_norm[tid];
    } else if (tid < D + D / 2) {
        rcs[tid - D] = a.rope_cs[(size_t) pspec * (D / 2) + tid - D];
        rsn[tid - D] = a.rope_sn[(size_t) pspec * (D / 2) + tid - D];
    }
    __syncthreads();   // barriers initialised
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    const int p = ld_relaxed(&col.s->pos) + col.off;
    const float *qkv = a.qkv + (size_t) c * a.qkv_stride;
    const float *cs = rcs, *sn = rsn;
    if (p != pspec) {
        cs = a.rope_cs + (size_t) p * (D / 2);
        sn = a.rope_sn + (size_t) p * (D / 2);
    }
    const size_t hrow = ((size_t) a.ai * a.n_head_kv + g) * a.n_ctx;   // this kv head's first row in the caches
    uint16_t *kc = (uint16_t *) col.kc + hrow * D, *vc = (uint16_t *) col.vc + hrow * D;
    const int s0 = a.window > 0 ? max(0, p - a.window + 1) : 0, nk = p - s0 + 1;
    const int ng = a.kv_fused ? nk - 1 : nk;   // positions whose V is read from the cache
    const int ntk = (nk + T - 1) / T, ntv = (ng + T - 1) / T, nt = ntk + ntv;
    auto slot = [&](int i) { return sm + (size_t) (i % NS) * ATK_TILE; };
    auto issue = [&](int i) {   // K tile i, or V tile i - ntk (rows past the tensor read as zeros)
        uint64_t *b = &full[i % NS];
        if (i < ntk) {
            mbar_expect_tx(b, (uint32_t) ATK_TILE);
            tma_load_2d(slot(i), tmk, 0, (int) (hrow + s0 + (size_t) i * T), b);
        } else {
            mbar_expect_tx(b, (uint32_t) ATK_TILE);
            tma_load_2d(slot(i), tmk + 1, 0, (int) (hrow + s0 + (size_t) (i - ntk) * T), b);
        }
    };
    if (tid == 0) {
        for (int i = 0; i < min(NS, nt); i++) issue(i);
        if (trace) trace[6] = global_ns();
    }
    // on a wait that gave up at tile i: the tiles in flight (i .. i + NS - 1) land before the CTA exits (bounded
    // waits), then it returns
    auto drain = [&](int i) {
        if (tid == 0)
            for (int j = i; j < min(nt, i + NS); j++) mbar_wait(&full[j % NS], (j / NS) & 1);
    };

    // this head's query, and this position's K and V, in one round of loads; then the rotations (warp 1 the query,
    // warp 0 the key)
    const float gv = tid < D ? qkv[H * D + 2 * kvd + h] : 0.0f;   // the gate input (seoul.cpp:451)
    if (tid < D) {
        q[tid] = qkv[h * D + tid];
        if (a.kv_fused) kf[tid] = qkv[H * D + g * D + tid];
    } else if (a.kv_fused && tid < 2 * D) {
        vf[tid - D] = qkv[H * D + kvd + g * D + tid - D];
    }
    __syncthreads();
    if (warp == 0 && a.kv_fused) {
        norm_rope<D>(kf, wk, cs, sn, a.eps, tk);
        for (int i = lane; i < D; i += 32) {
            kh[i] = f2h(kf[i]);
            vh[i] = f2h(vf[i]);
        }
    } else if (warp == 1) {
        norm_rope<D>(q, wq, cs, sn, a.eps, tq);
    }
    __syncthreads();
    if (trace && tid == 0) trace[2] = global_ns();
    if (a.kv_fused && h % grp == 0 && tid < D) {   // the group's first head writes this position's K/V
        kc[(size_t) p * D + tid] = kh[tid];
        vc[(size_t) p * D + tid] = vh[tid];
    }

    // scores (seoul.cpp:445): thread t takes position t of each K tile
    float qr[D];
#pragma unroll
    for (int i = 0; i < D; i++) qr[i] = q[i];
    float lmax = -INFINITY;
    for (int k = 0; k < ntk; k++) {
        const bool ok = mbar_wait(&full[k % NS], (k / NS) & 1);
        if (trace && tid == 0 && (k == 0 || k == ntk - 1)) trace[k == 0 ? 7 : 8] = global_ns();
        const int t = k * T + tid;
        if (ok && t < nk) {
            uint4 krow[D / 8];
            if (a.kv_fused && t == nk - 1) {   // this position: its own K (the cache row is being written)
#pragma unroll
                for (int w = 0; w < D / 8; w++) krow[w] = ((const uint4 *) kh)[w];
            } else {
                const uint8_t *row = slot(k) + (size_t) tid * (D * 2);
#pragma unroll
                for (int w = 0; w < D / 8; w++) krow[w] = *(const uint4 *) (row + ((w ^ (tid & 7)) << 4));
            }
            const float v = __fmul_rn(dot_h8<D>(qr, krow), a.scale);
            sc[t] = v;
            lmax = lmax < v ? v : lmax;
        }
        if (!__syncthreads_and(ok)) {   // every thread is done with the slot; a wait that gave up ends the CTA
            if (tid == 0) atomicExch(a.err, 7);
            drain(k);
            return;
        }
        if (tid == 0 && k + NS < nt) issue(k + NS);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) wmax[warp] = lmax;
    __syncthreads();
    if (trace && tid == 0) trace[3] = global_ns();
    float m = wmax[0];
    for (int w = 1; w < ATK_NW; w++) m = fmaxf(m, wmax[w]);
    // exp and the double sum (seoul.cpp:446-448); every thread adds the warps' sums in the same order
    double ls = 0.0;
    for (int t = tid; t < nk; t += ATK_NT) {
        const float e = exp_cr(__fsub_rn(sc[t], m));
        sc[t] = e;
        ls += (double) e;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane == 0) dsum[warp] = ls;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < ATK_NW; w++) tot += dsum[w];
    const float iv2 = __double2float_rn(1.0 / tot);
    for (int t = tid; t < nk; t += ATK_NT) sc[t] = __fmul_rn(sc[t], iv2);
    __syncthreads();
    if (trace && tid == 0) trace[4] = global_ns();

    // P.V (seoul.cpp:449-450): o_i = fma(p_t, v_t,i, o_i) over positions in order; thread i < D owns dimension i
    float o = 0.0f;
    uint32_t off[8];   // where this thread's dimension sits in a swizzled row r: off[r & 7]
#pragma unroll
    for (int j = 0; j < 8; j++) off[j] = ((((uint32_t) tid >> 3) ^ j) << 4) | (((uint32_t) tid & 7) << 1);
    for (int k = 0; k < ntv; k++) {
        const int i = ntk + k;
        const bool ok = mbar_wait(&full[i % NS], (i / NS) & 1);
        if (trace && tid == 0 && (k == 0 || k == ntv - 1)) trace[k == 0 ? 9 : 10] = global_ns();
        if (ok && tid < D) {
            const uint8_t *vt = slot(i);
            const float *pr = sc + (size_t) k * T;
            const int n = min(T, ng - k * T);
            if (n == T) {
                o = pv_tile(vt, off, pr, o);
            } else {
                int t = 0;
                for (; t + 8 <= n; t += 8) {
                    uint16_t v8[8];
#pragma unroll
                    for (int u = 0; u < 8; u++) v8[u] = *(const uint16_t *) (vt + (t + u) * 128 + off[u]);
                    const float4 p0 = *(const float4 *) (pr + t), p1 = *(const float4 *) (pr + t + 4);
                    o = __fmaf_rn(p0.x, h2f(v8[0]), o);
                    o = __fmaf_rn(p0.y, h2f(v8[1]), o);
                    o = __fmaf_rn(p0.z, h2f(v8[2]), o);
                    o = __fmaf_rn(p0.w, h2f(v8[3]), o);
                    o = __fmaf_rn(p1.x, h2f(v8[4]), o);
                    o = __fmaf_rn(p1.y, h2f(v8[5]), o);
                    o = __fmaf_rn(p1.z, h2f(v8[6]), o);
                    o = __fmaf_rn(p1.w, h2f(v8[7]), o);
                }
                for (; t < n; t++) {
                    const uint32_t ot = ((((uint32_t) tid >> 3) ^ (t & 7)) << 4) | (((uint32_t) tid & 7) << 1);
                    o = __fmaf_rn(pr[t], h2f(*(const uint16_t *) (vt + t * 128 + ot)), o);
                }
            }
        }
        if (!__syncthreads_and(ok)) {
            if (tid == 0) atomicExch(a.err, 7);
            drain(i);
            return;
        }
        if (tid == 0 && i + NS < nt) issue(i + NS);
    }
    if (trace && tid == 0) trace[5] = global_ns();
    if (tid < D) {
        if (ng < nk) o = __fmaf_rn(sc[nk - 1], h2f(vh[tid]), o);   // this position's own V
        const float gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-gv)));   // seoul.cpp:451
        const float yv = __fmul_rn(o, gate);
        a.att[(size_t) c * a.att_stride + h * D + tid] = yv;
        y[tid] = yv;
    }
    __syncthreads();
    // the 8-bit cut of this head's output blocks (imi_cut32 of seoul.cpp:457), so the o table only loads codes
    if (a.q8o_q && warp == 0) {
        const int HD = H * D;
        for (int q0 = 0; q0 < D / 4; q0 += 32) {
            const int qi = q0 + lane;
            const bool act = qi < D / 4;
            const float4 v = act ? ((const float4 *) y)[qi] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            cut_chunk(v, act, qi, a.q8o_q + (size_t) c * HD + h * D, a.q8o_d + (size_t) c * (HD / 32) + h * D / 32,
                      a.q8o_s + (size_t) c * (HD / 32) + h * D / 32);
        }
    }
    if (trace && tid == 0) trace[14] = global_ns();
}

// k_attn_grp: the same attention for many columns, one CTA of ATG_NT threads per (kv head g, column c) computing the
// GRP query heads g*GRP .. g*GRP+GRP-1 that share the kv head (GQA), so every cached K and V row of the group is read
// once for all of them instead of once per query head. Per query head the float order is k_attn's: q RMSNorm +
// rotation, scores by dot_h, the maximum, exp and the double sum, the normalised probabilities, the P.V chain over
// positions in order, the sigmoid gate and the 8-bit cut of the head's output. Scores: one thread per position, its K
// row converted once and dotted with the GRP queries; P.V: one thread per dimension running the GRP heads' chains
// (one V load for all), V rows in shared memory tiles (ATG_NTILE in flight from before the scores, cp.async).
// V tiles of ATG_VT positions (8 KB at head_dim 64), ATG_NTILE in flight: a tile takes ~1.5 us to arrive and its
// chains ~0.2 us, so with two in flight the P.V loop waited on every tile
constexpr int ATG_NT = 256, ATG_NW = ATG_NT / 32, ATG_VT = 64, ATG_NTILE = 8;
struct AttnGPlan {
    size_t q, ktmp, tmp, kh, vh, rcs, rsn, y, red, vt, sc, total;
};
// floats per query head's score row: a multiple of 4, so every row starts 16-byte aligned (float4 reads of P.V)
__host__ __device__ inline int attn_grp_sc_stride(int n_ctx) { return (n_ctx + 3) / 4 * 4; }
__host__ __device__ inline AttnGPlan attn_grp_plan(int D, int grp, int n_ctx) {
    AttnGPlan p;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 15) / 16 * 16; return r; };
    p.q = take(4 * (size_t) grp * D);
    p.ktmp = take(4 * (size_t) D);
    p.tmp = take(4 * (size_t) (grp + 1) * D);   // norm_rope scratch: warp 0 (this position's K), warps 1..grp (queries)
    p.kh = take(2 * (size_t) D);
    p.vh = take(2 * (size_t) D);
    p.rcs = take(4 * (size_t) D / 2);
    p.rsn = take(4 * (size_t) D / 2);
    p.y = take(4 * (size_t) grp * D);
    p.red = take(8 * (size_t) ATG_NW * grp + 4 * (size_t) ATG_NW * grp + 8 * (size_t) grp);
    p.vt = take((size_t) ATG_NTILE * ATG_VT * D * 2);
    p.sc = take(4 * (size_t) grp * attn_grp_sc_stride(n_ctx));
    p.total = o;
    return p;
}

template <int D, int GRP>
__global__ void __launch_bounds__(ATG_NT, 2) k_attn_grp(const __grid_constant__ AttnArgs a) {
    static_assert(D <= ATG_NT && (GRP == 2 || GRP == 4) && GRP + 1 <= ATG_NW, "a thread per dimension; a warp per query");
    extern __shared__ __align__(16) uint8_t sma[];
    const AttnGPlan L = attn_grp_plan(D, GRP, a.n_ctx);
    const int g = blockIdx.x, c = a.cols_d[blockIdx.y].order, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *trace = a.trace ? a.trace + (size_t) (blockIdx.y * gridDim.x + blockIdx.x) * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    float *q = (float *) (sma + L.q), *ktmp = (float *) (sma + L.ktmp), *tmp = (float *) (sma + L.tmp);
    float *y = (float *) (sma + L.y), *sc = (float *) (sma + L.sc);
    uint16_t *kh = (uint16_t *) (sma + L.kh), *vh = (uint16_t *) (sma + L.vh), *vt = (uint16_t *) (sma + L.vt);
    double *dsum = (double *) (sma + L.red);
    float *wmax = (float *) (sma + L.red + 8 * ATG_NW * GRP), *inv = wmax + ATG_NW * GRP;
    float *rcs = (float *) (sma + L.rcs), *rsn = (float *) (sma + L.rsn);
    pdl_trigger();
    const int H = a.n_head, kvd = a.n_head_kv * D, NC = a.n_ctx, SS = attn_grp_sc_stride(NC);
    const Col col = a.cols_d[c];
    const int pspec = ld_relaxed(&col.s->pos) + col.off;
    for (int i = tid; i < D / 2; i += ATG_NT) {
        rcs[i] = a.rope_cs[(size_t) pspec * (D / 2) + i];
        rsn[i] = a.rope_sn[(size_t) pspec * (D / 2) + i];
    }
    if (tid == 0) {   // before the wait: this kv head's cached K and V rows into L2 (a hint only)
        const int pp = ld_relaxed(&col.s->pos) + col.off, ps = a.window > 0 ? max(0, pp - a.window + 1) : 0;
        const size_t row = (size_t) D * 2, bytes = (size_t) max(pp - ps, 0) * row, hb = ((size_t) a.ai * a.n_head_kv + g) * NC;
        const uint8_t *kb = (const uint8_t *) col.kc + (hb + ps) * row;
        const uint8_t *vb0 = (const uint8_t *) col.vc + (hb + ps) * row;
        for (size_t o = 0; o < bytes; o += 65536) {
            const uint32_t n = (uint32_t) min((size_t) 65536, bytes - o);
            prefetch_l2(kb + o, n);
            prefetch_l2(vb0 + o, n);
        }
    }
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    const int p = ld_relaxed(&col.s->pos) + col.off;
    const float *qkv = a.qkv + (size_t) c * a.qkv_stride;
    const float *cs = rcs, *sn = rsn;
    if (p != pspec) {
        cs = a.rope_cs + (size_t) p * (D / 2);
        sn = a.rope_sn + (size_t) p * (D / 2);
    }
    // this kv head's rows of the layer: [position][D] (caches [layer][kv head][position][D])
    uint16_t *kc = (uint16_t *) col.kc + ((size_t) a.ai * a.n_head_kv + g) * NC * D;
    uint16_t *vc = (uint16_t *) col.vc + ((size_t) a.ai * a.n_head_kv + g) * NC * D;
    const int s0 = a.window > 0 ? max(0, p - a.window + 1) : 0, nk = p - s0 + 1;
    const int ng = a.kv_fused ? nk - 1 : nk;   // positions whose V is read from the cache
    const int ntile = (ng + ATG_VT - 1) / ATG_VT;
    auto load_tile = [&](int k) {   // V rows of positions s0 + k*VT .. into buffer k % ATG_NTILE, by all threads
        uint16_t *dst = vt + (size_t) (k % ATG_NTILE) * ATG_VT * D;
        const int t0 = k * ATG_VT, n = min(ATG_VT, ng - t0);
        for (int i = tid; i < n * (D / 8); i += ATG_NT) {
            const int t = i / (D / 8), ch = i - t * (D / 8);
            cp16(dst + (size_t) t * D + 8 * ch, vc + (size_t) (s0 + t0 + t) * D + 8 * ch);
        }
    };
    __syncthreads();   // the rotary rows are in shared memory
    for (int k = 0; k < ATG_NTILE - 1; k++) {   // the first V tiles load while the setup and the scores run
        if (k < ntile) load_tile(k);
        cp_commit();
    }
    // this position's K and V (warp 0) and the group's rotated queries (warp 1 + j for query head g*GRP + j)
    if (a.kv_fused) kv_make<D>(a, qkv, g, p, ktmp, tmp, kh, vh);
    if (warp >= 1 && warp <= GRP) {
        const int j = warp - 1, h = g * GRP + j;
        float *qj = q + j * D;
        for (int i = lane; i < D; i += 32) qj[i] = qkv[h * D + i];
        __syncwarp();
        norm_rope<D>(qj, a.q_norm, cs, sn, a.eps, tmp + (j + 1) * D);
    }
    __syncthreads();
    if (a.kv_fused && tid < D) {
        kc[(size_t) p * D + tid] = kh[tid];
        vc[(size_t) p * D + tid] = vh[tid];
    }

    // scores (seoul.cpp:445): one thread per position; the K row's halves converted once, dotted with every query in
    // dot_h8's order (8 lane accumulators in steps of 8, then imi_hsum)
    float lmax[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) lmax[j] = -INFINITY;
    constexpr int SB = GRP * D >= ATG_NT ? 1 : 2;   // K rows a thread loads together (registers allow one at full width)
#pragma unroll 1
    for (int t0 = tid; t0 < nk; t0 += SB * ATG_NT) {
        uint4 kr[SB][D / 8];
#pragma unroll
        for (int u = 0; u < SB; u++) {
            const int t = t0 + u * ATG_NT, pt = s0 + t;
            if (t < nk) {
                const uint4 *src = (a.kv_fused && pt == p) ? (const uint4 *) kh : (const uint4 *) (kc + (size_t) pt * D);
#pragma unroll
                for (int w = 0; w < D / 8; w++) kr[u][w] = src[w];
            }
        }
#pragma unroll
        for (int u = 0; u < SB; u++) {
            const int t = t0 + u * ATG_NT;
            if (t < nk) {
                float acc[GRP][8];
#pragma unroll
                for (int j = 0; j < GRP; j++)
#pragma unroll
                    for (int l = 0; l < 8; l++) acc[j][l] = 0.0f;
#pragma unroll
                for (int w = 0; w < D / 8; w++) {
                    const uint32_t uu[4] = { kr[u][w].x, kr[u][w].y, kr[u][w].z, kr[u][w].w };
                    float kf[8];
#pragma unroll
                    for (int hh = 0; hh < 4; hh++) {
                        kf[2 * hh] = h2f((uint16_t) (uu[hh] & 0xffff));
                        kf[2 * hh + 1] = h2f((uint16_t) (uu[hh] >> 16));
                    }
#pragma unroll
                    for (int j = 0; j < GRP; j++) {
                        const float4 qa = *(const float4 *) (q + j * D + 8 * w), qb = *(const float4 *) (q + j * D + 8 * w + 4);
                        acc[j][0] = __fmaf_rn(qa.x, kf[0], acc[j][0]);
                        acc[j][1] = __fmaf_rn(qa.y, kf[1], acc[j][1]);
                        acc[j][2] = __fmaf_rn(qa.z, kf[2], acc[j][2]);
                        acc[j][3] = __fmaf_rn(qa.w, kf[3], acc[j][3]);
                        acc[j][4] = __fmaf_rn(qb.x, kf[4], acc[j][4]);
                        acc[j][5] = __fmaf_rn(qb.y, kf[5], acc[j][5]);
                        acc[j][6] = __fmaf_rn(qb.z, kf[6], acc[j][6]);
                        acc[j][7] = __fmaf_rn(qb.w, kf[7], acc[j][7]);
                    }
                }
#pragma unroll
                for (int j = 0; j < GRP; j++) {
                    const float r0 = __fadd_rn(acc[j][0], acc[j][4]), r1 = __fadd_rn(acc[j][1], acc[j][5]),
                                r2 = __fadd_rn(acc[j][2], acc[j][6]), r3 = __fadd_rn(acc[j][3], acc[j][7]);
                    const float v = __fmul_rn(__fadd_rn(__fadd_rn(r0, r2), __fadd_rn(r1, r3)), a.scale);
                    sc[(size_t) j * SS + t] = v;
                    lmax[j] = lmax[j] < v ? v : lmax[j];
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        float m = lmax[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[warp * GRP + j] = m;
    }
    __syncthreads();
    float m[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        m[j] = wmax[j];
        for (int w = 1; w < ATG_NW; w++) m[j] = fmaxf(m[j], wmax[w * GRP + j]);
    }
    // exp and the double sum (seoul.cpp:446-448), per query head
    double ls[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) ls[j] = 0.0;
    for (int t = tid; t < nk; t += ATG_NT)
#pragma unroll
        for (int j = 0; j < GRP; j++) {
            const float e = exp_cr(__fsub_rn(sc[(size_t) j * SS + t], m[j]));
            sc[(size_t) j * SS + t] = e;
            ls[j] += (double) e;
        }
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        double v = ls[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) dsum[warp * GRP + j] = v;
    }
    __syncthreads();
    if (tid < GRP) {
        double t = 0.0;
        for (int w = 0; w < ATG_NW; w++) t += dsum[w * GRP + tid];
        inv[tid] = __double2float_rn(1.0 / t);
    }
    __syncthreads();
    for (int t = tid; t < nk; t += ATG_NT)
#pragma unroll
        for (int j = 0; j < GRP; j++) sc[(size_t) j * SS + t] = __fmul_rn(sc[(size_t) j * SS + t], inv[j]);

    // P.V (seoul.cpp:449-450): thread i < D runs, for each query head j of the group, o_j = fma(p_jt, v_t,i, o_j) over
    // positions in order; one load of v_t,i serves all GRP chains, the probabilities arrive 4 positions per load
    const int i = tid;
    const bool pv = tid < D;
    float o[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) o[j] = 0.0f;
    for (int k = 0; k < ntile; k++) {
        if (k + ATG_NTILE - 1 < ntile) load_tile(k + ATG_NTILE - 1);   // into the buffer tile k - 1 left
        cp_commit();
        cp_wait_group<ATG_NTILE - 1>();   // tile k's group is complete
        __syncthreads();
        if (pv) {
            const uint16_t *vb = vt + (size_t) (k % ATG_NTILE) * ATG_VT * D + i;
            const float *pr = sc + (size_t) k * ATG_VT;   // + j * SS: head j's probabilities of this tile
            const int n = min(ATG_VT, ng - k * ATG_VT);
            int t = 0;
            for (; t + 4 <= n; t += 4) {   // 4 positions: their loads first
                float4 p4[GRP];
                uint16_t v4[4];
#pragma unroll
                for (int j = 0; j < GRP; j++) p4[j] = *(const float4 *) (pr + (size_t) j * SS + t);
#pragma unroll
                for (int u = 0; u < 4; u++) v4[u] = vb[(size_t) (t + u) * D];
                const float f0 = h2f(v4[0]), f1 = h2f(v4[1]), f2 = h2f(v4[2]), f3 = h2f(v4[3]);
#pragma unroll
                for (int j = 0; j < GRP; j++) {
                    o[j] = __fmaf_rn(p4[j].x, f0, o[j]);
                    o[j] = __fmaf_rn(p4[j].y, f1, o[j]);
                    o[j] = __fmaf_rn(p4[j].z, f2, o[j]);
                    o[j] = __fmaf_rn(p4[j].w, f3, o[j]);
                }
            }
            for (; t < n; t++) {
                const float f = h2f(vb[(size_t) t * D]);
#pragma unroll
                for (int j = 0; j < GRP; j++) o[j] = __fmaf_rn(pr[(size_t) j * SS + t], f, o[j]);
            }
        }
        __syncthreads();   // the buffer is free for the tile issued ATG_NTILE - 1 rounds on
    }
    cp_wait_group<0>();
    if (pv) {
#pragma unroll
        for (int j = 0; j < GRP; j++) {
            const int h = g * GRP + j;
            float oj = o[j];
            if (ng < nk) oj = __fmaf_rn(sc[(size_t) j * SS + nk - 1], h2f(vh[i]), oj);   // this position's own V
            const float gv = qkv[H * D + 2 * kvd + h];
            const float gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-gv)));   // seoul.cpp:451
            const float yv = __fmul_rn(oj, gate);
            a.att[(size_t) c * a.att_stride + h * D + i] = yv;
            y[j * D + i] = yv;
        }
    }
    __syncthreads();
    // the 8-bit cut of each query head's output blocks (imi_cut32 of seoul.cpp:457): warp j cuts head g*GRP + j
    if (a.q8o_q && warp < GRP) {
        const int HD = H * D, h = g * GRP + warp;
        for (int q0 = 0; q0 < D / 4; q0 += 32) {
            const int qi = q0 + lane;
            const bool act = qi < D / 4;
            const float4 v = act ? ((const float4 *) (y + warp * D))[qi] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            cut_chunk(v, act, qi, a.q8o_q + (size_t) c * HD + h * D, a.q8o_d + (size_t) c * (HD / 32) + h * D / 32,
                      a.q8o_s + (size_t) c * (HD / 32) + h * D / 32);
        }
    }
    if (trace && tid == 0) trace[14] = global_ns();
}

// k_attn_gtma: k_attn_grp's work (one CTA per (kv head g, column) for the GRP query heads sharing it, each in
// k_attn's float order) at head_dim 64, with k_attn_tma's copy ring: the kv head's K tiles and then its V tiles by 2D
// tensor copies of ATK_T rows (32 KB, 128-byte swizzle) through ns slots, two CTAs per SM (ATGK_SMEM each) while the
// score rows leave room for two slots, else one (ATK_SMEM). Scores: one thread per position of a K tile, its row
// converted once and dotted with the GRP queries; P.V: 128 threads, one per (dimension, half of the heads), each
// running GRP / 2 chains from one V load, the next 8 positions' values and probabilities loaded while these 8 go
// through the chains.
struct AttgkPlan {
    size_t q, kf, vf, tmp, wq, wk, y, kh, vh, rcs, rsn, red, bar, sc, total;
    int ns;   // ring slots (the ring starts at the 1024-byte aligned base)
};
__host__ __device__ inline AttgkPlan attgk_layout(int grp, int n_ctx, int ns) {
    AttgkPlan p;
    p.ns = ns;
    const size_t D = ATK_D;
    size_t o = (size_t) ns * ATK_TILE;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 15) / 16 * 16; return r; };
    p.q = take(4 * grp * D);
    p.kf = take(4 * D);
    p.vf = take(4 * D);
    p.tmp = take(4 * (grp + 1) * D);   // norm_rope scratch: warp 0 (this position's K), warps 1..grp (the queries)
    p.y = p.tmp;                        // the heads' outputs, at the end (the scratch is free then)
    p.wq = take(4 * D);
    p.wk = take(4 * D);
    p.kh = take(2 * D);
    p.vh = take(2 * D);
    p.rcs = take(4 * D / 2);
    p.rsn = take(4 * D / 2);
    p.red = take(8 * (size_t) ATK_NW * grp + 4 * (size_t) ATK_NW * grp);
    p.bar = take(8 * ATGK_NSMAX);
    p.sc = take(4 * (size_t) grp * attn_grp_sc_stride(n_ctx));
    p.total = o + 1024;   // + slack to align the base to 1024 bytes
    return p;
}
__host__ __device__ inline AttgkPlan attgk_plan(int grp, int n_ctx) {
    const long small = (long) attgk_layout(grp, n_ctx, 0).total;
    long ns = (ATGK_SMEM - small) / ATK_TILE;         // two CTAs per SM
    if (ns < 2) ns = (ATK_SMEM - small) / ATK_TILE;   // one
    if (ns < 0) ns = 0;
    return attgk_layout(grp, n_ctx, (int) (ns < ATGK_NSMAX ? ns : ATGK_NSMAX));
}

// n positions of a swizzled V tile through CH chains of dimension d: o_j = fma(p_jt, v_t, o_j) in position order;
// pr + j * SS: chain j's probabilities of the tile
template <int CH>
__device__ __forceinline__ void pv_chains(const uint8_t *vt, const uint32_t (&off)[8], const float *pr, int SS, int n,
                                          float (&o)[CH], int d) {
    const int n8 = n & ~7;
    if (n8 > 0) {
        uint16_t v[8];
        float4 pa[CH][2];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = *(const uint16_t *) (vt + u * 128 + off[u]);
#pragma unroll
        for (int j = 0; j < CH; j++) {
            pa[j][0] = *(const float4 *) (pr + (size_t) j * SS);
            pa[j][1] = *(const float4 *) (pr + (size_t) j * SS + 4);
        }
        for (int t = 0; t < n8; t += 8) {
            const bool more = t + 8 < n8;
            uint16_t vn[8];
            float4 pn[CH][2];
            if (more) {
#pragma unroll
                for (int u = 0; u < 8; u++) vn[u] = *(const uint16_t *) (vt + (t + 8 + u) * 128 + off[u]);
#pragma unroll
                for (int j = 0; j < CH; j++) {
                    pn[j][0] = *(const float4 *) (pr + (size_t) j * SS + t + 8);
                    pn[j][1] = *(const float4 *) (pr + (size_t) j * SS + t + 12);
                }
            }
            float f[8];
#pragma unroll
            for (int u = 0; u < 8; u++) f[u] = h2f(v[u]);
#pragma unroll
            for (int j = 0; j < CH; j++) {
                o[j] = __fmaf_rn(pa[j][0].x, f[0], o[j]);
                o[j] = __fmaf_rn(pa[j][0].y, f[1], o[j]);
                o[j] = __fmaf_rn(pa[j][0].z, f[2], o[j]);
                o[j] = __fmaf_rn(pa[j][0].w, f[3], o[j]);
                o[j] = __fmaf_rn(pa[j][1].x, f[4], o[j]);
                o[j] = __fmaf_rn(pa[j][1].y, f[5], o[j]);
                o[j] = __fmaf_rn(pa[j][1].z, f[6], o[j]);
                o[j] = __fmaf_rn(pa[j][1].w, f[7], o[j]);
            }
            if (more) {
#pragma unroll
                for (int u = 0; u < 8; u++) v[u] = vn[u];
#pragma unroll
                for (int j = 0; j < CH; j++) {
                    pa[j][0] = pn[j][0];
                    pa[j][1] = pn[j][1];
                }
            }
        }
    }
    for (int t = n8; t < n; t++) {
        const uint32_t ot = ((((uint32_t) d >> 3) ^ (t & 7)) << 4) | (((uint32_t) d & 7) << 1);
        const float fv = h2f(*(const uint16_t *) (vt + t * 128 + ot));
#pragma unroll
        for (int j = 0; j < CH; j++) o[j] = __fmaf_rn(pr[(size_t) j * SS + t], fv, o[j]);
    }
}

template <int GRP>
__global__ void __launch_bounds__(ATK_NT, 2) k_attn_gtma(const __grid_constant__ AttnArgs a) {
    constexpr int D = ATK_D, T = ATK_T, CH = GRP / 2;
    static_assert((GRP == 2 || GRP == 4) && GRP + 1 <= ATK_NW, "a warp per query; two P.V threads per dimension");
    extern __shared__ __align__(128) uint8_t smg[];
    uint8_t *sm = smg + ((1024 - (smem_u32(smg) & 1023)) & 1023);
    const AttgkPlan L = attgk_plan(GRP, a.n_ctx);
    const int NS = L.ns;
    const int g = blockIdx.x, c = a.cols_d[blockIdx.y].order, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long *trace = a.trace ? a.trace + (size_t) (blockIdx.y * gridDim.x + blockIdx.x) * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    float *q = (float *) (sm + L.q), *kf = (float *) (sm + L.kf), *vf = (float *) (sm + L.vf);
    float *tmp = (float *) (sm + L.tmp), *wq = (float *) (sm + L.wq), *wk = (float *) (sm + L.wk);
    float *y = (float *) (sm + L.y), *sc = (float *) (sm + L.sc);
    uint16_t *kh = (uint16_t *) (sm + L.kh), *vh = (uint16_t *) (sm + L.vh);
    double *dsum = (double *) (sm + L.red);
    float *wmax = (float *) (sm + L.red + 8 * ATK_NW * GRP);
    float *rcs = (float *) (sm + L.rcs), *rsn = (float *) (sm + L.rsn);
    uint64_t *full = (uint64_t *) (sm + L.bar);
    if (tid == 0) {
        for (int i = 0; i < NS; i++) mbar_init(&full[i], 1);
        fence_barrier_init();
    }
    pdl_trigger();
    const int H = a.n_head, kvd = a.n_head_kv * D, SS = attn_grp_sc_stride(a.n_ctx);
    const Col col = a.cols_d[c];
    // before the wait (none of it is written by the previous kernel): the rotary rows of the position read now, both
    // norm weights, and the tensor maps into the copy unit's cache
    const int pspec = ld_relaxed(&col.s->pos) + col.off;
    const CUtensorMap *tmk = (const CUtensorMap *) ((const uint8_t *) col.s + ATK_TMAP_OFF);
    if (tid == ATK_NT - 1) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(tmk) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(tmk + 1) : "memory");
    }
    if (tid < D) {
        wq[tid] = a.q_norm[tid];
        wk[tid] = a.k_norm[tid];
    } else if (tid < D + D / 2) {
        rcs[tid - D] = a.rope_cs[(size_t) pspec * (D / 2) + tid - D];
        rsn[tid - D] = a.rope_sn[(size_t) pspec * (D / 2) + tid - D];
    }
    __syncthreads();   // barriers initialised
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    const int p = ld_relaxed(&col.s->pos) + col.off;
    const float *qkv = a.qkv + (size_t) c * a.qkv_stride;
    const float *cs = rcs, *sn = rsn;
    if (p != pspec) {
        cs = a.rope_cs + (size_t) p * (D / 2);
        sn = a.rope_sn + (size_t) p * (D / 2);
    }
    const size_t hrow = ((size_t) a.ai * a.n_head_kv + g) * a.n_ctx;   // this kv head's first row in the caches
    uint16_t *kc = (uint16_t *) col.kc + hrow * D, *vc = (uint16_t *) col.vc + hrow * D;
    const int s0 = a.window > 0 ? max(0, p - a.window + 1) : 0, nk = p - s0 + 1;
    const int ng = a.kv_fused ? nk - 1 : nk;   // positions whose V is read from the cache
    const int ntk = (nk + T - 1) / T, ntv = (ng + T - 1) / T, nt = ntk + ntv;
    auto slot = [&](int i) { return sm + (size_t) (i % NS) * ATK_TILE; };
    auto issue = [&](int i) {   // K tile i, or V tile i - ntk (rows past the tensor read as zeros)
        uint64_t *b = &full[i % NS];
        mbar_expect_tx(b, (uint32_t) ATK_TILE);
        tma_load_2d(slot(i), tmk + (i < ntk ? 0 : 1), 0, (int) (hrow + s0 + (size_t) (i < ntk ? i : i - ntk) * T), b);
    };
    if (tid == 0) {
        for (int i = 0; i < min(NS, nt); i++) issue(i);
        if (trace) trace[6] = global_ns();
    }
    auto drain = [&](int i) {   // after a wait that gave up at tile i: the tiles in flight land (bounded waits)
        if (tid == 0)
            for (int j = i; j < min(nt, i + NS); j++) mbar_wait(&full[j % NS], (j / NS) & 1);
    };

    // the group's queries and this position's K and V in one round of loads; then the rotations (warp 0 the key,
    // warp 1 + j query j)
    const int i = tid & (D - 1), j0 = (tid >> 6) * CH;   // P.V thread (tid < 2 * D): dimension i, heads j0 .. j0+CH-1
    for (int k = tid; k < GRP * D; k += ATK_NT) q[k] = qkv[(size_t) g * GRP * D + k];
    if (a.kv_fused) {
        if (tid < D) kf[tid] = qkv[H * D + g * D + tid];
        else if (tid < 2 * D) vf[tid - D] = qkv[H * D + kvd + g * D + tid - D];
    }
    __syncthreads();
    if (warp == 0 && a.kv_fused) {
        norm_rope<D>(kf, wk, cs, sn, a.eps, tmp);
        for (int k = lane; k < D; k += 32) {
            kh[k] = f2h(kf[k]);
            vh[k] = f2h(vf[k]);
        }
    } else if (warp >= 1 && warp <= GRP) {
        norm_rope<D>(q + (warp - 1) * D, wq, cs, sn, a.eps, tmp + warp * D);
    }
    __syncthreads();
    if (trace && tid == 0) trace[2] = global_ns();
    if (a.kv_fused && tid < D) {   // this position's K/V into the caches
        kc[(size_t) p * D + tid] = kh[tid];
        vc[(size_t) p * D + tid] = vh[tid];
    }

    // scores (seoul.cpp:445): thread t takes position t of each K tile, its row converted once and dotted with every
    // query in dot_h8's order (8 lane accumulators in steps of 8, then imi_hsum)
    float lmax[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) lmax[j] = -INFINITY;
    for (int k = 0; k < ntk; k++) {
        const bool ok = mbar_wait(&full[k % NS], (k / NS) & 1);
        if (trace && tid == 0 && (k == 0 || k == ntk - 1)) trace[k == 0 ? 7 : 8] = global_ns();
        const int t = k * T + tid;
        if (ok && t < nk) {
            // this position's own K (its cache row is being written), else the row in the slot; one chunk at a time
            const bool own = a.kv_fused && t == nk - 1;
            const uint8_t *row = own ? (const uint8_t *) kh : slot(k) + (size_t) tid * (D * 2);
            const uint32_t sw = own ? 0u : (uint32_t) (tid & 7);
            float acc[GRP][8];
#pragma unroll
            for (int j = 0; j < GRP; j++)
#pragma unroll
                for (int l = 0; l < 8; l++) acc[j][l] = 0.0f;
#pragma unroll
            for (int w = 0; w < D / 8; w++) {
                const uint4 kw = *(const uint4 *) (row + ((w ^ sw) << 4));
                const uint32_t uu[4] = { kw.x, kw.y, kw.z, kw.w };
                float kv8[8];
#pragma unroll
                for (int hh = 0; hh < 4; hh++) {
                    kv8[2 * hh] = h2f((uint16_t) (uu[hh] & 0xffff));
                    kv8[2 * hh + 1] = h2f((uint16_t) (uu[hh] >> 16));
                }
#pragma unroll
                for (int j = 0; j < GRP; j++) {
                    const float4 qa = *(const float4 *) (q + j * D + 8 * w), qb = *(const float4 *) (q + j * D + 8 * w + 4);
                    acc[j][0] = __fmaf_rn(qa.x, kv8[0], acc[j][0]);
                    acc[j][1] = __fmaf_rn(qa.y, kv8[1], acc[j][1]);
                    acc[j][2] = __fmaf_rn(qa.z, kv8[2], acc[j][2]);
                    acc[j][3] = __fmaf_rn(qa.w, kv8[3], acc[j][3]);
                    acc[j][4] = __fmaf_rn(qb.x, kv8[4], acc[j][4]);
                    acc[j][5] = __fmaf_rn(qb.y, kv8[5], acc[j][5]);
                    acc[j][6] = __fmaf_rn(qb.z, kv8[6], acc[j][6]);
                    acc[j][7] = __fmaf_rn(qb.w, kv8[7], acc[j][7]);
                }
            }
#pragma unroll
            for (int j = 0; j < GRP; j++) {
                const float r0 = __fadd_rn(acc[j][0], acc[j][4]), r1 = __fadd_rn(acc[j][1], acc[j][5]),
                            r2 = __fadd_rn(acc[j][2], acc[j][6]), r3 = __fadd_rn(acc[j][3], acc[j][7]);
                const float v = __fmul_rn(__fadd_rn(__fadd_rn(r0, r2), __fadd_rn(r1, r3)), a.scale);
                sc[(size_t) j * SS + t] = v;
                lmax[j] = lmax[j] < v ? v : lmax[j];
            }
        }
        if (!__syncthreads_and(ok)) {   // every thread is done with the slot; a wait that gave up ends the CTA
            if (tid == 0) atomicExch(a.err, 7);
            drain(k);
            return;
        }
        if (tid == 0 && k + NS < nt) issue(k + NS);
    }
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        float m = lmax[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) wmax[warp * GRP + j] = m;
    }
    __syncthreads();
    if (trace && tid == 0) trace[3] = global_ns();
    float m[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        m[j] = wmax[j];
        for (int w = 1; w < ATK_NW; w++) m[j] = fmaxf(m[j], wmax[w * GRP + j]);
    }
    // exp and the double sum (seoul.cpp:446-448), per query head; every thread adds the warps' sums in the same order
    double ls[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) ls[j] = 0.0;
    for (int t = tid; t < nk; t += ATK_NT)
#pragma unroll
        for (int j = 0; j < GRP; j++) {
            const float e = exp_cr(__fsub_rn(sc[(size_t) j * SS + t], m[j]));
            sc[(size_t) j * SS + t] = e;
            ls[j] += (double) e;
        }
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        double v = ls[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) dsum[warp * GRP + j] = v;
    }
    __syncthreads();
    float inv[GRP];
#pragma unroll
    for (int j = 0; j < GRP; j++) {
        double tot = 0.0;
        for (int w = 0; w < ATK_NW; w++) tot += dsum[w * GRP + j];
        inv[j] = __double2float_rn(1.0 / tot);
    }
    for (int t = tid; t < nk; t += ATK_NT)
#pragma unroll
        for (int j = 0; j < GRP; j++) sc[(size_t) j * SS + t] = __fmul_rn(sc[(size_t) j * SS + t], inv[j]);
    __syncthreads();
    if (trace && tid == 0) trace[4] = global_ns();

    // P.V (seoul.cpp:449-450)
    float o[CH];
#pragma unroll
    for (int jj = 0; jj < CH; jj++) o[jj] = 0.0f;
    uint32_t off[8];   // where dimension i sits in a swizzled row r: off[r & 7]
#pragma unroll
    for (int j = 0; j < 8; j++) off[j] = ((((uint32_t) i >> 3) ^ j) << 4) | (((uint32_t) i & 7) << 1);
    for (int k = 0; k < ntv; k++) {
        const int it = ntk + k;
        const bool ok = mbar_wait(&full[it % NS], (it / NS) & 1);
        if (trace && tid == 0 && (k == 0 || k == ntv - 1)) trace[k == 0 ? 9 : 10] = global_ns();
        if (ok && tid < 2 * D)
            pv_chains<CH>(slot(it), off, sc + (size_t) j0 * SS + (size_t) k * T, SS, min(T, ng - k * T), o, i);
        if (!__syncthreads_and(ok)) {
            if (tid == 0) atomicExch(a.err, 7);
            drain(it);
            return;
        }
        if (tid == 0 && it + NS < nt) issue(it + NS);
    }
    if (trace && tid == 0) trace[5] = global_ns();
    if (tid < 2 * D) {
#pragma unroll
        for (int jj = 0; jj < CH; jj++) {
            const int j = j0 + jj, h = g * GRP + j;
            float oj = o[jj];
            if (ng < nk) oj = __fmaf_rn(sc[(size_t) j * SS + nk - 1], h2f(vh[i]), oj);   // this position's own V
            const float gv = qkv[H * D + 2 * kvd + h];
            const float gate = __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_cr(-gv)));   // seoul.cpp:451
            const float yv = __fmul_rn(oj, gate);
            a.att[(size_t) c * a.att_stride + h * D + i] = yv;
            y[j * D + i] = yv;
        }
    }
    __syncthreads();
    // the 8-bit cut of each query head's output blocks (imi_cut32 of seoul.cpp:457): warp j cuts head g*GRP + j
    if (a.q8o_q && warp < GRP) {
        const int HD = H * D, h = g * GRP + warp;
        for (int q0 = 0; q0 < D / 4; q0 += 32) {
            const int qi = q0 + lane;
            const bool act = qi < D / 4;
            const float4 v = act ? ((const float4 *) (y + warp * D))[qi] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            cut_chunk(v, act, qi, a.q8o_q + (size_t) c * HD + h * D, a.q8o_d + (size_t) c * (HD / 32) + h * D / 32,
                      a.q8o_s + (size_t) c * (HD / 32) + h * D / 32);
        }
    }
    if (trace && tid == 0) trace[14] = global_ns();
}

// ---------------------------------------------------------------------------------------------------------------
// the failure path of the bounded device waits: a wait on an mbarrier no thread ever arrives at (a flag nothing
// sets), with a short limit, gives up, reports IMI_E_TIMEOUT's code in the error flag and returns; no copy is in
// flight, so the CTA exits cleanly and the context stays usable
// ---------------------------------------------------------------------------------------------------------------
__global__ void k_wait_check(long long limit, int *err) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (!mbar_wait(&bar, 0, limit) && threadIdx.x == 0) atomicExch(err, 7);
}

// the conversation records of a step's columns into 32-byte slots (one read-back for all of them)
__global__ void k_gather_sess(const Col *cols, int n, uint8_t *dst) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c < n) *(SessDev *) (dst + 32 * c) = *cols[c].s;
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

// ---------------------------------------------------------------------------------------------------------------
// the Q6_K word table of the product's own files (imi_q8k / imi_q6k_row, tables.cpp:200-278)
// ---------------------------------------------------------------------------------------------------------------
// imi_q8k::from: one warp per 256 values (8 per lane, lane L holding values 8L..8L+7): amax, d = amax/127,
// id = d ? 1/d : 0, q = round-half-even(x * id), the code sum of every 16 values
__global__ void k_q8k_cut(const float *x, int n, int8_t *q, float *d, int16_t *bsums) {
    const int lane = threadIdx.x & 31, j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (j >= n / 256) return;   // whole warps only
    q8k_block(x + 256 * j, lane, q + 256 * j, d + j, bsums + 16 * j);
}

// the word score of one Q6_K row (210 bytes per 256 values: ql[128], qh[64], int8 scales[16], fp16 d) for a q8k
// input, in imi_q6k_row's AVX2 order: 8 threads per row, thread m the integer lane m (values 128n + 32k + 4m .. +3,
// n < 2, k < 4, each 4 times the scale of its 16, minus 32 * (scales[2m] bsums[2m] + scales[2m+1] bsums[2m+1]),
// exact), then lane m's float chain acc = fma(d * dx, float(int), acc) over the blocks in order, and the 8 lanes
// summed as ((a0+a4)+(a2+a6)) + ((a1+a5)+(a3+a7)). A CTA stages its rows (blockDim / 8 of them, contiguous) and the
// input codes in shared memory with coalesced loads first (2.2x faster than reading the 2-byte-aligned blocks
// byte by byte from global memory).
__global__ void __launch_bounds__(256) k_q6k_scores(const uint8_t *W, int rows, int nb, const int8_t *xq,
                                                    const float *xd, const int16_t *bsums, float *out) {
    extern __shared__ __align__(16) uint8_t smq[];
    int8_t *xs = (int8_t *) smq;
    uint8_t *tile = smq + 256 * nb;
    const int tid = threadIdx.x, rpc = blockDim.x / 8, r0 = blockIdx.x * rpc, nr = min(rpc, rows - r0);
    const size_t rb = (size_t) nb * 210, bytes = (size_t) nr * rb;
    for (int i = tid; i < 16 * nb; i += blockDim.x) ((uint4 *) xs)[i] = ((const uint4 *) xq)[i];
    const uint8_t *src = W + (size_t) r0 * rb;
    if (((uintptr_t) src & 15) == 0 && (bytes & 15) == 0) {
        for (size_t i = tid; i < bytes / 16; i += blockDim.x) ((uint4 *) tile)[i] = __ldcs(((const uint4 *) src) + i);
    } else {   // rows of an odd number of 8-block groups: 2-byte pieces (blocks are 2-byte aligned)
        for (size_t i = tid; i < bytes / 2; i += blockDim.x) ((uint16_t *) tile)[i] = ((const uint16_t *) src)[i];
    }
    __syncthreads();
    const int rl = tid >> 3, m = tid & 7;
    const bool act = rl < nr;
    const uint8_t *row = tile + (size_t) (act ? rl : 0) * rb;
    float acc = 0.0f;
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = row + (size_t) i * 210;
        const int8_t *sc = (const int8_t *) (b + 192);
        int lane = 0;
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const uint8_t *qh = b + 128 + 32 * n + 4 * m;
            const uint32_t qh4 = (uint32_t) qh[0] | ((uint32_t) qh[1] << 8) | ((uint32_t) qh[2] << 16) | ((uint32_t) qh[3] << 24);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint8_t *ql = b + 64 * n + (k & 1) * 32 + 4 * m;
                const uint32_t ql4 = (uint32_t) ql[0] | ((uint32_t) ql[1] << 8) | ((uint32_t) ql[2] << 16) | ((uint32_t) ql[3] << 24);
                const uint32_t lo = (k < 2 ? ql4 : ql4 >> 4) & 0x0f0f0f0fu;
                const uint32_t codes = lo | (((qh4 >> (2 * k)) & 0x03030303u) << 4);
                const int x4 = *(const int *) (xs + 256 * i + 128 * n + 32 * k + 4 * m);
                lane += __dp4a((int) codes, x4, 0) * (int) sc[8 * n + 2 * k + (m >= 4)];   // codes <= 63: signed is exact
            }
        }
        const int16_t *bs = bsums + 16 * i;
        lane -= 32 * ((int) sc[2 * m] * bs[2 * m] + (int) sc[2 * m + 1] * bs[2 * m + 1]);
        const float s = __fmul_rn(h2f((uint16_t) (b[208] | (b[209] << 8))), xd[i]);
        acc = __fmaf_rn(s, __int2float_rn(lane), acc);
    }
    // the 8 lanes of a row sit in 8 consecutive threads (an aligned group of 8 within the warp)
    const float r4 = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));   // m < 4: a_m + a_{m+4}
    const float r2 = __fadd_rn(r4, __shfl_down_sync(0xffffffffu, r4, 2));     // m < 2: r_m + r_{m+2}
    const float r1 = __fadd_rn(r2, __shfl_down_sync(0xffffffffu, r2, 1));     // m = 0: (r0 + r2) + (r1 + r3)
    if (act && m == 0) out[r0 + rl] = r1;
}
// the word scores of a Q6_K word table for ncol inputs (each cut per 256 values) into each column's logits (when it
// has them), with imi's greedy pick (the first maximum, the lowest id on ties: the keys of the Q4_0 word-table read),
// each CTA's best key combined by atomicMax in the conversation record; the last CTA to finish ends the step as the
// Q4_0 word-table read does (next token, pick, position). Rows staged as in k_q6k_scores.
__global__ void __launch_bounds__(256) k_q6k_head(const __grid_constant__ Q6HeadArgs a) {
    extern __shared__ __align__(16) uint8_t smq[];
    __shared__ unsigned long long wbest[8][MV_MAX_COLS];
    __shared__ int last_cta;
    const int tid = threadIdx.x, nb = a.nb, nc = a.ncol, rpc = blockDim.x / 8;
    unsigned long long *trace = a.trace ? a.trace + (size_t) blockIdx.x * MV_TRACE : nullptr;
    if (trace && tid == 0) trace[0] = global_ns();
    pdl_trigger();
    int8_t *xs = (int8_t *) smq;                       // [c][256 nb]
    uint8_t *tile = smq + (size_t) 256 * nb * nc;
    const int r0 = blockIdx.x * rpc, nr = min(rpc, a.rows - r0);
    const size_t rb = (size_t) nb * 210, bytes = (size_t) nr * rb;
    const uint8_t *src = a.W + (size_t) r0 * rb;   // the table does not depend on the launches in flight
    if (((uintptr_t) src & 15) == 0 && (bytes & 15) == 0) {
        for (size_t i = tid; i < bytes / 16; i += blockDim.x) ((uint4 *) tile)[i] = __ldcs(((const uint4 *) src) + i);
    } else {
        for (size_t i = tid; i < bytes / 2; i += blockDim.x) ((uint16_t *) tile)[i] = ((const uint16_t *) src)[i];
    }
    pdl_wait();
    if (trace && tid == 0) trace[1] = global_ns();
    for (int i = tid; i < 16 * nb * nc; i += blockDim.x) ((uint4 *) xs)[i] = ((const uint4 *) a.xq)[i];
    __syncthreads();
    const int rl = tid >> 3, m = tid & 7, warp = tid >> 5, lane = tid & 31;
    const bool act = rl < nr;
    const uint8_t *row = tile + (size_t) (act ? rl : 0) * rb;
    // every block's codes unpacked once and used for all the columns (each column its own integer lane and chain)
    float acc[MV_MAX_COLS];
#pragma unroll
    for (int c = 0; c < MV_MAX_COLS; c++) acc[c] = 0.0f;
    for (int i = 0; i < nb; i++) {
        const uint8_t *b = row + (size_t) i * 210;
        const int8_t *sc = (const int8_t *) (b + 192);
        uint32_t codes[8];
        int scl[8];
#pragma unroll
        for (int n = 0; n < 2; n++) {
            const uint8_t *qh = b + 128 + 32 * n + 4 * m;
            const uint32_t qh4 = (uint32_t) qh[0] | ((uint32_t) qh[1] << 8) | ((uint32_t) qh[2] << 16) | ((uint32_t) qh[3] << 24);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint8_t *ql = b + 64 * n + (k & 1) * 32 + 4 * m;
                const uint32_t ql4 = (uint32_t) ql[0] | ((uint32_t) ql[1] << 8) | ((uint32_t) ql[2] << 16) | ((uint32_t) ql[3] << 24);
                codes[4 * n + k] = ((k < 2 ? ql4 : ql4 >> 4) & 0x0f0f0f0fu) | (((qh4 >> (2 * k)) & 0x03030303u) << 4);
                scl[4 * n + k] = sc[8 * n + 2 * k + (m >= 4)];
            }
        }
        const float dblk = h2f((uint16_t) (b[208] | (b[209] << 8)));
        const int s2m = sc[2 * m], s2m1 = sc[2 * m + 1];
#pragma unroll
        for (int c = 0; c < MV_MAX_COLS; c++) {
            if (c >= nc) break;
            const int8_t *x0 = xs + (size_t) c * 256 * nb + 256 * i;
            int lanesum = 0;
#pragma unroll
            for (int g = 0; g < 8; g++) {
                const int x4 = *(const int *) (x0 + 128 * (g >> 2) + 32 * (g & 3) + 4 * m);
                lanesum += __dp4a((int) codes[g], x4, 0) * scl[g];   // codes <= 63: signed is exact
            }
            const int16_t *bs = a.xb + (size_t) c * 16 * nb + 16 * i;
            lanesum -= 32 * (s2m * bs[2 * m] + s2m1 * bs[2 * m + 1]);
            const float s = __fmul_rn(dblk, a.xd[(size_t) c * nb + i]);
            acc[c] = __fmaf_rn(s, __int2float_rn(lanesum), acc[c]);
        }
    }
#pragma unroll
    for (int c = 0; c < MV_MAX_COLS; c++) {
        if (c >= nc) break;
        const float r4 = __fadd_rn(acc[c], __shfl_down_sync(0xffffffffu, acc[c], 4));
        const float r2 = __fadd_rn(r4, __shfl_down_sync(0xffffffffu, r4, 2));
        const float r1 = __fadd_rn(r2, __shfl_down_sync(0xffffffffu, r2, 1));
        unsigned long long key = 0ull;
        if (act && m == 0) {
            const int id = r0 + rl;
            float *lg = a.cols_d[c].logits;
            if (lg) lg[id] = r1;
            key = amax_key(r1, id);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const unsigned long long u = __shfl_xor_sync(0xffffffffu, key, o);
            key = u > key ? u : key;
        }
        if (lane == 0) wbest[warp][c] = key;
    }
    __syncthreads();
    if (tid < nc) {
        unsigned long long k = 0ull;
        for (int w = 0; w < (int) (blockDim.x >> 5); w++) k = wbest[w][tid] > k ? wbest[w][tid] : k;
        atomicMax(&a.cols_d[tid].s->amax, k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_cta = atomicAdd(a.done, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last_cta && tid < nc) {
        __threadfence();
        const Col col = a.cols_d[tid];
        const unsigned long long k = atomicExch(&col.s->amax, 0ull);
        const int id = (int) (0xffffffffu - (uint32_t) (k & 0xffffffffu));
        col.s->next_token = id;
        col.s->amax_val = amax_val(k);
        if (col.picks) col.picks[col.s->pos + col.off] = id;
        if (col.pos_inc) atomicAdd(&col.s->pos, col.pos_inc);
    }
    if (last_cta && tid == 0) *a.done = 0;
    if (trace && tid == 0) trace[14] = global_ns();
}
// rows per CTA of the Q6_K head for nc inputs: a multiple of 4, at most 32, within 220 KB of shared memory
__host__ __device__ inline int q6k_head_rows_per_cta(int nb, int nc) {
    const long room = 220L * 1024 - 256L * nb * nc, per = 210L * nb;
    const long r = room > 0 ? room / per : 0;
    return (int) ((r > 32 ? 32 : r) / 4 * 4);
}
// rows per CTA of k_q6k_scores: a multiple of 4 (whole warps), at most 32, the staged rows within 220 KB (0: too wide)
__host__ __device__ inline int q6k_rows_per_cta(int nb) {
    const long room = 220L * 1024 - 256L * nb, per = 210L * nb;
    const long r = room > 0 ? room / per : 0;
    return (int) ((r > 32 ? 32 : r) / 4 * 4);
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

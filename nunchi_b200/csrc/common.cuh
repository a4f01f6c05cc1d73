// Shared definitions of the B200 decode engine: per-step column descriptors, kernel argument blocks, and the exact
// device math that reproduces imi's AVX2 float order (imi/core/vec.h, imi/core/tables.cpp, imi/core/seoul.cpp).
//
// Exactness rules used throughout (the library is built with --fmad=false, and every float operation that imi's
// result depends on is written with an explicitly rounded intrinsic):
//   * a*b+c that imi computes with _mm256_fmadd_ps  -> __fmaf_rn(a, b, c)
//   * a*b, a+b, a-b, a/b computed separately         -> __fmul_rn, __fadd_rn, __fsub_rn, __fdiv_rn
//   * sqrtf, 1/x                                      -> __fsqrt_rn, __fdiv_rn(1, x)
//   * float <-> fp16 (F16C _cvtss_sh / _cvtph_ps)     -> __float2half_rn / __half2float (both exact or RNE)
//   * round-half-even to int (_mm256_round_ps)        -> __float2int_rn
//   * expf                                            -> exp() in double, rounded once to float (correctly rounded;
//     glibc's expf agrees on all but ~0.06% of inputs)
//   * cosf/sinf of the rotary angles                  -> tables built on the host with the C library's own cosf/sinf
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace imi {

constexpr int MV_IWARPS = 16;              // table-read CTA (one per SM): warps computing integer block dots
constexpr int MV_CWARPS = 4;               // warps running the per-row float chains (and the output stage)
constexpr int MV_ITHREADS = 32 * MV_IWARPS, MV_CTHREADS = 32 * MV_CWARPS;
constexpr int MV_THREADS = MV_ITHREADS + MV_CTHREADS;
constexpr int MV_NBUF = 4;                 // block-dot buffers: stage s goes to buffer (and chain warp) s % MV_NBUF
constexpr int MV_MAX_STAGES = 8;           // weight stages in flight per CTA at most (TMA bulk copies; MvArgs::nstage)
constexpr int MV_STAGE_BYTES = 36864;      // one K=8192 row group of 8 rows, or 32 rows of K=2048
constexpr int MV_MAX_COLS = 8;             // inputs sharing one table read in the small-batch kernel
constexpr int MV_SMEM_BUDGET = 220 * 1024; // shared memory of one table-read CTA (one per SM)

// Per-conversation scalars that live on the device (the rest of imi_seoul_state is device buffers).
struct SessDev {
    int pos;                   // positions read so far (imi_seoul::pos)
    int next_token;            // greedy pick of the latest step with logits
    unsigned long long amax;   // running argmax key of the step in flight (0 between steps)
    float amax_val;
    int pad;
};

// the attention kernel that streams K and V by the copy engine (kernels.cu: k_attn_tma): head_dim, positions per tile,
// most ring slots, threads, shared-memory budget; the conversation's K tensor map sits ATK_TMAP_OFF bytes into its
// device record
constexpr int ATK_D = 64, ATK_T = 256, ATK_NSMAX = 6, ATK_NT = 256, ATK_NW = ATK_NT / 32;
constexpr int ATK_TILE = ATK_T * ATK_D * 2, ATK_TMAP_OFF = 128, ATK_SMEM = 220 * 1024;
// its many-column form (kernels.cu: k_attn_gtma): shared memory of one CTA when two share an SM (228 KB less 1 KB
// reserved per CTA), else ATK_SMEM; most ring slots
constexpr int ATGK_SMEM = 113 * 1024, ATGK_NSMAX = 3;

// One input column of a step. Written by the host before each launch (or left in place for greedy replay).
struct Col {
    SessDev *s;
    __half *kc, *vc;           // [n_attn][n_head_kv][n_ctx][head_dim]
    float *ring;               // conv memory [n_conv][d_conv+1][n_embd]; slot of position p is p mod (d_conv+1)
    float *hid_out;            // where this column's final hidden state goes (null = nowhere)
    float *logits;             // word scores (null = not wanted)
    const float *embd;         // device copy of the input vector when token == -1
    int *picks;                // [n_ctx]: the greedy pick made at each position (written with word scores)
    int token;                 // >= 0 word id, -1 embd, -2 the session's last pick
    int off;                   // position = s->pos + off
    int pos_inc;               // added to s->pos when the step ends
    int order;                 // (the record at index r) the column whose batched attention is launched r-th: the
                               // columns by decreasing attended length, so the longest start first
};

enum Pro : int {
    P_EMBED_NORM = 0,   // x = word row | embd; h = norm(x) * w_pre                       (seoul.cpp:363-365,404)
    P_RESID_NORM = 1,   // x += norm(r) * w_post; h = norm(x) * w_pre                     (seoul.cpp:462-464,473+404)
    P_CONV = 2,         // u = c * (b*x*w_last + sum_k state_k * w_k)                     (seoul.cpp:410-414)
    P_CUT = 3,          // the input as it is                                             (seoul.cpp:457,469)
    P_FINAL = 4,        // x += norm(fo) * w_post; hidden = norm(x) * out_norm            (seoul.cpp:473,476)
    P_Q8IN = 5          // codes given (known-answer tests)
};
enum Epi : int { E_STORE = 0, E_SILU = 1, E_HEAD = 2 };

struct MvArgs {
    const uint8_t *W;          // table rows: [rows][cols/2 code bytes | cols/32 fp16 scales]
    int rows, cols, row_bytes, unit, sr;   // sr: rows per stage
    int nstage;                // weight stages in flight (1..MV_MAX_STAGES)
    const Col *cols_d;
    int ncol;
    const float *in;           // prologue input vector per column
    int in_stride;
    float *xin, *xout;         // residual stream (per column)
    int x_stride;
    const float *wpost, *wpre;
    float eps;
    const uint8_t *emb;        // word table (same row layout) for P_EMBED_NORM
    int emb_row_bytes;
    int emb_q6k;               // 1: the word table is Q6_K (rows of 210-byte blocks per 256 values, as in the file)
    int has_m;                 // 1: Q4_1 rows (codes | scales | minimums); the result is acc + cor, cor over the minimums
    const float *conv_w;       // [d_conv+1][n_embd]
    int d_conv, conv_layer, n_embd;
    int ring_layer;            // >= 0: write the conv memory slots of this layer from ring_src (bcx rows); in P_CONV
                               // (a step of distinct conversations) the conv's own input is written to it
    const float *ring_src;
    int ring_src_stride;
    const int8_t *q8_q;        // P_Q8IN: codes [ncol][cols], scales and sums [ncol][cols/32]
    const float *q8_d, *q8_s;
    int32_t *dots;             // optional: integer block dots [rows][cols/32] of column 0
    float *out;
    int out_stride;
    unsigned int *done;        // CTA counter (E_HEAD finalize)
    int *err;
    unsigned long long *trace; // optional: per-CTA phase timestamps (ns), [grid][MV_TRACE] (diagnostics only)
    // E_SILU: the 8-bit cut of the produced values, per column [c][rows/2] codes and [c][rows/64] scales / sums,
    // made here (each CTA owns whole 32-value blocks: unit = 64 rows) so the next read only loads codes
    int8_t *q8o_q;
    float *q8o_d, *q8o_s;
    int ab_len;                // produced values per column a CTA holds (max over CTAs)
};
constexpr int MV_TRACE = 16;

struct AttnArgs {
    const Col *cols_d;
    int ncol;
    const float *qkv;
    int qkv_stride;
    float *att;
    int att_stride;
    const float *q_norm, *k_norm;
    float eps, scale;
    const float *rope_cs, *rope_sn;   // [n_ctx][head_dim/2] for this layer's base (and frequency factors)
    int ai, n_head, n_head_kv, head_dim, n_ctx, window;
    int kv_fused;                     // 1: write K/V at the column's position here and use own copies for it
    int *err;
    int8_t *q8o_q;                    // the 8-bit cut of the attention output, per column [c][n_head*head_dim] codes,
    float *q8o_d, *q8o_s;             // [c][n_head*head_dim/32] scales and scale*sums (the o table reads only these)
    unsigned long long *trace;        // optional: per-CTA timestamps (ns), [grid][MV_TRACE]: 0 start, 1 after wait, 14 end
};

struct FinalArgs {
    const Col *cols_d;
    int ncol;
    const float *in;                  // fo per column
    int in_stride;
    const float *xin;                 // residual (per column)
    int x_stride;
    const float *wpost, *out_norm;
    float eps;
    int n_embd;
    unsigned long long *trace;        // optional: per-CTA timestamps (ns), [grid][MV_TRACE]
    // Q6_K word table: the output-normed hidden state also cut per 256 values (imi_q8k::from) into
    // q8k_q[c][n_embd], q8k_d[c][n_embd/256], q8k_b[c][n_embd/16], and the position left to the word-score launch
    int8_t *q8k_q;
    float *q8k_d;
    int16_t *q8k_b;
};

// the word scores of a Q6_K word table for ncol inputs cut per 256 values, with the first-maximum pick and the
// end-of-step bookkeeping of the word-table read (k_q6k_head)
struct Q6HeadArgs {
    const Col *cols_d;
    int ncol;
    const uint8_t *W;                 // rows of nb 210-byte blocks
    int rows, nb;
    const int8_t *xq;                 // [c][256 nb]
    const float *xd;                  // [c][nb]
    const int16_t *xb;                // [c][16 nb]
    unsigned *done;                   // CTAs finished (the last one picks and resets it)
    unsigned long long *trace;
};

// ---- shared-memory plan of the table-read kernel (host and device agree on it) ----
// fs: integer block dots as floats, [MV_NBUF][nc][sr][nb+4]; dd: block scales (fp16 bits), [MV_NBUF][sr][nb+4];
// vb: prologue vectors [nc][vb_len] (overlapping fs/dd); pc: per-column facts read before the dependency wait;
// red: reductions and argmax partials.
struct PreCol {
    const SessDev *s;
    float *ring;
    const float *embd;
    int pos, off, tok, pad;
};
struct MvPlan {
    int stage, sstride, bar, xq, xd, xs, fs, dd, vb, vo, ab, pc, red, total;
};
__host__ __device__ inline int align_up(int x, int a) { return (x + a - 1) / a * a; }
// hm: Q4_1 rows (a minimum per block besides the scale): the scale buffers hold the minimums in a second half
__host__ __device__ inline MvPlan mv_plan(int cols, int sr, int nc, int vb_len, int ab_len, int ns, int hm = 0) {
    MvPlan p;
    const int nb = cols / 32, ld = nb + 4;   // row strides: 16-byte aligned, conflict-free for vector loads
    int o = 0;
    // weight stages sized to their rows (a stage holds sr rows of at most MV_STAGE_BYTES): where the block-dot buffers
    // leave few rows per stage (8 inputs), more stages stay in flight
    p.sstride = align_up(sr * (cols / 32) * (hm ? 20 : 18), 128);
    p.stage = o; o += ns * p.sstride;
    p.bar = o;   o = align_up(o + 8 * MV_MAX_STAGES, 16);
    p.xq = o;    o = align_up(o + nc * cols, 16);
    p.xd = o;    o = align_up(o + 4 * nc * nb, 16);
    p.xs = o;    o = align_up(o + 4 * nc * nb, 16);
    // the prologue's vectors (vb) are dead before the first block dot is stored: they share the dot buffers' space
    const int u = o;
    p.fs = o;    o = align_up(o + MV_NBUF * 4 * nc * sr * ld, 16);
    p.dd = o;    o = align_up(o + (hm ? 2 : 1) * MV_NBUF * 2 * sr * ld, 16);
    p.vo = o;
    p.vb = u;    o = o > align_up(u + 4 * nc * vb_len, 16) ? o : align_up(u + 4 * nc * vb_len, 16);
    p.ab = o;    o = align_up(o + 4 * nc * ab_len, 16);
    p.pc = o;    o = align_up(o + (int) sizeof(PreCol) * MV_MAX_COLS, 16);
    p.red = o;   o = align_up(o + 4 * 64 + 8 * MV_MAX_COLS * MV_CWARPS + 16, 16);
    p.total = o;
    return p;
}

// floats per column staged in shared memory by the input preparation of `pro`
__host__ __device__ inline int mv_vb_len(int pro, int cols, int n_embd, int nc, int d_conv) {
    // P_RESID_NORM / P_FINAL stage two vectors per column (the post-normed input and the residual) for up to 2
    // columns; with more, the residual is read from global memory where it is used. P_CONV keeps, for up to 2
    // columns, the product of every tap made before the dependency wait: [d_conv][n_embd].
    return pro == P_CUT ? cols : (pro == P_RESID_NORM || pro == P_FINAL) ? (nc <= 2 ? 2 : 1) * n_embd
                               : pro == P_EMBED_NORM ? n_embd : pro == P_CONV ? (nc <= 2 ? d_conv : 0) * n_embd : 0;
}

// the column-count instance a launch of ncol inputs runs (1, 2, 4 or 8; 0: too many)
__host__ __device__ inline int mv_nc_slot(int ncol) {
    return ncol <= 1 ? 1 : ncol <= 2 ? 2 : ncol <= 4 ? 4 : ncol <= MV_MAX_COLS ? 8 : 0;
}

// rows per weight stage (a.sr) and stages in flight (a.nstage) of one table read of `grid` CTAs: full stages (at most
// 64 rows of one MV_STAGE_BYTES stage) and as many of them as a CTA's slice needs (up to MV_MAX_STAGES), within one
// CTA's shared memory (MV_SMEM_BUDGET); fewer stages first (down to 2), then fewer rows per stage. Stages hold a
// multiple of `gran` rows. a.rows, cols, row_bytes, unit, ncol, n_embd, ab_len, d_conv and has_m must be set (the
// engine's table_launch sets them). Returns the plan's shared-memory bytes (0: nothing fits; a.sr = gran and
// a.nstage = 1 then, and the launch reports the excess).
inline int mv_plan_stages(MvArgs &a, int pro, int gran, int grid) {
    const int nc = mv_nc_slot(a.ncol), units = a.rows / a.unit, rows_cta = (units + grid - 1) / grid * a.unit;
    const int cap = MV_STAGE_BYTES / a.row_bytes < 64 ? MV_STAGE_BYTES / a.row_bytes : 64;
    const int full = cap / gran * gran > gran ? cap / gran * gran : gran;
    const int vb = mv_vb_len(pro, a.cols, a.n_embd, nc, a.d_conv);
    for (int sr = full; sr >= gran; sr -= gran) {
        const int nst = (rows_cta + sr - 1) / sr > 1 ? (rows_cta + sr - 1) / sr : 1;
        for (int ns = nst < MV_MAX_STAGES ? nst : MV_MAX_STAGES; ns >= (nst < 2 ? nst : 2); ns--) {
            const int total = mv_plan(a.cols, sr, nc, vb, a.ab_len, ns, a.has_m).total;
            if (total <= MV_SMEM_BUDGET) {
                a.sr = sr;
                a.nstage = ns;
                return total;
            }
        }
    }
    a.sr = gran;
    a.nstage = 1;
    return 0;
}

#ifdef __CUDACC__
// ---------------- exact scalar helpers ----------------
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float exp_cr(float x) { return __double2float_rn(exp((double) x)); }

// imi_rms_scale's AVX2 order (vec.h:20-28) for a vector in shared memory, n a multiple of 32, computed by ONE warp:
// lane L accumulates x[L], x[L+32], ... with fma (the 4 x 8 lanes a0..a3), then (a0+a1)+(a2+a3) per lane of 8,
// then imi_hsum's tree ((t0+t4)+(t2+t6)) + ((t1+t5)+(t3+t7)) (vec.h:12-16). Returns 1/sqrt(s/n + eps) to all lanes.
__device__ __forceinline__ float warp_rms_scale(const float *x, int n, float eps) {
    const int L = threadIdx.x & 31;
    float a = 0.0f;
    int i = L;
    if (i + 15 * 32 < n) {
        float v[16];
#pragma unroll
        for (int k = 0; k < 16; k++) v[k] = x[i + 32 * k];
        for (; i + 15 * 32 < n; i += 16 * 32) {   // the next 16 values load while these 16 accumulate, in order
            float w[16];
            const bool more = i + 16 * 32 + 15 * 32 < n;
#pragma unroll
            for (int k = 0; k < 16; k++) w[k] = more ? x[i + 16 * 32 + 32 * k] : 0.0f;
#pragma unroll
            for (int k = 0; k < 16; k++) a = __fmaf_rn(v[k], v[k], a);
#pragma unroll
            for (int k = 0; k < 16; k++) v[k] = w[k];
        }
    }
    for (; i < n; i += 32) a = __fmaf_rn(x[i], x[i], a);
    const unsigned F = 0xffffffffu;
    const float a8 = __shfl_down_sync(F, a, 8), a16 = __shfl_down_sync(F, a, 16), a24 = __shfl_down_sync(F, a, 24);
    const float t = __fadd_rn(__fadd_rn(a, a8), __fadd_rn(a16, a24));   // lanes 0..7
    const float r = __fadd_rn(t, __shfl_down_sync(F, t, 4));             // lanes 0..3: t_m + t_{m+4}
    const float q = __fadd_rn(r, __shfl_down_sync(F, r, 2));             // lane 0: r0+r2, lane 1: r1+r3
    const float s = __fadd_rn(q, __shfl_down_sync(F, q, 1));             // lane 0
    const float s0 = __shfl_sync(F, s, 0);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s0, (float) n), eps)));
}

// imi_cut32 (vec.h:47-77) of one 32-value block held one value per lane: d = max|x|/127, id = 1/d (0 if d == 0),
// q = round-half-even(x * id); returns q; d and the code sum go to lane-uniform outputs.
__device__ __forceinline__ int warp_cut32(float v, float &d, int &sum) {
    const unsigned F = 0xffffffffu;
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(F, amax, o));
    d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q = __float2int_rn(__fmul_rn(v, id));
    int s = q;
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(F, s, o);
    sum = s;
    return q;
}

// imi_cut32 of one 32-value block held by 8 consecutive lanes (lane & 7 = g holds values 4g..4g+3): the same
// d, id, codes and sum as warp_cut32. Every lane of the warp calls it (each group of 8 reduces among itself).
// Returns this lane's 4 codes packed in a word (value 4g in the low byte); d and the block's code sum to every lane.
__device__ __forceinline__ uint32_t cut32_g8(float4 v, float &d, int &sum) {
    const unsigned F = 0xffffffffu;
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    amax = fmaxf(amax, __shfl_xor_sync(F, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(F, amax, 2));
    amax = fmaxf(amax, __shfl_xor_sync(F, amax, 4));
    d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q0 = __float2int_rn(__fmul_rn(v.x, id)), q1 = __float2int_rn(__fmul_rn(v.y, id)),
              q2 = __float2int_rn(__fmul_rn(v.z, id)), q3 = __float2int_rn(__fmul_rn(v.w, id));
    int s = (q0 + q1) + (q2 + q3);
    s += __shfl_xor_sync(F, s, 1);
    s += __shfl_xor_sync(F, s, 2);
    s += __shfl_xor_sync(F, s, 4);
    sum = s;
    return ((uint32_t) q0 & 0xffu) | (((uint32_t) q1 & 0xffu) << 8) | (((uint32_t) q2 & 0xffu) << 16) |
           ((uint32_t) q3 << 24);
}
// cut32_g8 of chunk q (values 4q..4q+3) with the results stored when `act`: codes at q8 + 4q, the block's scale
// and scale * code sum at d[q / 8], s[q / 8] (written by lane g == 0). All 32 lanes call it.
__device__ __forceinline__ void cut_chunk(float4 v, bool act, int q, int8_t *q8, float *d, float *s) {
    float dv;
    int sum;
    const uint32_t w = cut32_g8(act ? v : make_float4(0.0f, 0.0f, 0.0f, 0.0f), dv, sum);
    if (act) {
        *(uint32_t *) (q8 + 4 * q) = w;
        if ((q & 7) == 0) {
            d[q >> 3] = dv;
            s[q >> 3] = __fmul_rn(dv, (float) sum);
        }
    }
}

// dot_h of seoul.cpp:29-35: 8 lane accumulators over the row in steps of 8, then imi_hsum's order.
// q: floats (shared), k: one row of n fp16 loaded as uint4 (8 values each).
template <int D>
__device__ __forceinline__ float dot_h8(const float *q, const uint4 *k) {
    float a[8];
#pragma unroll
    for (int l = 0; l < 8; l++) a[l] = 0.0f;
#pragma unroll
    for (int w = 0; w < D / 8; w++) {
        const uint4 v = k[w];
        const uint32_t u[4] = { v.x, v.y, v.z, v.w };
#pragma unroll
        for (int h = 0; h < 4; h++) {
            a[2 * h] = __fmaf_rn(q[8 * w + 2 * h], h2f((uint16_t) (u[h] & 0xffff)), a[2 * h]);
            a[2 * h + 1] = __fmaf_rn(q[8 * w + 2 * h + 1], h2f((uint16_t) (u[h] >> 16)), a[2 * h + 1]);
        }
    }
    const float r0 = __fadd_rn(a[0], a[4]), r1 = __fadd_rn(a[1], a[5]), r2 = __fadd_rn(a[2], a[6]),
                r3 = __fadd_rn(a[3], a[7]);
    return __fadd_rn(__fadd_rn(r0, r2), __fadd_rn(r1, r3));
}

// ---------------- PTX wrappers: mbarrier, bulk async copy, programmatic dependent launch ----------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t) __cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait (by default about one second at the boost clock): false if the phase never completed
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, long long limit = 2000000000LL) {
    const long long t0 = clock64();
    while (!mbar_try_wait(b, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}
// a 2D tensor copy (TMA) of one box at element coordinates (x, y) into shared memory, completing on an mbarrier; the
// tensor map lives in global, constant or parameter memory (x times the element size a multiple of 16 bytes)
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
// global -> shared bulk copy completing on an mbarrier (addresses 16-byte aligned, bytes a multiple of 16)
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// bulk prefetch of global memory into L2 (16-byte aligned address, size a multiple of 16)
__device__ __forceinline__ void prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// 16-byte global -> shared copy without registers (cp.async, L2 only: the source may be fresh from the last launch)
__device__ __forceinline__ void cp16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// a coherent (L2) read of a value another launch may change (no compiler barrier: loads that do not depend on it
// may be issued beside it; it stays after the dependency wait, another volatile asm)
__device__ __forceinline__ int ld_relaxed(const int *p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

}  // namespace imi

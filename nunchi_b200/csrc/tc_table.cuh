// k_tc_table: one 4-bit table times many inputs (16..256 columns) on the 5th-generation tensor cores: the batched
// read of imi_q8b + imi_q4_group_batch (imi/core/tables.cpp:405-477), used where a step reads a table for dozens of
// conversations or prefill positions at once.
//
// The tensor cores compute imi's per-block integer dots exactly: for a 32-value block j the dot sum_i code_ri * x_ci
// of 4-bit codes (0..15) and 8-bit input codes (-127..127) is an integer below 2^16 in magnitude, and the int8 MMA
// (kind::i8, both operands s8, int32 accumulator) forms it with one instruction per block (K = 32). imi scales each
// block's dot before it accumulates, so the MMA must not sum over blocks: every block gets its own TMEM columns
// (D_j[row][col] = dot of block j), and the epilogue runs imi's two float chains per (row, column) in block order
// (group_avx2<false>, tables.cpp:127-143):
//     acc = fma(dot_j, d_rj * dx_cj, acc),  cor = fma(d_rj, s_cj, cor),  out = acc - 8 cor (one rounding).
//
// The weights come from the table's tiled copy (made once at load by k_tc_tile): for every tile of 128 rows and stage
// of 128 values one contiguous TC_WSTAGE-byte block holding the codes already as 8-bit values in the MMA's canonical
// K-major layout (8-row x 16-byte core matrices; chunk 2p of block p holds its values 0..15, chunk 2p+1 its values
// 16..31) and then the rows' fp16 block scales. A stage is thus one bulk copy that the MMA reads where it lands (a
// row-wise tensor copy of the row-major table moved only ~14 GB/s per SM: 128 separate 80-byte rows per stage).
//
// Work unit: a tile of 128 rows x a group of G columns (G = 16, 32 or 64). Warp roles (one CTA per SM, persistent
// over units):
//   warp 0      producer: per ring slot (TC_CP stages) one barrier for two bulk copies (the tile's weight stages, the
//               columns' 8-bit codes in the MMA's K-major layout with their scales and sums); it waits only for the
//               slot, so bytes stream up to the ring's depth ahead of the math;
//   warp 1      TMEM owner (512 columns) and MMA issuer: per block one tcgen05.mma kind::i8 (K = 32) into the block's
//               own TMEM columns; the 4 blocks of a stage fill one TMEM stage slot, committed to its barrier once (a
//               commit-to-wait hand-off costs about 0.3 us, so it is made per stage, not per block);
//   warps 2..   epilogue, 4 per 8 or 16 columns (tc_ch): per TMEM slot tcgen05.ld of the blocks' dots, up to 4
//               blocks per wait (warp w reads lanes 32 (w % 4) ..), converted to float exactly, the rows' scales and
//               the columns' scales and sums read from the ring slot, the two fma chains per column (packed f32x2
//               operations, each lane rounded as imi's scalar chain), the result stored at the end of the unit; the
//               slot is released when the MMAs and every epilogue warp are done with it.
// Every wait on an mbarrier is bounded (about one second); a wait that gives up sets the error flag, the CTA stops
// issuing work, waits (bounded) for its copies and MMAs in flight, frees its TMEM and returns.
#pragma once
#include "common.cuh"

namespace imi {

constexpr int TC_M = 128;              // rows per tile (the MMA's M; TMEM lanes)
constexpr int TC_KS = 128;             // values per K stage
constexpr int TC_BPS = TC_KS / 32;     // blocks per stage
// bytes of one (tile, stage) block of a table's tiled copy: 8-bit codes [TC_KS / 16][TC_M][16], fp16 scales [TC_M][4]
constexpr int TC_WCODES = TC_KS * TC_M, TC_WSTAGE = TC_WCODES + TC_M * TC_BPS * 2;
// a ring slot holds TC_CP stages fetched by two bulk copies: their weights (contiguous in the tiled copy) and the
// columns' operand (contiguous in its layout, codes and scales interleaved per stage). Fewer, larger copies stream
// faster on their own (one CTA completes a copy about every 0.3 us: 10 KB copies ~31 GB/s per SM, 40 KB ones ~85),
// but two stages per slot made the 64-session step 1.5% slower than one (3.19-3.23 against 3.14-3.15 ms): a slot
// frees only when both of its stages are done
constexpr int TC_CP = 1;
// ring slots: as many as shared memory holds, TC_NR_MIN..TC_NR_MAX
constexpr int TC_NR_MIN = 2, TC_NR_MAX = 12;
constexpr int TC_SMEM = 220 * 1024;   // dynamic shared memory of one CTA at most
constexpr int TC_WARP_PROD = 0, TC_WARP_MMA = 1, TC_WARP_EPI = 2;
// columns per epilogue thread: 8 in groups of 16 or 32 columns (more warps to hide the TMEM and shared-memory
// latencies of the chains), 16 in groups of 64 (the thread count stays within one CTA's)
__host__ __device__ constexpr int tc_ch(int G) { return G >= 64 ? 16 : 8; }
// epilogue warps: 4 per tc_ch(G) columns (one per TMEM lane quarter)
__host__ __device__ constexpr int tc_epi_warps(int G) { return 4 * (G / tc_ch(G)); }
__host__ __device__ constexpr int tc_threads(int G) { return 32 * (TC_WARP_EPI + tc_epi_warps(G)); }
constexpr int TC_TMEM_COLS = 512;

// output stage: TE_STORE out[c][row]; TE_SILU rows (2i, 2i+1) are (gate_i, up_i) of an interleaved gate/up table:
// out[c][i] = silu(gate) * up (seoul.cpp:384-391); TE_HEAD word scores into each column's logits (when it has them)
// and imi's greedy pick (first maximum, lowest id on ties), ending the step as the small-batch word-table read does
enum TcEpi : int { TE_STORE = 0, TE_SILU = 1, TE_HEAD = 2 };

// the columns' operand of one group (G columns) and stage (TC_KS values): the 8-bit codes [TC_KS / 16][G][16] in the
// MMA's K-major layout, then per block of the stage the G scales and the G scale * code sums, [TC_BPS][2][G] floats;
// stages follow one another per group: [group][cols / TC_KS][tc_xb_bytes(G)]
__host__ __device__ constexpr int tc_xb_codes(int G) { return TC_KS / 16 * G * 16; }
__host__ __device__ constexpr int tc_xb_bytes(int G) { return tc_xb_codes(G) + TC_BPS * 2 * G * 4; }
// byte offsets in the operand: value k of column cg of group g; block j's scale (h = 0) or scale * code sum (h = 1)
__host__ __device__ inline size_t tc_xb_code(int G, int K, int g, int cg, int k) {
    return ((size_t) g * (K / TC_KS) + k / TC_KS) * tc_xb_bytes(G) + ((size_t) ((k % TC_KS) / 16) * G + cg) * 16 + k % 16;
}
__host__ __device__ inline size_t tc_xb_scale(int G, int K, int g, int cg, int j, int h) {
    return ((size_t) g * (K / TC_KS) + j / TC_BPS) * tc_xb_bytes(G) + tc_xb_codes(G) +
           ((size_t) ((j % TC_BPS) * 2 + h) * G + cg) * 4;
}

struct TcArgs {
    const uint8_t *wt;        // the table's tiled copy: [tiles][cols / TC_KS] blocks of TC_WSTAGE bytes (k_tc_tile)
    int rows, cols;           // cols a multiple of TC_CP * TC_KS
    int ncol, G, groups;      // columns, columns per group, groups (units = tiles * groups)
    const uint8_t *xb;        // the columns' operand, [group][cols / TC_KS][tc_xb_bytes(G)]
    float *out;               // out[c * out_stride + row]
    int out_stride;
    int epi;
    const Col *cols_d;        // TE_HEAD: the columns (logits, conversation records)
    unsigned *done;           // TE_HEAD: CTAs finished (the last one picks and resets it)
    int *err;
    unsigned long long *trace;   // optional (diagnostics): CTA 0's timeline, [TC_TRACE_ROWS][64] ns (imi_cuda_trace_tc)
};
constexpr int TC_TRACE = 64, TC_TRACE_ROWS = 9;

// bytes of a table's tiled copy
__host__ __device__ inline size_t tc_tiled_bytes(int rows, int cols) {
    return (size_t) ((rows + TC_M - 1) / TC_M) * (cols / TC_KS) * TC_WSTAGE;
}

struct TcPlan {
    int raw, bar, tptr, total;
    int raw_bytes, raw_stride, op_off, xb, nslot;   // op_off: the operand in a slot; xb: its bytes per stage
    int nr;   // ring slots (TC_CP stages each)
};
// a ring slot: [the TC_CP weight stages (TC_WSTAGE each) | the TC_CP stages of the columns' operand]
__host__ __device__ inline TcPlan tc_plan(int G) {
    TcPlan p;
    p.xb = tc_xb_bytes(G);
    p.op_off = TC_CP * TC_WSTAGE;
    p.raw_bytes = p.op_off + TC_CP * p.xb;
    p.raw_stride = align_up(p.raw_bytes, 128);
    p.nslot = TC_TMEM_COLS / (G * TC_BPS);               // TMEM stage slots: a stage's 4 blocks, G columns each
    const int fixed = 8 * (2 * TC_NR_MAX + 2 * 32 + 1) + 16 + 256;
    p.nr = (TC_SMEM - fixed) / p.raw_stride;
    p.nr = p.nr < TC_NR_MIN ? TC_NR_MIN : p.nr > TC_NR_MAX ? TC_NR_MAX : p.nr;
    int o = 0;
    p.raw = o;  o += p.nr * p.raw_stride;
    p.bar = o;  o += 8 * (2 * TC_NR_MAX + 2 * 32 + 1);
    p.tptr = o; o += 16;
    p.total = align_up(o, 128) + 128;                     // + slack to align the base to 128 bytes
    return p;
}

#if defined(__CUDACC__) && defined(IMI_KERNELS)   // device code: compiled in kernels.cu only
// the tiled copy of a table (engine row layout: [cols / 2 code bytes | cols / 32 fp16 scales] per row) for the
// tensor-core read: for tile t and stage s, at ((t * (cols / TC_KS)) + s) * TC_WSTAGE, the 8-bit codes
// [TC_KS / 16][TC_M][16] (chunk 2p: the low nibbles of block p's 16 code bytes = its values 0..15; chunk 2p + 1: the
// high nibbles = values 16..31) then the rows' 4 fp16 block scales [TC_M][4]; rows past the table's end are zeros.
// One thread per (tile, stage, row).
__global__ void k_tc_tile(const uint8_t *W, int rows, int cols, int row_bytes, uint8_t *dst) {
    const int nst = cols / TC_KS, tiles = (rows + TC_M - 1) / TC_M;
    const long long n = (long long) tiles * nst * TC_M;
    constexpr uint32_t LO = 0x0F0F0F0Fu;
    for (long long idx = blockIdx.x * (long long) blockDim.x + threadIdx.x; idx < n;
         idx += (long long) gridDim.x * blockDim.x) {
        const int row = (int) (idx % TC_M);
        const long long ts = idx / TC_M;
        const int s = (int) (ts % nst), grow = (int) (ts / nst) * TC_M + row;
        uint8_t *o = dst + ts * TC_WSTAGE;
        uint4 c[TC_BPS];
        uint2 sc = make_uint2(0u, 0u);
#pragma unroll
        for (int p = 0; p < TC_BPS; p++) c[p] = make_uint4(0u, 0u, 0u, 0u);
        if (grow < rows) {
            const uint8_t *src = W + (size_t) grow * row_bytes;
#pragma unroll
            for (int p = 0; p < TC_BPS; p++) c[p] = *(const uint4 *) (src + 16 * (TC_BPS * s + p));
            sc = *(const uint2 *) (src + cols / 2 + 2 * TC_BPS * s);
        }
#pragma unroll
        for (int p = 0; p < TC_BPS; p++) {
            *(uint4 *) (o + ((2 * p) * TC_M + row) * 16) = make_uint4(c[p].x & LO, c[p].y & LO, c[p].z & LO, c[p].w & LO);
            *(uint4 *) (o + ((2 * p + 1) * TC_M + row) * 16) =
                make_uint4((c[p].x >> 4) & LO, (c[p].y >> 4) & LO, (c[p].z >> 4) & LO, (c[p].w >> 4) & LO);
        }
        *(uint2 *) (o + TC_WCODES + row * 8) = sc;
    }
}

// ---- tcgen05 wrappers ----
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b))
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
// D[tmem] = A[smem] . B[smem]^T, kind::i8 (s8 inputs, s32 result; K = 32), not accumulated
__device__ __forceinline__ void tc_mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0)
        : "memory");
}
// shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices, lbo between the two 16-byte K
// chunks of an MMA, sbo between 8-row groups (tcgen05 descriptor: start >> 4, lbo >> 4 at bit 16, sbo >> 4 at bit 32,
// version 1 at bit 46, layout 0 = no swizzle at bits 61-63)
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFF) | ((uint64_t) ((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// instruction descriptor of kind::i8: D s32 (2 at bit 4), A and B signed 8-bit (1 at bits 7 and 10), both K-major,
// N >> 3 at bit 17, M >> 4 at bit 24
__host__ __device__ constexpr uint32_t tc_idesc_i8(int n, int m) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (m >> 4) << 24);
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&v)[N]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t t, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(t));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t t, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                   "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(t));
}
template <>
__device__ __forceinline__ void tmem_ld<32>(uint32_t t, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(t));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// an int32 dot below 2^22 in magnitude as float, exactly: its bits added to those of 1.5 * 2^23 make the float
// 1.5 * 2^23 + dot (an integer in [2^23, 2^24)), from which 1.5 * 2^23 is subtracted without rounding
__device__ __forceinline__ float2 dots_f2(uint32_t a, uint32_t b) {
    const float2 v = make_float2(__uint_as_float(a + 0x4B400000u), __uint_as_float(b + 0x4B400000u));
    return __fadd2_rn(v, make_float2(-12582912.0f, -12582912.0f));
}

template <int G>
__global__ void __launch_bounds__(tc_threads(G), 1) k_tc_table(const __grid_constant__ TcArgs a) {
    extern __shared__ __align__(128) uint8_t smt[];
    // NLD: blocks loaded per TMEM wait (4 at 8 columns a thread; 1 at 16, where the registers of a CTA this wide
    // hold one block's dots beside the chains)
    constexpr int CH = tc_ch(G), NEW = tc_epi_warps(G), NLD = CH == 8 ? 4 : 1;
    const TcPlan P = tc_plan(G);
    uint8_t *sm = smt + ((128 - (smem_u32(smt) & 127)) & 127);
    uint64_t *bars = (uint64_t *) (sm + P.bar);
    // raw_full: the copies of a stage landed (1 arrival + bytes); raw_empty: read by the MMAs (1 commit) and by every
    // epilogue warp; tm_full, fin: tcgen05.commit; tm_empty: the epilogue warps
    uint64_t *raw_full = bars, *raw_empty = raw_full + TC_NR_MAX, *tm_full = raw_empty + TC_NR_MAX,
             *tm_empty = tm_full + 32, *fin = tm_empty + 32;
    uint32_t *tptr = (uint32_t *) (sm + P.tptr);
    __shared__ int abort_flag, last_cta;
    __shared__ unsigned long long best[256];   // TE_HEAD: this CTA's best key per column
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (a.epi == TE_HEAD)
        for (int k = tid; k < 256; k += blockDim.x) best[k] = 0ull;
    const int K = a.cols, nst = K / TC_KS, tiles = (a.rows + TC_M - 1) / TC_M, units = tiles * a.groups;
    const int nslot = P.nslot, NR = P.nr;

    if (tid == 0) {
        for (int i = 0; i < NR; i++) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 1 + NEW); }
        for (int i = 0; i < nslot; i++) { mbar_init(&tm_full[i], 1); mbar_init(&tm_empty[i], NEW); }
        mbar_init(fin, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == TC_WARP_MMA) {   // the whole warp allocates the 512 TMEM columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tptr)),
                     "r"(TC_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tptr;
    pdl_trigger();

    auto fail = [&]() {
        abort_flag = 1;
        atomicExch(a.err, 7);
    };
    auto wait = [&](uint64_t *b, uint32_t parity) -> bool {
        if (*(volatile int *) &abort_flag) return false;
        if (mbar_wait(b, parity)) return true;
        fail();
        return false;
    };
    // the same wait by every lane of a warp, one outcome for all (a lane that gave up fails the warp)
    auto wait_warp = [&](uint64_t *b, uint32_t parity) -> bool { return __all_sync(0xffffffffu, wait(b, parity)); };
    auto raw_at = [&](int r) { return sm + P.raw + r * P.raw_stride; };

    // producer and MMA issuer: the whole warp runs the role's loop and waits (its control flow stays converged), lane 0
    // issues the copies, the MMAs and the commits
    if (warp == TC_WARP_PROD) {
        // ---------------- producer ----------------
        // before the dependency wait: the weights of the first unit's first slots (they do not depend on the launches
        // in flight; the columns' operand does), so they stream while the previous launch finishes
        const int pre = blockIdx.x < units ? min(NR, nst / TC_CP) : 0;
        if (lane == 0 && pre > 0) {
            const uint8_t *wt = a.wt + (size_t) (blockIdx.x / a.groups) * nst * TC_WSTAGE;
            for (int k = 0; k < pre; k++) {
                mbar_expect_tx(&raw_full[k], (uint32_t) P.raw_bytes);   // both copies of the slot
                bulk_g2s(raw_at(k), wt + (size_t) k * TC_CP * TC_WSTAGE, (uint32_t) (TC_CP * TC_WSTAGE), &raw_full[k]);
            }
        }
        pdl_wait();
        int i = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const int tile = u / a.groups, g = u - tile * a.groups;
            const uint8_t *wt = a.wt + (size_t) tile * nst * TC_WSTAGE;
            const uint8_t *xb = a.xb + (size_t) g * nst * P.xb;
            for (int s = 0; s < nst; s += TC_CP, i++) {   // i: slots filled
                const int r = i % NR;
                if (i < pre) {   // its weights are on their way: the operand only
                    if (lane == 0) bulk_g2s(raw_at(r) + P.op_off, xb + (size_t) s * P.xb, (uint32_t) (TC_CP * P.xb), &raw_full[r]);
                    __syncwarp();
                    continue;
                }
                if (!(ok = wait_warp(&raw_empty[r], ((i / NR) & 1) ^ 1))) break;
                if (lane == 0) {
                    uint8_t *raw = raw_at(r);
                    mbar_expect_tx(&raw_full[r], (uint32_t) P.raw_bytes);
                    bulk_g2s(raw, wt + (size_t) s * TC_WSTAGE, (uint32_t) (TC_CP * TC_WSTAGE), &raw_full[r]);
                    bulk_g2s(raw + P.op_off, xb + (size_t) s * P.xb, (uint32_t) (TC_CP * P.xb), &raw_full[r]);
                    if (a.trace && blockIdx.x == 0 && i < TC_TRACE) a.trace[0 * TC_TRACE + i] = global_ns();
                }
                __syncwarp();
            }
        }
        if (!ok && lane == 0)   // the copies in flight land before the CTA exits (bounded waits on the last slots filled)
            for (int k = i > NR ? i - NR : 0; k < i; k++) mbar_wait(&raw_full[k % NR], (k / NR) & 1);
    } else if (warp == TC_WARP_MMA) {
        // ---------------- MMA issuer ----------------
        pdl_wait();
        const uint32_t idesc = tc_idesc_i8(G, TC_M);
        int i = 0, b = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            for (int s = 0; s < nst && ok; s++, i++) {   // i: stages; stage i sits in slot (i / TC_CP) % NR
                const int q = i / TC_CP, sub = i % TC_CP, r = q % NR, slot = i % nslot;
                if (!(ok = wait_warp(&raw_full[r], (q / NR) & 1))) break;
                if (lane == 0 && a.trace && blockIdx.x == 0 && i < TC_TRACE) a.trace[7 * TC_TRACE + i] = global_ns();
                if (!(ok = wait_warp(&tm_empty[slot], ((i / nslot) & 1) ^ 1))) break;
                if (lane == 0 && a.trace && blockIdx.x == 0 && i < TC_TRACE) a.trace[8 * TC_TRACE + i] = global_ns();
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t abase = smem_u32(raw_at(r)) + sub * TC_WSTAGE,
                                   bbase = smem_u32(raw_at(r)) + P.op_off + sub * P.xb;
                    for (int jj = 0; jj < TC_BPS; jj++) {   // block jj: 16-byte chunks 2jj, 2jj + 1
                        tc_mma_i8(tmem + (slot * TC_BPS + jj) * G, tc_desc(abase + 2 * jj * TC_M * 16, TC_M * 16, 128),
                                  tc_desc(bbase + 2 * jj * G * 16, G * 16, 128), idesc);
                        if (a.trace && blockIdx.x == 0 && b + jj < TC_TRACE) a.trace[3 * TC_TRACE + b + jj] = global_ns();
                    }
                    tc_commit(&tm_full[slot]);
                    if (sub == TC_CP - 1) tc_commit(&raw_empty[r]);   // the slot's last stage
                }
                b += TC_BPS;
                __syncwarp();
            }
        }
        if (!ok && lane == 0) {   // the MMAs issued complete before TMEM is freed
            tc_commit(fin);
            mbar_wait(fin, 0);
        }
    } else {
        // ---------------- epilogue: imi's float chains per (row, column) ----------------
        pdl_wait();
        const int qd = warp & 3, h = (warp - TC_WARP_EPI) >> 2, row = qd * 32 + lane;
        const uint32_t tl = tmem + ((uint32_t) (qd * 32) << 16) + h * CH;
        int i = 0, b = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            const int tile = u / a.groups, g = u - tile * a.groups;
            float2 acc[CH / 2], cor[CH / 2];
#pragma unroll
            for (int k = 0; k < CH / 2; k++) acc[k] = cor[k] = make_float2(0.0f, 0.0f);
            for (int s = 0; s < nst && ok; s++, i++) {
                const int q = i / TC_CP, sub = i % TC_CP, r = q % NR, slot = i % nslot;
                // the slot's copies (this warp reads their scales) and the stage's MMAs
                if (!(ok = wait_warp(&raw_full[r], (q / NR) & 1) && wait_warp(&tm_full[slot], (i / nslot) & 1))) break;
                tc_fence_after();
                const uint8_t *ep = raw_at(r);
                const uint2 dq = *(const uint2 *) (ep + sub * TC_WSTAGE + TC_WCODES + row * 8);   // the row's 4 block scales
                const uint16_t dsc[4] = { (uint16_t) (dq.x & 0xffff), (uint16_t) (dq.x >> 16), (uint16_t) (dq.y & 0xffff),
                                          (uint16_t) (dq.y >> 16) };
                const float *xds = (const float *) (ep + P.op_off + sub * P.xb + tc_xb_codes(G));
                for (int j0 = 0; j0 < TC_BPS; j0 += NLD) {
                    const bool tr = a.trace && blockIdx.x == 0 && warp == TC_WARP_EPI && lane == 0 && b < TC_TRACE;
                    if (tr) a.trace[4 * TC_TRACE + b] = global_ns();
                    uint32_t f[NLD][CH];
#pragma unroll
                    for (int u2 = 0; u2 < NLD; u2++) tmem_ld<CH>(tl + (slot * TC_BPS + j0 + u2) * G, f[u2]);
                    tmem_ld_wait();
                    if (tr) a.trace[6 * TC_TRACE + b] = global_ns() + (unsigned long long) (f[0][0] & 0);
#pragma unroll
                    for (int u2 = 0; u2 < NLD; u2++, b++) {
                        const int jj = j0 + u2;
                        const float d = h2f(dsc[jj]);
                        const float2 dd = make_float2(d, d);
                        const float4 *xd = (const float4 *) (xds + jj * 2 * G + h * CH),
                                     *xs = (const float4 *) (xds + jj * 2 * G + G + h * CH);
#pragma unroll
                        for (int k = 0; k < CH / 4; k++) {   // 4 columns per pair of 16-byte loads
                            const float4 dx = xd[k], sx = xs[k];
                            const float2 f0 = dots_f2(f[u2][4 * k], f[u2][4 * k + 1]),
                                         f1 = dots_f2(f[u2][4 * k + 2], f[u2][4 * k + 3]);
                            acc[2 * k] = __ffma2_rn(f0, __fmul2_rn(dd, make_float2(dx.x, dx.y)), acc[2 * k]);
                            acc[2 * k + 1] = __ffma2_rn(f1, __fmul2_rn(dd, make_float2(dx.z, dx.w)), acc[2 * k + 1]);
                            cor[2 * k] = __ffma2_rn(dd, make_float2(sx.x, sx.y), cor[2 * k]);
                            cor[2 * k + 1] = __ffma2_rn(dd, make_float2(sx.z, sx.w), cor[2 * k + 1]);
                        }
                    }
                    if (tr) a.trace[5 * TC_TRACE + b - NLD] = global_ns() + (unsigned long long) (__float_as_uint(acc[0].x) & 0);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tm_empty[slot]);
                    if (sub == TC_CP - 1) mbar_arrive(&raw_empty[r]);
                }
                if (a.trace && blockIdx.x == 0 && lane == 0 && i < TC_TRACE) atomicMax(&a.trace[2 * TC_TRACE + i], global_ns());
            }
            if (!ok) break;
            const int grow = tile * TC_M + row;
            const bool live = grow < a.rows;
#pragma unroll
            for (int k = 0; k < CH; k++) {
                const int cc = g * G + h * CH + k;
                const float v = (k & 1) ? __fmaf_rn(-8.0f, cor[k / 2].y, acc[k / 2].y) : __fmaf_rn(-8.0f, cor[k / 2].x, acc[k / 2].x);
                if (a.epi == TE_STORE) {
                    if (live && cc < a.ncol) a.out[(size_t) cc * a.out_stride + grow] = v;
                } else if (a.epi == TE_SILU) {   // the up row is the next lane's
                    const float up = __shfl_down_sync(0xffffffffu, v, 1);
                    if (live && (grow & 1) == 0 && cc < a.ncol) {
                        const float sl = __fdiv_rn(v, __fadd_rn(1.0f, exp_cr(-v)));
                        a.out[(size_t) cc * a.out_stride + grow / 2] = __fmul_rn(sl, up);
                    }
                } else {   // TE_HEAD: word scores, and the running first maximum per column
                    unsigned long long key = 0ull;
                    if (live && cc < a.ncol) {
                        float *lg = a.cols_d[cc].logits;
                        if (lg) lg[grow] = v;
                        key = amax_key(v, grow);
                    }
#pragma unroll
                    for (int o = 16; o; o >>= 1) {
                        const unsigned long long u2 = __shfl_xor_sync(0xffffffffu, key, o);
                        key = u2 > key ? u2 : key;
                    }
                    if (lane == 0 && cc < a.ncol && key) atomicMax(&best[cc], key);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TC_WARP_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS) : "memory");
    }
    if (a.epi == TE_HEAD) {   // the step ends here: pick, position, counters (one CTA, the last to finish)
        if (tid < a.ncol && best[tid] && abort_flag == 0) atomicMax(&a.cols_d[tid].s->amax, best[tid]);
        __threadfence();
        __syncthreads();
        if (tid == 0) last_cta = atomicAdd(a.done, 1u) == gridDim.x - 1;
        __syncthreads();
        if (last_cta && tid < a.ncol) {
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
    }
}
#endif

}  // namespace imi

// k_tc_table: one 4-bit table times many inputs (16..256 columns) on the 5th-generation tensor cores: the batched
// read of imi_q8b + imi_q4_group_batch (imi/core/tables.cpp:405-477), used where a step reads a table for dozens of
// conversations or prefill positions at once.
//
// The exact numbers allow tensor cores because imi's per-block integer dots are exact: for a 32-value block j the dot
// sum_i code_ri * x_ci of 4-bit codes (0..15) and 8-bit input codes (-127..127) is an integer below 2^16 in
// magnitude, which an fp16 x fp16 -> fp32 tensor-core product computes exactly (every product and every partial sum is
// an integer that fp32 holds exactly). imi scales each block's dot before it accumulates, so the MMA must not sum over
// blocks: every block gets its own TMEM columns (D_j[row][col] = dot of block j), and the epilogue runs imi's two
// float chains per (row, column) in block order (group_avx2<false>, tables.cpp:127-143):
//     acc = fma(dot_j, d_rj * dx_cj, acc),  cor = fma(d_rj, s_cj, cor),  out = acc - 8 cor (one rounding).
//
// Work unit: a tile of 128 rows x a group of G columns (G = 16, 32 or 64). K is read in stages of 128 values (4
// blocks). Warp roles (one CTA per SM, persistent over units):
//   warp 0      producer: per stage one barrier for four copies into a ring slot: TMA of the tile's 4-bit codes
//               (128 rows x 80 bytes, 64 used: a padded shared-memory row stride keeps the unpack's reads free of
//               bank conflicts) and fp16 scales, bulk copies of the columns' fp16 codes (already in the MMA's K-major
//               layout, read by the MMA where they land) and of their scales and sums; it waits only for the slot, so
//               weight bytes stream several stages ahead of the math;
//   warp 1      TMEM owner (512 columns) and MMA issuer: per block two tcgen05.mma kind::f16 (K = 16 each) into the
//               block's own TMEM columns; the 4 blocks of a stage fill one TMEM stage slot, committed to its barrier
//               once (a commit-to-wait hand-off costs about 0.3 us, so it is made per stage, not per block);
//   warps 2-5   unpack: 4-bit codes -> fp16 in the MMA's canonical K-major layout (8-row x 16-byte core matrices),
//               the rows' block scales and the columns' scales and sums handed to the epilogue;
//   warps 6..   epilogue, 4 per 16 columns: per TMEM slot a tcgen05.ld of the block's dots (warp w reads lanes
//               32 (w % 4) ..), the two fma chains for 16 columns per thread (packed f32x2 operations, each lane rounded
//               as imi's scalar chain), the result stored at the end of the unit.
// Every wait on an mbarrier is bounded (about one second); a wait that gives up sets the error flag, the CTA stops
// issuing work, waits (bounded) for its copies and MMAs in flight, frees its TMEM and returns.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace imi {

constexpr int TC_M = 128;              // rows per tile (the MMA's M; TMEM lanes)
constexpr int TC_KS = 128;             // values per K stage
constexpr int TC_BPS = TC_KS / 32;     // blocks per stage
constexpr int TC_RAW_W = 80;           // bytes per row of a raw code stage in shared memory (64 used)
constexpr int TC_NR = 4, TC_NA = 2, TC_NE = 4;   // rings: copied stages, unpacked weight stages, epilogue stages
constexpr int TC_WARP_PROD = 0, TC_WARP_MMA = 1, TC_WARP_UNP = 2, TC_WARP_EPI = 6;
constexpr int TC_CH = 16;   // columns per epilogue thread
// epilogue warps: 4 per 16 columns (one per TMEM lane quarter), so each thread runs 16 columns' chains
__host__ __device__ constexpr int tc_epi_warps(int G) { return 4 * (G / TC_CH); }
__host__ __device__ constexpr int tc_threads(int G) { return 32 * (TC_WARP_EPI + tc_epi_warps(G)); }
constexpr int TC_TMEM_COLS = 512;

// output stage: TE_STORE out[c][row]; TE_SILU rows (2i, 2i+1) are (gate_i, up_i) of an interleaved gate/up table:
// out[c][i] = silu(gate) * up (seoul.cpp:384-391); TE_HEAD word scores into each column's logits (when it has them)
// and imi's greedy pick (first maximum, lowest id on ties), ending the step as the small-batch word-table read does
enum TcEpi : int { TE_STORE = 0, TE_SILU = 1, TE_HEAD = 2 };

struct TcArgs {
    CUtensorMap tm_codes;     // the table's rows as bytes [rows][row_bytes], box {TC_RAW_W, 128}
    CUtensorMap tm_scales;    // the same rows, box {16, 128} (8 fp16 scales of two stages)
    int rows, cols, row_bytes;
    int ncol, G, groups;      // columns, columns per group, groups (units = tiles * groups)
    const uint8_t *xh;        // the columns' 8-bit codes as fp16, [group][cols / 8][G][8]
    const float *xds;         // per group and block: G scales then G scale * code sums, [group][cols / 32][2][G]
    float *out;               // out[c * out_stride + row]
    int out_stride;
    int epi;
    const Col *cols_d;        // TE_HEAD: the columns (logits, conversation records)
    unsigned *done;           // TE_HEAD: CTAs finished (the last one picks and resets it)
    int *err;
    unsigned long long *trace;   // optional (diagnostics): CTA 0's timeline, [7][64] ns (see k_tc_table)
};
constexpr int TC_TRACE = 64;

struct TcPlan {
    int raw, a, epi, bar, tptr, total;
    int raw_bytes, raw_stride, b_off, x_off, a_bytes, b_bytes, xds_bytes, epi_bytes, nslot;   // nslot: TMEM stage slots
};
// a copied stage: [codes 128 x TC_RAW_W | scales 128 x 16 | columns' fp16 codes | columns' scales and sums]
__host__ __device__ inline TcPlan tc_plan(int G) {
    TcPlan p;
    p.b_bytes = (TC_KS / 8) * G * 16;                     // fp16 codes of G columns
    p.xds_bytes = TC_BPS * 2 * G * 4;
    p.b_off = TC_M * TC_RAW_W + TC_M * 16;
    p.x_off = p.b_off + p.b_bytes;
    p.raw_bytes = p.x_off + p.xds_bytes;
    p.raw_stride = align_up(p.raw_bytes, 128);
    p.a_bytes = (TC_KS / 8) * TC_M * 16;                  // fp16 codes of 128 rows, 16 chunks of 8 values
    p.epi_bytes = align_up(p.xds_bytes + TC_M * 8, 128);  // the columns' scales and sums + the rows' 4 block scales
    p.nslot = TC_TMEM_COLS / (G * TC_BPS);               // TMEM stage slots: a stage's 4 blocks, G columns each
    int o = 0;
    p.raw = o;  o += TC_NR * p.raw_stride;
    p.a = o;    o += TC_NA * p.a_bytes;
    p.epi = o;  o += TC_NE * p.epi_bytes;
    p.bar = o;  o += 8 * (2 * TC_NR + 2 * TC_NA + 2 * TC_NE + 2 * 32 + 1);
    p.tptr = o; o += 16;
    p.total = align_up(o, 128) + 128;                     // + slack to align the base to 128 bytes
    return p;
}

#if defined(__CUDACC__) && defined(IMI_KERNELS)   // device code: compiled in kernels.cu only
// ---- tcgen05 / TMA wrappers ----
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b))
                 : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16 (fp16 inputs, fp32 accumulate)
__device__ __forceinline__ void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, int acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// shared-memory matrix descriptor, K-major, no swizzle: 8-row x 16-byte core matrices, lbo between the two 16-byte K
// chunks of an MMA, sbo between 8-row groups (tcgen05 descriptor: start >> 4, lbo >> 4 at bit 16, sbo >> 4 at bit 32,
// version 1 at bit 46, layout 0 = no swizzle at bits 61-63)
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFF) | ((uint64_t) ((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}
// instruction descriptor: D f32 (bit 4), A and B f16 (format 0), both K-major, N >> 3 at bit 17, M >> 4 at bit 24
__host__ __device__ constexpr uint32_t tc_idesc_f16(int n, int m) {
    return (1u << 4) | ((uint32_t) (n >> 3) << 17) | ((uint32_t) (m >> 4) << 24);
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

// 8 values (the low or the high nibbles of the 8 code bytes w0, w1) as fp16: every nibble spread into a 16-bit lane
// under the byte 0x64, i.e. 0x6400 | v = 1024 + v in fp16, then minus 1024 (exact)
__device__ __forceinline__ uint32_t h2sub1024(uint32_t m) {
    const __half2 r = __hsub2(*reinterpret_cast<const __half2 *>(&m), __half2(__ushort_as_half(0x6400), __ushort_as_half(0x6400)));
    return *reinterpret_cast<const uint32_t *>(&r);
}
__device__ __forceinline__ uint4 nib8(uint32_t w0, uint32_t w1, int hi) {
    const uint32_t n0 = (hi ? w0 >> 4 : w0) & 0x0F0F0F0Fu, n1 = (hi ? w1 >> 4 : w1) & 0x0F0F0F0Fu;
    return make_uint4(h2sub1024(__byte_perm(n0, 0x64646464u, 0x7170)), h2sub1024(__byte_perm(n0, 0x64646464u, 0x7372)),
                      h2sub1024(__byte_perm(n1, 0x64646464u, 0x7170)), h2sub1024(__byte_perm(n1, 0x64646464u, 0x7372)));
}

template <int G>
__global__ void __launch_bounds__(tc_threads(G), 1) k_tc_table(const __grid_constant__ TcArgs a) {
    extern __shared__ __align__(128) uint8_t smt[];
    constexpr int CH = TC_CH, NEW = tc_epi_warps(G);
    const TcPlan P = tc_plan(G);
    uint8_t *sm = smt + ((128 - (smem_u32(smt) & 127)) & 127);
    uint64_t *bars = (uint64_t *) (sm + P.bar);
    // raw_full: the four copies of a stage landed (1 arrival + bytes); raw_empty: unpacked (4 warps) and read by the
    // MMAs (1 commit); a_full / e_full: the 4 unpack warps; a_empty, tm_full, fin: tcgen05.commit; e_empty, tm_empty:
    // the epilogue warps
    uint64_t *raw_full = bars, *raw_empty = raw_full + TC_NR, *a_full = raw_empty + TC_NR, *a_empty = a_full + TC_NA,
             *e_full = a_empty + TC_NA, *e_empty = e_full + TC_NE, *tm_full = e_empty + TC_NE, *tm_empty = tm_full + 32,
             *fin = tm_empty + 32;
    uint32_t *tptr = (uint32_t *) (sm + P.tptr);
    __shared__ int abort_flag, last_cta;
    __shared__ unsigned long long best[256];   // TE_HEAD: this CTA's best key per column
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (a.epi == TE_HEAD)
        for (int k = tid; k < 256; k += blockDim.x) best[k] = 0ull;
    const int K = a.cols, nst = K / TC_KS, tiles = (a.rows + TC_M - 1) / TC_M, units = tiles * a.groups;
    const int nslot = P.nslot;

    if (tid == 0) {
        for (int i = 0; i < TC_NR; i++) { mbar_init(&raw_full[i], 1); mbar_init(&raw_empty[i], 5); }
        for (int i = 0; i < TC_NA; i++) { mbar_init(&a_full[i], 4); mbar_init(&a_empty[i], 1); }
        for (int i = 0; i < TC_NE; i++) { mbar_init(&e_full[i], 4); mbar_init(&e_empty[i], NEW); }
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
    pdl_wait();

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
    auto raw_at = [&](int r) { return sm + P.raw + r * P.raw_stride; };

    if (warp == TC_WARP_PROD) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int i = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                const int tile = u / a.groups, g = u - tile * a.groups;
                const uint8_t *xh = a.xh + (size_t) g * (K / 8) * G * 16;
                const float *xds = a.xds + (size_t) g * (K / 32) * 2 * G;
                for (int s = 0; s < nst; s++, i++) {
                    const int r = i % TC_NR;
                    if (!(ok = wait(&raw_empty[r], ((i / TC_NR) & 1) ^ 1))) break;
                    uint8_t *raw = raw_at(r);
                    mbar_expect_tx(&raw_full[r], (uint32_t) P.raw_bytes);
                    tma_load_2d(raw, &a.tm_codes, s * (TC_KS / 2), tile * TC_M, &raw_full[r]);
                    tma_load_2d(raw + TC_M * TC_RAW_W, &a.tm_scales, K / 2 + 16 * (s / 2), tile * TC_M, &raw_full[r]);
                    bulk_g2s(raw + P.b_off, xh + (size_t) s * (TC_KS / 8) * G * 16, (uint32_t) P.b_bytes, &raw_full[r]);
                    bulk_g2s(raw + P.x_off, xds + (size_t) s * TC_BPS * 2 * G, (uint32_t) P.xds_bytes, &raw_full[r]);
                    if (a.trace && blockIdx.x == 0 && i < TC_TRACE) a.trace[0 * TC_TRACE + i] = global_ns();
                }
            }
            if (!ok)   // the copies in flight land before the CTA exits (bounded waits on the last stages issued)
                for (int k = i > TC_NR ? i - TC_NR : 0; k < i; k++) mbar_wait(&raw_full[k % TC_NR], (k / TC_NR) & 1);
        }
    } else if (warp == TC_WARP_MMA) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = tc_idesc_f16(G, TC_M);
            int i = 0, b = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                for (int s = 0; s < nst && ok; s++, i++) {
                    const int r = i % TC_NR, o = i % TC_NA;
                    if (!(ok = wait(&a_full[o], (i / TC_NA) & 1) && wait(&raw_full[r], (i / TC_NR) & 1))) break;
                    tc_fence_after();
                    const uint32_t abase = smem_u32(sm + P.a + o * P.a_bytes), bbase = smem_u32(raw_at(r) + P.b_off);
                    const int slot = i % nslot;
                    if (!(ok = wait(&tm_empty[slot], ((i / nslot) & 1) ^ 1))) break;
                    tc_fence_after();
                    for (int jj = 0; jj < TC_BPS; jj++, b++) {
#pragma unroll
                        for (int h = 0; h < 2; h++) {   // K = 16 per MMA: chunks 4jj + 2h, 4jj + 2h + 1
                            const int q = 4 * jj + 2 * h;
                            tc_mma_f16(tmem + (slot * TC_BPS + jj) * G, tc_desc(abase + q * TC_M * 16, TC_M * 16, 128),
                                       tc_desc(bbase + q * G * 16, G * 16, 128), idesc, h);
                        }
                        if (a.trace && blockIdx.x == 0 && b < TC_TRACE) a.trace[3 * TC_TRACE + b] = global_ns();
                    }
                    tc_commit(&tm_full[slot]);
                    tc_commit(&a_empty[o]);
                    tc_commit(&raw_empty[r]);
                }
            }
            if (!ok) {   // the MMAs issued complete before TMEM is freed
                tc_commit(fin);
                mbar_wait(fin, 0);
            }
        }
    } else if (warp < TC_WARP_EPI) {
        // ---------------- unpack: 4-bit codes -> fp16, canonical K-major layout ----------------
        const int row = tid - TC_WARP_UNP * 32;   // 0..127: this thread's row of the tile
        int i = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
            for (int s = 0; s < nst; s++, i++) {
                const int r = i % TC_NR, o = i % TC_NA, e = i % TC_NE;
                if (!(ok = wait(&raw_full[r], (i / TC_NR) & 1) && wait(&a_empty[o], ((i / TC_NA) & 1) ^ 1) &&
                           wait(&e_empty[e], ((i / TC_NE) & 1) ^ 1)))
                    break;
                if (a.trace && blockIdx.x == 0 && row == 0 && i < TC_TRACE) a.trace[1 * TC_TRACE + i] = global_ns();
                const uint8_t *raw = raw_at(r);
                uint8_t *A = sm + P.a + o * P.a_bytes, *ep = sm + P.epi + e * P.epi_bytes;
#pragma unroll
                for (int p = 0; p < TC_BPS; p++) {   // block p of the stage: 16 code bytes -> 4 chunks of 8 fp16
                    const uint4 c = *(const uint4 *) (raw + row * TC_RAW_W + 16 * p);
                    *(uint4 *) (A + ((4 * p + 0) * TC_M + row) * 16) = nib8(c.x, c.y, 0);   // values 0..7
                    *(uint4 *) (A + ((4 * p + 1) * TC_M + row) * 16) = nib8(c.z, c.w, 0);   // 8..15
                    *(uint4 *) (A + ((4 * p + 2) * TC_M + row) * 16) = nib8(c.x, c.y, 1);   // 16..23
                    *(uint4 *) (A + ((4 * p + 3) * TC_M + row) * 16) = nib8(c.z, c.w, 1);   // 24..31
                }
                // the row's 4 block scales of this stage (8 bytes of the 16-byte scale box), the columns' scales/sums
                *(uint2 *) (ep + P.xds_bytes + row * 8) = *(const uint2 *) (raw + TC_M * TC_RAW_W + row * 16 + 8 * (s & 1));
                if (row < P.xds_bytes / 16) *(uint4 *) (ep + 16 * row) = *(const uint4 *) (raw + P.x_off + 16 * row);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&a_full[o]);
                    mbar_arrive(&raw_empty[r]);
                    mbar_arrive(&e_full[e]);
                }
                if (a.trace && blockIdx.x == 0 && row == 0 && i < TC_TRACE) a.trace[2 * TC_TRACE + i] = global_ns();
            }
        }
    } else {
        // ---------------- epilogue: imi's float chains per (row, column) ----------------
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
                const int e = i % TC_NE, slot = i % nslot;
                if (!(ok = wait(&e_full[e], (i / TC_NE) & 1) && wait(&tm_full[slot], (i / nslot) & 1))) break;
                tc_fence_after();
                const uint8_t *ep = sm + P.epi + e * P.epi_bytes;
                const uint16_t *dsc = (const uint16_t *) (ep + P.xds_bytes + row * 8);
                for (int jj = 0; jj < TC_BPS; jj++, b++) {
                    const bool tr = a.trace && blockIdx.x == 0 && warp == TC_WARP_EPI && lane == 0 && b < TC_TRACE;
                    if (tr) a.trace[4 * TC_TRACE + b] = global_ns();
                    uint32_t f[CH];
                    tmem_ld<CH>(tl + (slot * TC_BPS + jj) * G, f);
                    tmem_ld_wait();
                    if (tr) a.trace[6 * TC_TRACE + b] = global_ns() + (unsigned long long) (f[0] & 0);
                    const float d = h2f(dsc[jj]);
                    const float2 dd = make_float2(d, d);
                    const float4 *xd = (const float4 *) ((const float *) ep + jj * 2 * G + h * CH),
                                 *xs = (const float4 *) ((const float *) ep + jj * 2 * G + G + h * CH);
#pragma unroll
                    for (int k = 0; k < CH / 4; k++) {   // 4 columns per pair of 16-byte loads
                        const float4 dx = xd[k], sx = xs[k];
                        const float2 f0 = make_float2(__uint_as_float(f[4 * k]), __uint_as_float(f[4 * k + 1])),
                                     f1 = make_float2(__uint_as_float(f[4 * k + 2]), __uint_as_float(f[4 * k + 3]));
                        acc[2 * k] = __ffma2_rn(f0, __fmul2_rn(dd, make_float2(dx.x, dx.y)), acc[2 * k]);
                        acc[2 * k + 1] = __ffma2_rn(f1, __fmul2_rn(dd, make_float2(dx.z, dx.w)), acc[2 * k + 1]);
                        cor[2 * k] = __ffma2_rn(dd, make_float2(sx.x, sx.y), cor[2 * k]);
                        cor[2 * k + 1] = __ffma2_rn(dd, make_float2(sx.z, sx.w), cor[2 * k + 1]);
                    }
                    if (tr) a.trace[5 * TC_TRACE + b] = global_ns() + (unsigned long long) (__float_as_uint(acc[0].x) & 0);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tm_empty[slot]);
                    mbar_arrive(&e_empty[e]);
                }
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

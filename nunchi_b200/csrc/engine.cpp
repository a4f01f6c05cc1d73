// The decode engine's host side: GGUF load and repack, device residency, conversation states, the per-step kernel
// schedule (captured once per shape into a CUDA graph and replayed), and the C-ABI of imi_cuda.h.
//
// Step schedule (one launch per stop of imi's step, seoul.cpp:402-488; every launch is a programmatic dependent of the
// previous one):
//   layer l, conv:      [in_proj: residual + attn_norm + cut] [out_proj: conv + cut] [gate_up: residual + ffn_norm
//                       + cut, SiLU(gate)*up, conv memory write] [down: cut]
//   layer l, attention: [qkvg: residual + attn_norm + cut] [attention] [o: cut] [gate_up] [down]
//   end:                [word table: residual + out_norm -> hidden, cut, scores, first-max pick, position++]
//                       or, without scores, [final norm, position++]
#include "../../include/imi_cuda.h"
#include "gguf_file.h"
#include "launch.h"

#include <cudaTypedefs.h>


#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

namespace imi {
void rope_table(int n_ctx, int n, float base, const float *ff, float *cs, float *sn);
}
using namespace imi;

static thread_local std::string g_err;
static imi_cuda_status fail(imi_cuda_status st, const std::string &msg) {
    g_err = msg;
    return st;
}
#define CK(x)                                                                                                 \
    do {                                                                                                      \
        cudaError_t e_ = (x);                                                                                 \
        if (e_ != cudaSuccess) return fail(e_ == cudaErrorMemoryAllocation ? IMI_E_NOMEM : IMI_E_CUDA,        \
                                           std::string(#x) + ": " + cudaGetErrorString(e_));                  \
    } while (0)

// a device allocation counted against the engine's budget (IMI_CUDA_MAX_DEVICE_BYTES)
#define DALLOC(e, ptr, n)                                                                                     \
    do {                                                                                                      \
        const size_t n_ = (n);                                                                                \
        if ((e)->dev_used + n_ > (e)->dev_budget)                                                             \
            return fail(IMI_E_NOMEM, "device memory budget (IMI_CUDA_MAX_DEVICE_BYTES = " +                  \
                                         std::to_string((e)->dev_budget) + ") exceeded: " +                   \
                                         std::to_string((e)->dev_used) + " bytes held, " + std::to_string(n_) + \
                                         " more asked");                                                      \
        CK(cudaMalloc((void **) &(ptr), n_));                                                                 \
        (e)->dev_used += n_;                                                                                  \
    } while (0)

namespace {

constexpr int STEP_COLS = 8;      // columns per launch of the small-batch table kernel
constexpr int TC_CHUNK = 128;     // prefill positions per batched read (tensor-core path)
constexpr int BATCH_GROUP = 64;   // step_batch checks the context per 64 positions, as seoul.cpp:496-498

struct TableRef {
    size_t off = 0;
    int rows = 0, cols = 0, row_bytes = 0;
    bool has_m = false;   // Q4_1 rows: a minimum per block after the scales
    TcArgs tc = {};       // the tensor-core batched read of this table: its TMA views (Q4_0 tables)
};
struct LayerRef {
    bool conv = false, swa = false;
    int ai = -1, ci = -1;
    TableRef in_proj, out_proj, qkvg, o, gate_up, down;
    size_t attn_norm = 0, post_attn_norm = 0, ffn_norm = 0, post_ffn_norm = 0, conv_w = 0, q_norm = 0, k_norm = 0;
};

}  // namespace

struct imi_cuda_engine {
    int device = 0, sm_count = 0;
    cudaStream_t stream = nullptr;
    int n_embd = 0, n_vocab = 0, n_ctx = 0, n_layer = 0, n_attn = 0, n_conv = 0, n_head = 0, n_head_kv = 0,
        head_dim = 0, n_ff = 0, d_conv = 0, n_swa = 0, max_batch = 0;
    float eps = 1e-5f, rope_base = 1e6f, rope_base_swa = 1e4f;
    uint8_t *w = nullptr;
    size_t w_bytes = 0;
    std::vector<LayerRef> layers;
    TableRef tok;
    bool tok_q6k = false;   // the word table is Q6_K (kept as in the file) rather than Q4_0
    int8_t *q8k_q = nullptr;   // Q6_K word table: the hidden state cut per 256 values [col][n_embd], scales, sums
    float *q8k_d = nullptr;
    int16_t *q8k_b = nullptr;
    size_t out_norm = 0;
    float *rope_cs = nullptr, *rope_sn = nullptr;   // [2][n_ctx][head_dim/2]: full layers, window layers
    int big_n = 0;
    float *X = nullptr, *big = nullptr, *y = nullptr, *att = nullptr, *act = nullptr, *fo = nullptr, *embd = nullptr,
          *hid = nullptr;
    int8_t *qa_q = nullptr, *qt_q = nullptr;   // 8-bit cuts of act [col][n_ff] and att [col][n_head*head_dim]
    float *qa_d = nullptr, *qa_s = nullptr, *qt_d = nullptr, *qt_s = nullptr;
    Col *cols_d = nullptr, *cols_h = nullptr;
    std::vector<int> cols_pos;   // each column's session position as the host knows it (decode_col)
    float *embd_h = nullptr;
    // columns one launch takes at most: 8 in the small-batch table kernel; up to ncmax (the larger of max_batch and
    // a prefill chunk) in the tensor-core batched read, when every table is Q4_0 (tc_batch)
    int ncmax = STEP_COLS;
    bool tc_batch = false;
    uint8_t *tc_w = nullptr;    // every table's tiled copy for the batched read (k_tc_tile)
    uint8_t *tc_xb = nullptr;   // the batched read's column operand (codes, block scales and sums)
    SessDev *reply_d = nullptr;   // the last step's conversation records gathered for one read-back
    // pinned: what the host reads back after a step (session records at 32-byte slots from 0, the error word after
    // them), so the read is one small DMA into page-locked memory instead of staged copies into pageable memory. One
    // read brings every conversation of the last step; it stays valid until anything changes a session (gen moves on).
    uint8_t *reply_h = nullptr;
    uint64_t gen = 1, reply_gen = 0;
    int last_n = 0, reply_n = 0;
    std::vector<const SessDev *> last_s, reply_src;
    unsigned *done = nullptr;
    int *err = nullptr;
    cudaEvent_t staged = nullptr;   // the last host->device copy of the staging buffers has run
    cudaEvent_t t0 = nullptr, t1 = nullptr;   // around the last step's graph (imi_cuda_last_step_ms)
    bool timed = false;
    std::map<int, cudaGraphExec_t> graphs;
    size_t state_bytes = 0;
    size_t dev_budget = SIZE_MAX, dev_used = 0;   // IMI_CUDA_MAX_DEVICE_BYTES and what the engine + states hold
    uint8_t *qbuf = nullptr;
    // diagnostics: when trace_buf is set, every launch enqueued gets its own [grid][MV_TRACE] slice
    unsigned long long *trace_buf = nullptr;
    int trace_n = 0, trace_max = 0;
    std::vector<int> trace_kind, trace_grid;
    unsigned long long *trace_slot(int kind, int grid) {
        if (!trace_buf || trace_n >= trace_max || grid > sm_count) return nullptr;   // a slot holds sm_count CTAs
        trace_kind.push_back(kind);
        trace_grid.push_back(grid);
        return trace_buf + (size_t) (trace_n++) * sm_count * MV_TRACE;
    }
    const float *f32(size_t off) const { return (const float *) (w + off); }
    ~imi_cuda_engine();
};

struct imi_cuda_state {
    imi_cuda_engine *e = nullptr;
    void *mem = nullptr;
    size_t mem_bytes = 0;
    SessDev *s = nullptr;
    __half *kc = nullptr, *vc = nullptr;
    float *ring = nullptr, *hidden = nullptr, *logits = nullptr;
    int *picks = nullptr;
    int pos = 0;
};

imi_cuda_engine::~imi_cuda_engine() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (auto &g : graphs) cudaGraphExecDestroy(g.second);
    cudaFree(w);
    cudaFree(rope_cs);
    cudaFree(X);
    cudaFree(qbuf);
    cudaFree(q8k_q);
    cudaFree(cols_d);
    cudaFree(tc_w);
    cudaFree(tc_xb);
    cudaFreeHost(cols_h);
    cudaFreeHost(embd_h);
    cudaFreeHost(reply_h);
    if (staged) cudaEventDestroy(staged);
    if (t0) cudaEventDestroy(t0);
    if (t1) cudaEventDestroy(t1);
    if (stream) cudaStreamDestroy(stream);
}

// ---------------------------------------------------------------------------------------------------------------
// load
// ---------------------------------------------------------------------------------------------------------------
namespace {

// bytes of one table row in the engine's layout: Q4_0 [cols/2 code bytes | cols/32 fp16 scales], Q4_1 the same
// followed by [cols/32 fp16 minimums]
size_t engine_row_bytes(const gguf_tensor *t) { return (size_t) (t->ne[0] / 32) * (t->type == T_Q4_1 ? 20 : 18); }

// rows of Q4_0 / Q4_1 tables, in order, into the engine's row layout. The code bytes of block j keep the file's order
// (byte i: column i in the low nibble, column 16+i in the high one). File blocks: Q4_0 [d | 16 code bytes], Q4_1
// [d | m | 16 code bytes] (ggml's block_q4_0 / block_q4_1).
void repack_rows(uint8_t *dst, const std::vector<std::pair<const gguf_tensor *, int>> &rows) {
    for (size_t r = 0; r < rows.size(); r++) {
        const gguf_tensor *t = rows[r].first;
        const int nb = (int) (t->ne[0] / 32), hm = t->type == T_Q4_1, fb = hm ? 20 : 18;
        const uint8_t *src = t->data + (size_t) rows[r].second * t->row_bytes;
        uint8_t *codes = dst + r * (size_t) nb * fb, *scales = codes + (size_t) nb * 16, *mins = scales + (size_t) nb * 2;
        for (int j = 0; j < nb; j++) {
            memcpy(scales + 2 * j, src + fb * j, 2);
            if (hm) memcpy(mins + 2 * j, src + fb * j + 2, 2);
            memcpy(codes + 16 * j, src + fb * j + 2 + 2 * hm, 16);
        }
    }
}

constexpr int T_Q4_ANY = -1;   // Loader::need: a layer table, Q4_0 or Q4_1

struct Loader {
    const gguf_file &f;
    std::string err;
    size_t off = 0;
    std::vector<std::pair<size_t, const gguf_tensor *>> f32s;                                  // (offset, tensor)
    std::vector<std::pair<size_t, std::vector<std::pair<const gguf_tensor *, int>>>> tables;   // (offset, rows)
    std::vector<std::pair<size_t, const gguf_tensor *>> convs;                                 // transposed taps
    explicit Loader(const gguf_file &ff) : f(ff) {}
    size_t take(size_t n) {
        const size_t o = off;
        off = (off + n + 255) / 256 * 256;
        return o;
    }
    const gguf_tensor *need(const std::string &name, int type) {
        const gguf_tensor *t = f.tensor(name);
        if (!t) { if (err.empty()) err = "missing tensor " + name; return nullptr; }
        const bool ok = type == T_Q4_ANY ? (t->type == T_Q4_0 || t->type == T_Q4_1) : t->type == type;
        if (!ok || !t->data) {
            if (err.empty()) err = name + ": type " + std::to_string(t->type) + " is not read by this engine";
            return nullptr;
        }
        return t;
    }
    bool vec(const std::string &name, int64_t n, size_t &at) {
        const gguf_tensor *t = need(name, T_F32);
        if (!t) return false;
        if (t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3] != n) { err = name + ": unexpected size"; return false; }
        at = take((size_t) n * 4);
        f32s.push_back({ at, t });
        return true;
    }
    bool table(TableRef &tr, const std::vector<std::pair<const gguf_tensor *, int>> &rows) {
        if (rows.empty()) { err = "empty table"; return false; }
        const int cols = (int) rows[0].first->ne[0];
        for (auto &r : rows)
            if (r.first->ne[0] != cols) { err = r.first->name + ": widths of a stacked table differ"; return false; }
        for (auto &r : rows)   // one layout per table: stacked tables share the rows' format
            if (r.first->type != rows[0].first->type) { err = r.first->name + ": types of a stacked table differ"; return false; }
        if (cols % 256) { err = rows[0].first->name + ": width must be a multiple of 256"; return false; }
        tr.rows = (int) rows.size();
        tr.cols = cols;
        tr.has_m = rows[0].first->type == T_Q4_1;
        tr.row_bytes = (int) engine_row_bytes(rows[0].first);
        if (2 * tr.row_bytes > MV_STAGE_BYTES) { err = rows[0].first->name + ": rows too wide"; return false; }
        tr.off = take((size_t) tr.rows * tr.row_bytes);
        tables.push_back({ tr.off, rows });
        return true;
    }
    static void all_rows(std::vector<std::pair<const gguf_tensor *, int>> &o, const gguf_tensor *t) {
        for (int r = 0; r < t->ne[1]; r++) o.push_back({ t, r });
    }
};

}  // namespace

// ---------------------------------------------------------------------------------------------------------------
// the tensor-core batched read: column group width, the columns' operands in the MMA's layout
// ---------------------------------------------------------------------------------------------------------------
namespace {

// column group width (16, 32 or 64) of one batched read of a `rows`-row table for ncol columns: the narrowest whose
// units (128-row tiles x column groups) still fit one wave of the SMs, so a short table spreads over more SMs (each
// CTA's epilogue, the part that bounds a unit, runs G columns); a tall table keeps 64 (one group of 64 columns)
int tc_group(int rows, int ncol, int sms) {
    const int tiles = (rows + TC_M - 1) / TC_M;
    for (int G = 16; G < 64; G *= 2)
        if (G >= ncol || tiles * ((ncol + G - 1) / G) <= sms) return G;
    return 64;
}

// the columns' 8-bit codes, scales and scale * code sums ([ncol][cols], [ncol][cols/32]) as the batched read's
// operand (tc_table.cuh: tc_xb_code, tc_xb_scale; zeros for the padding columns)
void tc_operands_host(const int8_t *xq, const float *xd, const float *xs, int ncol, int cols, int G,
                      std::vector<uint8_t> &xb) {
    const int groups = (ncol + G - 1) / G, nb = cols / 32;
    xb.assign((size_t) groups * (cols / TC_KS) * tc_xb_bytes(G), 0);
    for (int c = 0; c < ncol; c++) {
        const int g = c / G, cg = c - g * G;
        for (int k = 0; k < cols; k++) xb[tc_xb_code(G, cols, g, cg, k)] = (uint8_t) xq[(size_t) c * cols + k];
        for (int j = 0; j < nb; j++) {
            memcpy(&xb[tc_xb_scale(G, cols, g, cg, j, 0)], &xd[(size_t) c * nb + j], 4);
            memcpy(&xb[tc_xb_scale(G, cols, g, cg, j, 1)], &xs[(size_t) c * nb + j], 4);
        }
    }
}

}  // namespace

static imi_cuda_status load_impl(const char *path, int device, int n_ctx, int max_batch, imi_cuda_engine **out) {
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) return fail(IMI_E_NODEV, "no CUDA device");
    if (device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device " + std::to_string(device));
    if (!path || n_ctx <= 0 || max_batch <= 0) return fail(IMI_E_ARG, "bad load arguments");
    gguf_file f;
    if (!f.open(path)) return fail(IMI_E_FILE, f.error);
    std::unique_ptr<imi_cuda_engine> e(new imi_cuda_engine);
    e->device = device;
    e->n_ctx = n_ctx;
    e->max_batch = max_batch;
    CK(cudaSetDevice(device));
    CK(cudaDeviceGetAttribute(&e->sm_count, cudaDevAttrMultiProcessorCount, device));

    // hyperparameters: the keys and defaults of seoul.cpp:99-114
    e->eps = f.key_f("lfm3.attention.layer_norm_rms_epsilon", 1e-5f);
    e->rope_base = f.key_f("lfm3.rope.freq_base", 1e6f);
    e->rope_base_swa = f.key_f("lfm3.rope.freq_base_swa", 1e4f);
    e->n_swa = (int) f.key_i("lfm3.attention.sliding_window", 0);
    e->d_conv = (int) f.key_i("lfm3.shortconv.l_cache", 7) - 1;
    e->n_head = (int) f.key_i("lfm3.attention.head_count", 16);
    e->head_dim = (int) f.key_i("lfm3.attention.key_length", 128);
    e->n_layer = (int) f.key_i("lfm3.block_count", 0);
    const gguf_value *swa_pat = f.value("lfm3.attention.sliding_window_pattern");

    Loader L(f);
    const gguf_tensor *te = f.tensor("token_embd.weight");
    e->tok_q6k = te && te->type == T_Q6_K && te->data;   // the product's own word-table format (seoul.cpp:95-98)
    if (!e->tok_q6k) te = L.need("token_embd.weight", T_Q4_0);
    if (!te) return fail(IMI_E_FORMAT, L.err + " (the word table must be Q4_0 or Q6_K here)");
    e->n_embd = (int) te->ne[0];
    e->n_vocab = (int) te->ne[1];
    if (e->n_embd % 256) return fail(IMI_E_FORMAT, "n_embd must be a multiple of 256");
    if (e->n_layer <= 0 || e->d_conv < 1 || e->head_dim <= 0) return fail(IMI_E_FORMAT, "bad lfm3 hyperparameters");
    if (e->d_conv > 8 || e->n_embd > 6144)   // the input preparation keeps 8 taps and n_embd/4 float4 chunks in registers
        return fail(IMI_E_FORMAT, "conv width above 9 or n_embd above 6144 is not supported");
    const int E = e->n_embd;
    if (e->tok_q6k) {   // kept as in the file: rows of 210-byte blocks per 256 values, copied as they are
        e->tok.rows = e->n_vocab;
        e->tok.cols = E;
        e->tok.row_bytes = E / 256 * 210;
        e->tok.off = L.take(te->nbytes);
        L.f32s.push_back({ e->tok.off, te });
    } else {
        std::vector<std::pair<const gguf_tensor *, int>> rows;
        Loader::all_rows(rows, te);
        if (!L.table(e->tok, rows)) return fail(IMI_E_FORMAT, L.err);
    }
    if (!L.vec("output_norm.weight", E, e->out_norm)) return fail(IMI_E_FORMAT, L.err);
    const gguf_tensor *rf = f.tensor("rope_freqs.weight");
    if (rf && (rf->type != T_F32 || rf->ne[0] != e->head_dim / 2)) return fail(IMI_E_FORMAT, "rope_freqs.weight: bad shape");

    e->layers.resize(e->n_layer);
    for (int il = 0; il < e->n_layer; il++) {
        LayerRef &Lr = e->layers[il];
        const std::string p = "blk." + std::to_string(il) + ".";
        if (!L.vec(p + "attn_norm.weight", E, Lr.attn_norm) || !L.vec(p + "post_attention_norm.weight", E, Lr.post_attn_norm) ||
            !L.vec(p + "ffn_norm.weight", E, Lr.ffn_norm) || !L.vec(p + "post_ffw_norm.weight", E, Lr.post_ffn_norm))
            return fail(IMI_E_FORMAT, L.err);
        std::vector<std::pair<const gguf_tensor *, int>> rows;
        if (f.tensor(p + "shortconv.conv.weight")) {
            Lr.conv = true;
            Lr.ci = e->n_conv++;
            const gguf_tensor *cw = L.need(p + "shortconv.conv.weight", T_F32);
            if (!cw) return fail(IMI_E_FORMAT, L.err);
            if (cw->ne[0] != e->d_conv + 1 || cw->ne[1] != E) return fail(IMI_E_FORMAT, p + "shortconv.conv.weight: bad shape");
            Lr.conv_w = L.take((size_t) (e->d_conv + 1) * E * 4);
            L.convs.push_back({ Lr.conv_w, cw });
            const gguf_tensor *ip = L.need(p + "shortconv.in_proj.weight", T_Q4_ANY), *op = L.need(p + "shortconv.out_proj.weight", T_Q4_ANY);
            if (!ip || !op) return fail(IMI_E_FORMAT, L.err);
            if (ip->ne[0] != E || ip->ne[1] != 3 * E || op->ne[0] != E || op->ne[1] != E) return fail(IMI_E_FORMAT, p + "shortconv: bad shapes");
            Loader::all_rows(rows, ip);
            if (!L.table(Lr.in_proj, rows)) return fail(IMI_E_FORMAT, L.err);
            rows.clear();
            Loader::all_rows(rows, op);
            if (!L.table(Lr.out_proj, rows)) return fail(IMI_E_FORMAT, L.err);
        } else {
            const gguf_tensor *q = L.need(p + "attn_q.weight", T_Q4_ANY), *k = L.need(p + "attn_k.weight", T_Q4_ANY),
                              *v = L.need(p + "attn_v.weight", T_Q4_ANY), *g = L.need(p + "attn_gate.weight", T_Q4_ANY),
                              *o = L.need(p + "attn_output.weight", T_Q4_ANY);
            if (!q || !k || !v || !g || !o) return fail(IMI_E_FORMAT, L.err);
            const int D = e->head_dim;
            e->n_head_kv = (int) (k->ne[1] / D);   // seoul.cpp:153
            if (q->ne[1] != (int64_t) e->n_head * D || k->ne[1] != v->ne[1] || k->ne[1] % D || g->ne[1] != e->n_head ||
                o->ne[0] != (int64_t) e->n_head * D || o->ne[1] != E || q->ne[0] != E)
                return fail(IMI_E_FORMAT, p + "attention: bad shapes");
            if (e->n_head_kv <= 0 || e->n_head % e->n_head_kv) return fail(IMI_E_FORMAT, "heads do not group");
            for (auto *t : { q, k, v, g }) Loader::all_rows(rows, t);   // q|k|v|gate stacked, seoul.cpp:147
            if (!L.table(Lr.qkvg, rows)) return fail(IMI_E_FORMAT, L.err);
            rows.clear();
            Loader::all_rows(rows, o);
            if (!L.table(Lr.o, rows)) return fail(IMI_E_FORMAT, L.err);
            if (!L.vec(p + "attn_q_norm.weight", D, Lr.q_norm) || !L.vec(p + "attn_k_norm.weight", D, Lr.k_norm))
                return fail(IMI_E_FORMAT, L.err);
            Lr.swa = swa_pat && swa_pat->type == 9 && swa_pat->arr_type == 7 && (uint64_t) il < swa_pat->arr_n &&
                     swa_pat->arr[il] != 0;
            Lr.ai = e->n_attn++;
        }
        const gguf_tensor *fg = L.need(p + "ffn_gate.weight", T_Q4_ANY), *fu = L.need(p + "ffn_up.weight", T_Q4_ANY),
                          *fd = L.need(p + "ffn_down.weight", T_Q4_ANY);
        if (!fg || !fu || !fd) return fail(IMI_E_FORMAT, L.err);
        e->n_ff = (int) fg->ne[1];
        if (fu->ne[1] != e->n_ff || fg->ne[0] != E || fu->ne[0] != E || fd->ne[0] != e->n_ff || fd->ne[1] != E)
            return fail(IMI_E_FORMAT, p + "ffn: bad shapes");
        rows.clear();
        for (int t = 0; t < e->n_ff; t++) { rows.push_back({ fg, t }); rows.push_back({ fu, t }); }   // (gate_i, up_i)
        if (!L.table(Lr.gate_up, rows)) return fail(IMI_E_FORMAT, L.err);
        rows.clear();
        Loader::all_rows(rows, fd);
        if (!L.table(Lr.down, rows)) return fail(IMI_E_FORMAT, L.err);
    }
    if (e->n_attn && !attn_supported(e->head_dim, e->n_head / e->n_head_kv, e->n_ctx))
        return fail(IMI_E_FORMAT, "attention shape (head_dim " + std::to_string(e->head_dim) + ", group " +
                                      std::to_string(e->n_head / std::max(1, e->n_head_kv)) + ", n_ctx " +
                                      std::to_string(n_ctx) + ") not supported");
    if ((e->n_head * e->head_dim) % 256) return fail(IMI_E_FORMAT, "n_head * head_dim must be a multiple of 256");
    e->w_bytes = L.off;
    if (const char *cap = getenv("IMI_CUDA_MAX_DEVICE_BYTES")) e->dev_budget = (size_t) strtoull(cap, nullptr, 10);
    DALLOC(e, e->w, e->w_bytes);

    // upload: tables through a pinned staging buffer, small vectors directly
    size_t stage_max = 0;
    for (auto &t : L.tables) stage_max = std::max(stage_max, t.second.size() * engine_row_bytes(t.second[0].first));
    for (auto &c : L.convs) stage_max = std::max(stage_max, (size_t) (c.second->ne[0] * c.second->ne[1] * 4));
    uint8_t *stg = nullptr;
    CK(cudaMallocHost(&stg, stage_max));
    std::unique_ptr<uint8_t, decltype(&cudaFreeHost)> stg_guard(stg, cudaFreeHost);
    for (auto &t : L.tables) {
        repack_rows(stg, t.second);
        CK(cudaMemcpy(e->w + t.first, stg, t.second.size() * engine_row_bytes(t.second[0].first), cudaMemcpyHostToDevice));
    }
    for (auto &c : L.convs) {   // file [channel][tap] -> [tap][channel] (seoul.cpp:136-141)
        const int K = (int) c.second->ne[0], C = (int) c.second->ne[1];
        float *dst = (float *) stg;
        const float *src = (const float *) c.second->data;
        for (int ch = 0; ch < C; ch++)
            for (int k = 0; k < K; k++) dst[(size_t) k * C + ch] = src[(size_t) ch * K + k];
        CK(cudaMemcpy(e->w + c.first, stg, (size_t) K * C * 4, cudaMemcpyHostToDevice));
    }
    for (auto &v : L.f32s) CK(cudaMemcpy(e->w + v.first, v.second->data, v.second->nbytes, cudaMemcpyHostToDevice));

    // rotary tables: full layers use freq_base and rope_freqs, window layers freq_base_swa (seoul.cpp:428-429)
    if (e->n_attn) {
        const int D = e->head_dim;
        const size_t per = (size_t) n_ctx * (D / 2);
        std::vector<float> cs(2 * per), sn(2 * per);
        imi::rope_table(n_ctx, D, e->rope_base, rf ? (const float *) rf->data : nullptr, cs.data(), sn.data());
        imi::rope_table(n_ctx, D, e->rope_base_swa, nullptr, cs.data() + per, sn.data() + per);
        DALLOC(e, e->rope_cs, 4 * per * 4);
        e->rope_sn = e->rope_cs + 2 * per;
        CK(cudaMemcpy(e->rope_cs, cs.data(), 2 * per * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(e->rope_sn, sn.data(), 2 * per * 4, cudaMemcpyHostToDevice));
    }

    // the tensor-core batched read takes every Q4_0 layer table and a Q4_0 word table (a Q4_1 table or a Q6_K word
    // table keeps the small-batch kernel, 8 columns per read)
    const int HD = e->n_head * e->head_dim, kvd = e->n_head_kv * e->head_dim;
    e->tc_batch = !e->tok_q6k && !e->tok.has_m && e->n_embd % (TC_CP * TC_KS) == 0 &&
                  e->n_embd <= 4 * TP_PQ * TP_THREADS;   // k_tc_prep holds a thread's norm chunks in registers
    for (auto &Lr : e->layers)
        for (const TableRef *t : { &Lr.in_proj, &Lr.out_proj, &Lr.qkvg, &Lr.o, &Lr.gate_up, &Lr.down })
            if (t->rows && t->has_m) e->tc_batch = false;
    if ((HD % (TC_CP * TC_KS)) || (e->n_ff % (TC_CP * TC_KS))) e->tc_batch = false;
    e->ncmax = e->tc_batch ? std::max({ STEP_COLS, max_batch, TC_CHUNK }) : STEP_COLS;
    if (e->ncmax > 256) return fail(IMI_E_ARG, "max_batch above 256");
    const int NC = e->ncmax;
    // per-column scratch
    e->big_n = std::max(3 * E, HD + 2 * kvd + e->n_head);
    const size_t per_col = (size_t) 2 * E + e->big_n + E + HD + e->n_ff + E + E + E;
    DALLOC(e, e->X, per_col * NC * 4);
    e->big = e->X + (size_t) 2 * E * NC;
    e->y = e->big + (size_t) e->big_n * NC;
    e->att = e->y + (size_t) E * NC;
    e->act = e->att + (size_t) HD * NC;
    e->fo = e->act + (size_t) e->n_ff * NC;
    e->embd = e->fo + (size_t) E * NC;
    e->hid = e->embd + (size_t) E * NC;
    {
        const size_t na = (size_t) STEP_COLS * e->n_ff, nt = (size_t) NC * HD;
        uint8_t *q = nullptr;
        DALLOC(e, q, na + nt + 4 * 2 * (na / 32 + nt / 32) + 1024);
        e->qbuf = q;
        e->qa_q = (int8_t *) q;
        e->qt_q = (int8_t *) (q + na);
        e->qa_d = (float *) (q + (na + nt + 255) / 256 * 256);
        e->qa_s = e->qa_d + na / 32;
        e->qt_d = e->qa_s + na / 32;
        e->qt_s = e->qt_d + nt / 32;
        CK(cudaMemset(q, 0, na + nt + 4 * 2 * (na / 32 + nt / 32) + 1024));
    }
    if (e->tok_q6k) {
        if (q6k_head_ctas(e->n_vocab, E / 256, STEP_COLS) <= 0) return fail(IMI_E_FORMAT, "Q6_K word table too wide");
        uint8_t *q = nullptr;
        const size_t nq = (size_t) STEP_COLS * E, nd = (size_t) STEP_COLS * (E / 256), nbs = (size_t) STEP_COLS * (E / 16);
        DALLOC(e, q, nq + 4 * nd + 2 * nbs + 64);
        e->q8k_q = (int8_t *) q;
        e->q8k_d = (float *) (q + nq);
        e->q8k_b = (int16_t *) (q + nq + 4 * nd);
    }
    DALLOC(e, e->cols_d, sizeof(Col) * NC + 64 + 32 * NC);
    e->done = (unsigned *) (e->cols_d + NC);
    e->err = (int *) (e->done + 4);
    e->reply_d = (SessDev *) ((uint8_t *) e->cols_d + sizeof(Col) * NC + 64);
    CK(cudaMemset(e->cols_d, 0, sizeof(Col) * NC + 64 + 32 * NC));
    CK(cudaMallocHost(&e->cols_h, sizeof(Col) * NC));
    CK(cudaMallocHost(&e->embd_h, (size_t) E * 4 * NC));
    CK(cudaMallocHost(&e->reply_h, (size_t) 32 * NC + 64));
    memset(e->cols_h, 0, sizeof(Col) * NC);
    e->cols_pos.assign(NC, 0);
    e->last_s.assign(NC, nullptr);
    e->reply_src.assign(NC, nullptr);
    if (e->tc_batch) {   // the batched read's operand buffer and every table's tiled copy
        const int ncp = (NC + 63) / 64 * 64, kmax = std::max(std::max(E, HD), e->n_ff);
        DALLOC(e, e->tc_xb, (size_t) (ncp / 16) * (kmax / TC_KS) * tc_xb_bytes(16));   // the most for any group width
        // every table's tiled copy (the weights as the tensor-core read streams them), made here on the device
        std::vector<TableRef *> tcs;
        for (auto &Lr : e->layers)
            for (TableRef *t : { &Lr.in_proj, &Lr.out_proj, &Lr.qkvg, &Lr.o, &Lr.gate_up, &Lr.down })
                if (t->rows) tcs.push_back(t);
        tcs.push_back(&e->tok);
        size_t tb = 0;
        for (TableRef *t : tcs) tb += (tc_tiled_bytes(t->rows, t->cols) + 255) / 256 * 256;
        DALLOC(e, e->tc_w, tb);
        size_t o = 0;
        for (TableRef *t : tcs) {
            t->tc = {};
            t->tc.rows = t->rows; t->tc.cols = t->cols; t->tc.err = e->err; t->tc.wt = e->tc_w + o;
            CK(launch_tc_tile(e->w + t->off, t->rows, t->cols, t->row_bytes, e->tc_w + o, nullptr));
            o += (tc_tiled_bytes(t->rows, t->cols) + 255) / 256 * 256;
        }
    }
    CK(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
    CK(cudaEventCreateWithFlags(&e->staged, cudaEventDisableTiming));
    CK(cudaEventCreate(&e->t0));
    CK(cudaEventCreate(&e->t1));
    CK(prepare_kernels());
    e->state_bytes = ATK_TMAP_OFF + 2 * sizeof(CUtensorMap) + (size_t) 2 * e->n_attn * n_ctx * kvd * 2 +
                     (size_t) e->n_conv * (e->d_conv + 1) * E * 4 + (size_t) E * 4 + (size_t) e->n_vocab * 4 +
                     (size_t) n_ctx * 4 + 6 * 256;
    CK(cudaDeviceSynchronize());
    *out = e.release();
    return IMI_OK;
}

// ---------------------------------------------------------------------------------------------------------------
// the step schedule
// ---------------------------------------------------------------------------------------------------------------
namespace {

enum StepKind { K_DECODE = 0, K_PREFILL = 1, K_HEAD_ONLY = 2 };

void plan_stages(MvArgs &a, int pro, int gran, int grid) { mv_plan_stages(a, pro, gran, grid); }

// one table read: CTAs take whole `unit`s of rows (64 for the SiLU stage, which cuts whole 32-value blocks of its
// output; else 1), stages hold a multiple of `gran` rows (2 for the SiLU stage's (gate, up) pairs)
cudaError_t table_launch(imi_cuda_engine *e, const TableRef &t, int pro, int epi, MvArgs a) {
    a.W = e->w + t.off;
    a.rows = t.rows;
    a.cols = t.cols;
    a.row_bytes = t.row_bytes;
    a.has_m = t.has_m ? 1 : 0;
    const int gran = epi == E_SILU ? 2 : 1;
    a.unit = epi == E_SILU ? 64 : 1;
    const int units = t.rows / a.unit;
    const int grid = std::max(1, std::min(e->sm_count, units));
    a.ab_len = epi == E_SILU ? (units + grid - 1) / grid * a.unit / 2 : 0;
    plan_stages(a, pro, gran, grid);
    if (!a.trace) a.trace = e->trace_slot(10 * pro + epi, grid);
    return launch_table(pro, epi, a, grid, e->stream, true);
}

// the Q6_K word scores of the step's columns (cut beforehand into q8k_*), the pick and the end of the step
cudaError_t q6k_head_launch(imi_cuda_engine *e, int ncol) {
    Q6HeadArgs q = {};
    q.cols_d = e->cols_d;
    q.ncol = ncol;
    q.W = e->w + e->tok.off;
    q.rows = e->n_vocab;
    q.nb = e->n_embd / 256;
    q.xq = e->q8k_q;
    q.xd = e->q8k_d;
    q.xb = e->q8k_b;
    q.done = e->done;
    q.trace = e->trace_slot(102, q6k_head_ctas(e->n_vocab, q.nb, ncol));
    return launch_q6k_head(q, e->stream, true);
}

cudaError_t enqueue_step(imi_cuda_engine *e, int ncol, bool head, StepKind kind) {
    const int E = e->n_embd, HD = e->n_head * e->head_dim;
    MvArgs b = {};
    b.cols_d = e->cols_d;
    b.ncol = ncol;
    b.eps = e->eps;
    b.n_embd = E;
    b.d_conv = e->d_conv;
    b.ring_layer = -1;
    b.emb = e->w + e->tok.off;
    b.emb_row_bytes = e->tok.row_bytes;
    b.emb_q6k = e->tok_q6k ? 1 : 0;
    b.x_stride = 2 * E;
    b.err = e->err;
    b.done = e->done;
    float *X0 = e->X, *X1 = e->X + E;
    cudaError_t r;
    if (kind == K_HEAD_ONLY && e->tok_q6k) {   // the same with the Q6_K word table: the 256-value cut, then the head
        for (int c = 0; c < ncol; c++)
            if ((r = launch_q8k_cut(e->hid + (size_t) c * E, E, e->q8k_q + (size_t) c * E, e->q8k_d + (size_t) c * (E / 256),
                                    e->q8k_b + (size_t) c * (E / 16), e->stream)) != cudaSuccess)
                return r;
        return q6k_head_launch(e, ncol);
    }
    if (kind == K_HEAD_ONLY) {   // word scores of a hidden state already computed (seoul.cpp:507-516)
        MvArgs a = b;
        a.in = e->hid;
        a.in_stride = E;
        return table_launch(e, e->tok, P_CUT, E_HEAD, a);
    }
    for (int il = 0; il < e->n_layer; il++) {
        const LayerRef &L = e->layers[il];
        MvArgs a = b;
        a.wpre = e->f32(L.attn_norm);
        a.xout = X0;
        a.out = e->big;
        a.out_stride = e->big_n;
        int pro = P_EMBED_NORM;
        if (il > 0) {
            pro = P_RESID_NORM;
            a.in = e->fo;
            a.in_stride = E;
            a.xin = X1;
            a.wpost = e->f32(e->layers[il - 1].post_ffn_norm);
        }
        if ((r = table_launch(e, L.conv ? L.in_proj : L.qkvg, pro, E_STORE, a)) != cudaSuccess) return r;
        if (L.conv) {
            a = b;
            a.in = e->big;
            a.in_stride = e->big_n;
            a.conv_w = e->f32(L.conv_w);
            a.conv_layer = L.ci;
            a.out = e->y;
            a.out_stride = E;
            // a step of distinct conversations (one position each) writes the conv memory right here: no column of it
            // reads the slot it writes; a prefill chunk writes it one launch later (the gate_up read)
            if (kind == K_DECODE) a.ring_layer = L.ci;
            if ((r = table_launch(e, L.out_proj, P_CONV, E_STORE, a)) != cudaSuccess) return r;
        } else {
            AttnArgs t = {};
            t.cols_d = e->cols_d;
            t.ncol = ncol;
            t.qkv = e->big;
            t.qkv_stride = e->big_n;
            t.att = e->att;
            t.att_stride = HD;
            t.q_norm = e->f32(L.q_norm);
            t.k_norm = e->f32(L.k_norm);
            t.eps = e->eps;
            t.scale = 1.0f / sqrtf((float) e->head_dim);   // seoul.cpp:432
            const size_t per = (size_t) e->n_ctx * (e->head_dim / 2);
            t.rope_cs = e->rope_cs + (L.swa ? per : 0);
            t.rope_sn = e->rope_sn + (L.swa ? per : 0);
            t.ai = L.ai;
            t.n_head = e->n_head;
            t.n_head_kv = e->n_head_kv;
            t.head_dim = e->head_dim;
            t.n_ctx = e->n_ctx;
            t.window = (L.swa && e->n_swa > 0) ? e->n_swa : 0;   // seoul.cpp:431
            t.err = e->err;
            t.kv_fused = kind == K_DECODE;
            t.q8o_q = e->qt_q;
            t.q8o_d = e->qt_d;
            t.q8o_s = e->qt_s;
            if (kind == K_PREFILL && (r = launch_kvwrite(t, e->stream, true)) != cudaSuccess) return r;
            t.trace = e->trace_slot(100, e->n_head * ncol);
            if ((r = launch_attn(t, e->stream, true)) != cudaSuccess) return r;
            a = b;
            a.q8_q = e->qt_q;
            a.q8_d = e->qt_d;
            a.q8_s = e->qt_s;
            a.out = e->y;
            a.out_stride = E;
            if ((r = table_launch(e, L.o, P_Q8IN, E_STORE, a)) != cudaSuccess) return r;
        }
        a = b;
        a.in = e->y;
        a.in_stride = E;
        a.xin = X0;
        a.xout = X1;
        a.wpost = e->f32(L.post_attn_norm);
        a.wpre = e->f32(L.ffn_norm);
        a.out = e->act;
        a.out_stride = e->n_ff;
        a.q8o_q = e->qa_q;
        a.q8o_d = e->qa_d;
        a.q8o_s = e->qa_s;
        if (L.conv && kind != K_DECODE) {
            a.ring_layer = L.ci;
            a.ring_src = e->big;
            a.ring_src_stride = e->big_n;
        }
        if ((r = table_launch(e, L.gate_up, P_RESID_NORM, E_SILU, a)) != cudaSuccess) return r;
        a = b;
        a.q8_q = e->qa_q;
        a.q8_d = e->qa_d;
        a.q8_s = e->qa_s;
        a.out = e->fo;
        a.out_stride = E;
        if ((r = table_launch(e, L.down, P_Q8IN, E_STORE, a)) != cudaSuccess) return r;
    }
    const LayerRef &last = e->layers.back();
    if (head && !e->tok_q6k) {
        MvArgs a = b;
        a.in = e->fo;
        a.in_stride = E;
        a.xin = X1;
        a.wpost = e->f32(last.post_ffn_norm);
        a.wpre = e->f32(e->out_norm);
        return table_launch(e, e->tok, P_FINAL, E_HEAD, a);
    }
    FinalArgs fa = {};
    fa.cols_d = e->cols_d;
    fa.ncol = ncol;
    fa.in = e->fo;
    fa.in_stride = E;
    fa.xin = X1;
    fa.x_stride = 2 * E;
    fa.wpost = e->f32(last.post_ffn_norm);
    fa.out_norm = e->f32(e->out_norm);
    fa.eps = e->eps;
    fa.n_embd = E;
    fa.trace = e->trace_slot(101, ncol);
    if (head) {   // Q6_K word table: the final norm also cuts the hidden state; the word-score launch ends the step
        fa.q8k_q = e->q8k_q;
        fa.q8k_d = e->q8k_d;
        fa.q8k_b = e->q8k_b;
        if ((r = launch_final(fa, e->stream, true)) != cudaSuccess) return r;
        return q6k_head_launch(e, ncol);
    }
    return launch_final(fa, e->stream, true);
}

// one read of table t by the tensor-core batched path for the columns prepared in tc_xb
cudaError_t tc_read(imi_cuda_engine *e, const TableRef &t, int ncol, int epi, float *out, int out_stride) {
    TcArgs a = t.tc;
    a.ncol = ncol;
    a.G = tc_group(t.rows, ncol, e->sm_count);
    a.groups = (ncol + a.G - 1) / a.G;
    a.xb = e->tc_xb;
    a.out = out;
    a.out_stride = out_stride;
    a.epi = epi;
    a.cols_d = e->cols_d;
    a.done = e->done;
    a.err = e->err;
    const int units = (t.rows + TC_M - 1) / TC_M * a.groups;
    return launch_tc_table(a, std::min(e->sm_count, units), e->stream, true);
}

// the step schedule of the tensor-core batched path (more than 8 columns): before every table read one launch
// prepares the columns' inputs (k_tc_prep, one CTA per column), then the read (k_tc_table); attention as in the
// small-batch schedule. Same float order as enqueue_step's schedule, column by column.
cudaError_t enqueue_batch(imi_cuda_engine *e, int ncol, bool head, StepKind kind) {
    const int E = e->n_embd, HD = e->n_head * e->head_dim;
    TcPrepArgs p0 = {};
    p0.cols_d = e->cols_d;
    p0.ncol = ncol;
    p0.xb = e->tc_xb;
    p0.eps = e->eps;
    p0.n_embd = E;
    p0.d_conv = e->d_conv;
    p0.emb = e->w + e->tok.off;
    p0.emb_row_bytes = e->tok.row_bytes;
    p0.emb_q6k = 0;
    p0.x_stride = 2 * E;
    p0.ring_layer = -1;
    float *X0 = e->X, *X1 = e->X + E;
    cudaError_t r;
    // the input preparation of the read of table t: the columns' operand in the layout of t's column group width
    auto prep = [&](TcPrepArgs p, int K, const TableRef &t) {
        p.K = K;
        p.G = tc_group(t.rows, ncol, e->sm_count);
        return launch_tc_prep(p, e->stream, true);
    };
    if (kind == K_HEAD_ONLY) {   // word scores of a hidden state already computed (seoul.cpp:507-516)
        TcPrepArgs p = p0;
        p.pro = TP_CUT;
        p.in = e->hid;
        p.in_stride = E;
        if ((r = prep(p, E, e->tok)) != cudaSuccess) return r;
        return tc_read(e, e->tok, ncol, TE_HEAD, nullptr, 0);
    }
    for (int il = 0; il < e->n_layer; il++) {
        const LayerRef &L = e->layers[il];
        TcPrepArgs p = p0;
        p.pro = il > 0 ? TP_RESID_NORM : TP_EMBED_NORM;
        p.in = e->fo;
        p.in_stride = E;
        p.xin = X1;
        p.xout = X0;
        p.wpost = il > 0 ? e->f32(e->layers[il - 1].post_ffn_norm) : nullptr;
        p.wpre = e->f32(L.attn_norm);
        if ((r = prep(p, E, L.conv ? L.in_proj : L.qkvg)) != cudaSuccess) return r;
        if ((r = tc_read(e, L.conv ? L.in_proj : L.qkvg, ncol, TE_STORE, e->big, e->big_n)) != cudaSuccess) return r;
        if (L.conv) {
            p = p0;
            p.pro = TP_CONV;
            p.in = e->big;
            p.in_stride = e->big_n;
            p.conv_w = e->f32(L.conv_w);
            p.conv_layer = L.ci;
            p.ring_conv = kind == K_DECODE;   // distinct conversations: the conv's own input goes to memory here
            if ((r = prep(p, E, L.out_proj)) != cudaSuccess) return r;
            if ((r = tc_read(e, L.out_proj, ncol, TE_STORE, e->y, E)) != cudaSuccess) return r;
        } else {
            AttnArgs t = {};
            t.cols_d = e->cols_d;
            t.ncol = ncol;
            t.qkv = e->big;
            t.qkv_stride = e->big_n;
            t.att = e->att;
            t.att_stride = HD;
            t.q_norm = e->f32(L.q_norm);
            t.k_norm = e->f32(L.k_norm);
            t.eps = e->eps;
            t.scale = 1.0f / sqrtf((float) e->head_dim);   // seoul.cpp:432
            const size_t per = (size_t) e->n_ctx * (e->head_dim / 2);
            t.rope_cs = e->rope_cs + (L.swa ? per : 0);
            t.rope_sn = e->rope_sn + (L.swa ? per : 0);
            t.ai = L.ai;
            t.n_head = e->n_head;
            t.n_head_kv = e->n_head_kv;
            t.head_dim = e->head_dim;
            t.n_ctx = e->n_ctx;
            t.window = (L.swa && e->n_swa > 0) ? e->n_swa : 0;   // seoul.cpp:431
            t.err = e->err;
            t.kv_fused = kind == K_DECODE;
            t.q8o_q = e->qt_q;
            t.q8o_d = e->qt_d;
            t.q8o_s = e->qt_s;
            if (kind == K_PREFILL && (r = launch_kvwrite(t, e->stream, true)) != cudaSuccess) return r;
            // many columns: one CTA per (kv head, column) reads each cached row once for the heads sharing it
            const bool grp = attn_grp_supported(e->head_dim, e->n_head / e->n_head_kv, e->n_ctx);
            if ((r = (grp ? launch_attn_grp : launch_attn)(t, e->stream, true)) != cudaSuccess) return r;
            p = p0;
            p.pro = TP_Q8;
            p.q8_q = e->qt_q;
            p.q8_d = e->qt_d;
            p.q8_s = e->qt_s;
            if ((r = prep(p, HD, L.o)) != cudaSuccess) return r;
            if ((r = tc_read(e, L.o, ncol, TE_STORE, e->y, E)) != cudaSuccess) return r;
        }
        p = p0;
        p.pro = TP_RESID_NORM;
        p.in = e->y;
        p.in_stride = E;
        p.xin = X0;
        p.xout = X1;
        p.wpost = e->f32(L.post_attn_norm);
        p.wpre = e->f32(L.ffn_norm);
        if (L.conv && kind != K_DECODE) {   // a prefill chunk's conv memory, one launch after the conv read it
            p.ring_layer = L.ci;
            p.ring_src = e->big;
            p.ring_src_stride = e->big_n;
        }
        if ((r = prep(p, E, L.gate_up)) != cudaSuccess) return r;
        if ((r = tc_read(e, L.gate_up, ncol, TE_SILU, e->act, e->n_ff)) != cudaSuccess) return r;
        p = p0;
        p.pro = TP_CUT;
        p.in = e->act;
        p.in_stride = e->n_ff;
        if ((r = prep(p, e->n_ff, L.down)) != cudaSuccess) return r;
        if ((r = tc_read(e, L.down, ncol, TE_STORE, e->fo, E)) != cudaSuccess) return r;
    }
    const LayerRef &last = e->layers.back();
    if (head) {
        TcPrepArgs p = p0;
        p.pro = TP_FINAL;
        p.in = e->fo;
        p.in_stride = E;
        p.xin = X1;
        p.wpost = e->f32(last.post_ffn_norm);
        p.wpre = e->f32(e->out_norm);
        if ((r = prep(p, E, e->tok)) != cudaSuccess) return r;
        return tc_read(e, e->tok, ncol, TE_HEAD, nullptr, 0);
    }
    FinalArgs fa = {};
    fa.cols_d = e->cols_d;
    fa.ncol = ncol;
    fa.in = e->fo;
    fa.in_stride = E;
    fa.xin = X1;
    fa.x_stride = 2 * E;
    fa.wpost = e->f32(last.post_ffn_norm);
    fa.out_norm = e->f32(e->out_norm);
    fa.eps = e->eps;
    fa.n_embd = E;
    return launch_final(fa, e->stream, true);
}

imi_cuda_status run_step(imi_cuda_engine *e, int ncol, bool head, StepKind kind, bool copy_cols) {
    e->gen++;
    e->last_n = ncol;
    for (int c = 0; c < e->last_n; c++) e->last_s[c] = e->cols_h[c].s;
    if (copy_cols) {
        // the batched attention's launch order: columns by decreasing attended position (ties by index); greedy
        // replays keep it (every column moves on by one)
        std::vector<int> idx(ncol);
        for (int c = 0; c < ncol; c++) idx[c] = c;
        std::stable_sort(idx.begin(), idx.end(), [&](int x, int y) {
            return e->cols_pos[x] + e->cols_h[x].off > e->cols_pos[y] + e->cols_h[y].off;
        });
        for (int r = 0; r < ncol; r++) e->cols_h[r].order = idx[r];
        CK(cudaMemcpyAsync(e->cols_d, e->cols_h, sizeof(Col) * ncol, cudaMemcpyHostToDevice, e->stream));
        CK(cudaEventRecord(e->staged, e->stream));
    }
    const int key = ncol * 8 + (head ? 4 : 0) + (int) kind;
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t g = nullptr;
        CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
        const cudaError_t r = ncol > STEP_COLS ? enqueue_batch(e, ncol, head, kind) : enqueue_step(e, ncol, head, kind);
        const cudaError_t r2 = cudaStreamEndCapture(e->stream, &g);
        if (r != cudaSuccess || r2 != cudaSuccess) {
            if (g) cudaGraphDestroy(g);
            return fail(IMI_E_CUDA, std::string("step capture: ") + cudaGetErrorString(r != cudaSuccess ? r : r2));
        }
        cudaGraphExec_t ge = nullptr;
        const cudaError_t r3 = cudaGraphInstantiate(&ge, g, 0);
        cudaGraphDestroy(g);
        if (r3 != cudaSuccess) return fail(IMI_E_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(r3));
        it = e->graphs.emplace(key, ge).first;
    }
    CK(cudaEventRecord(e->t0, e->stream));
    CK(cudaGraphLaunch(it->second, e->stream));
    CK(cudaEventRecord(e->t1, e->stream));
    e->timed = true;
    return IMI_OK;
}

// the staging buffers may be rewritten once the previous step's copy has run
imi_cuda_status staging_wait(imi_cuda_engine *e) {
    CK(cudaEventSynchronize(e->staged));
    return IMI_OK;
}

Col decode_col(imi_cuda_state *s, int32_t token, bool has_embd, int c, bool want) {
    imi_cuda_engine *e = s->e;
    Col k = {};
    k.s = s->s;
    k.kc = s->kc;
    k.vc = s->vc;
    k.ring = s->ring;
    k.hid_out = s->hidden;
    k.logits = want ? s->logits : nullptr;
    k.embd = has_embd ? e->embd + (size_t) c * e->n_embd : nullptr;
    k.picks = s->picks;
    k.token = token >= 0 ? token : (has_embd ? -1 : -2);
    k.off = 0;
    k.pos_inc = 1;
    k.order = c;
    e->cols_pos[c] = s->pos;
    return k;
}

static_assert(sizeof(SessDev) <= 32, "a session record fits its slot of the reply buffer");
imi_cuda_status check_err(imi_cuda_engine *e) {
    int *hp = (int *) (e->reply_h + 32 * e->ncmax);
    CK(cudaMemcpyAsync(hp, e->err, 4, cudaMemcpyDeviceToHost, e->stream));
    CK(cudaStreamSynchronize(e->stream));
    const int h = *hp;
    if (h) {
        CK(cudaMemsetAsync(e->err, 0, 4, e->stream));
        return fail(IMI_E_TIMEOUT, "a device-side wait gave up (code " + std::to_string(h) + ")");
    }
    return IMI_OK;
}

// one decode step of n <= STEP_COLS distinct conversations
imi_cuda_status step_group(imi_cuda_state *const *s, int n, const int32_t *tokens, const float *embd,
                           const int *want, bool any_logits_forced) {
    imi_cuda_engine *e = s[0]->e;
    imi_cuda_status st;
    if ((st = staging_wait(e)) != IMI_OK) return st;
    bool head = any_logits_forced;
    bool any_embd = false;
    for (int c = 0; c < n; c++) {
        const int32_t t = tokens ? tokens[c] : -1;
        if (t >= e->n_vocab) return fail(IMI_E_ARG, "token out of range");
        const bool he = t < 0;
        if (he && !embd) return fail(IMI_E_ARG, "no token and no input vector");
        if (he) memcpy(e->embd_h + (size_t) c * e->n_embd, embd + (size_t) c * e->n_embd, (size_t) e->n_embd * 4);
        any_embd |= he;
        const bool w = want ? want[c] != 0 : true;
        head |= w;
        e->cols_h[c] = decode_col(s[c], t, he, c, w);
    }
    if (any_embd) CK(cudaMemcpyAsync(e->embd, e->embd_h, (size_t) n * e->n_embd * 4, cudaMemcpyHostToDevice, e->stream));
    if ((st = run_step(e, n, head, K_DECODE, true)) != IMI_OK) return st;
    for (int c = 0; c < n; c++) s[c]->pos++;
    return IMI_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------------------------------
// C-ABI
// ---------------------------------------------------------------------------------------------------------------
extern "C" {

const char *imi_cuda_error(void) { return g_err.c_str(); }

imi_cuda_status imi_cuda_load(const char *path, int device, int n_ctx, int max_batch, imi_cuda_engine **out) {
    if (!out) return fail(IMI_E_ARG, "out is null");
    *out = nullptr;
    return load_impl(path, device, n_ctx, max_batch, out);
}

void imi_cuda_free(imi_cuda_engine *e) { delete e; }

imi_cuda_status imi_cuda_get_info(const imi_cuda_engine *e, imi_cuda_info *o) {
    if (!e || !o) return fail(IMI_E_ARG, "null argument");
    o->n_embd = e->n_embd; o->n_vocab = e->n_vocab; o->n_ctx = e->n_ctx; o->n_layer = e->n_layer; o->n_attn = e->n_attn;
    o->n_head = e->n_head; o->n_head_kv = e->n_head_kv; o->head_dim = e->head_dim; o->n_ff = e->n_ff;
    o->d_conv = e->d_conv; o->n_swa = e->n_swa; o->max_batch = e->max_batch;
    o->weight_bytes = e->w_bytes;
    o->state_bytes = e->state_bytes;
    o->cols_per_read = e->ncmax;
    return IMI_OK;
}

namespace {
// cuTensorMapEncodeTiled from the driver, looked up once
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_encode_mu;
cudaError_t encode_fn() {
    std::lock_guard<std::mutex> g(g_encode_mu);
    if (g_encode) return cudaSuccess;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    const cudaError_t r = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (r != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000) fn;
    return cudaSuccess;
}
// the attention's view of a conversation's K or V cache (head_dim 64): rows of 64 fp16 values, [n_attn * n_kv *
// n_ctx] of them, read in boxes of ATK_T rows with the 128-byte swizzle (kernels.cu: k_attn_tma)
cudaError_t kv_tensor_map(const imi_cuda_engine *e, const __half *kc, CUtensorMap *out) {
    cudaError_t r = encode_fn();
    if (r != cudaSuccess) return r;
    const cuuint64_t rows = (cuuint64_t) e->n_attn * e->n_head_kv * e->n_ctx;
    cuuint64_t dims[2] = { (cuuint64_t) ATK_D, rows }, strides[1] = { (cuuint64_t) ATK_D * 2 };
    cuuint32_t box[2] = { (cuuint32_t) ATK_D, (cuuint32_t) ATK_T }, es[2] = { 1, 1 };
    const CUresult c = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, (void *) kc, dims, strides, box, es,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return c == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}
}  // namespace

imi_cuda_status imi_cuda_state_new(imi_cuda_engine *e, imi_cuda_state **out) {
    if (!e || !out) return fail(IMI_E_ARG, "null argument");
    e->gen++;
    CK(cudaSetDevice(e->device));
    std::unique_ptr<imi_cuda_state> s(new imi_cuda_state);
    s->e = e;
    const int E = e->n_embd, kvd = e->n_head_kv * e->head_dim;
    size_t o = 0;
    auto take = [&](size_t n) { const size_t r = o; o = (o + n + 255) / 256 * 256; return r; };
    const size_t o_s = take(ATK_TMAP_OFF + 2 * sizeof(CUtensorMap)), o_k = take((size_t) e->n_attn * e->n_ctx * kvd * 2),
                 o_v = take((size_t) e->n_attn * e->n_ctx * kvd * 2),
                 o_r = take((size_t) e->n_conv * (e->d_conv + 1) * E * 4), o_h = take((size_t) E * 4),
                 o_l = take((size_t) e->n_vocab * 4), o_p = take((size_t) e->n_ctx * 4);
    DALLOC(e, s->mem, o);
    s->mem_bytes = o;
    uint8_t *m = (uint8_t *) s->mem;
    s->s = (SessDev *) (m + o_s);
    s->kc = (__half *) (m + o_k);
    s->vc = (__half *) (m + o_v);
    s->ring = (float *) (m + o_r);
    s->hidden = (float *) (m + o_h);
    s->logits = (float *) (m + o_l);
    s->picks = (int *) (m + o_p);
    CK(cudaMemsetAsync(s->mem, 0, o, e->stream));
    CK(cudaStreamSynchronize(e->stream));
    if (e->head_dim == ATK_D && e->n_attn > 0) {   // the attention's K and V tensor maps, in the record after SessDev
        static_assert(sizeof(SessDev) <= ATK_TMAP_OFF, "record slot");
        CUtensorMap tm[2];
        CK(kv_tensor_map(e, s->kc, &tm[0]));
        CK(kv_tensor_map(e, s->vc, &tm[1]));
        CK(cudaMemcpy((uint8_t *) s->s + ATK_TMAP_OFF, tm, sizeof tm, cudaMemcpyHostToDevice));
    }
    *out = s.release();
    return IMI_OK;
}

void imi_cuda_state_free(imi_cuda_state *s) {
    if (!s) return;
    s->e->gen++;
    cudaSetDevice(s->e->device);
    cudaStreamSynchronize(s->e->stream);
    cudaFree(s->mem);
    s->e->dev_used -= s->mem_bytes;
    delete s;
}

imi_cuda_status imi_cuda_state_reset(imi_cuda_state *s) {
    if (!s) return fail(IMI_E_ARG, "null state");
    imi_cuda_engine *e = s->e;
    CK(cudaSetDevice(e->device));
    e->gen++;
    CK(cudaMemsetAsync(s->s, 0, sizeof(SessDev), e->stream));
    CK(cudaMemsetAsync(s->ring, 0, (size_t) e->n_conv * (e->d_conv + 1) * e->n_embd * 4, e->stream));
    s->pos = 0;
    return IMI_OK;
}

int imi_cuda_state_pos(const imi_cuda_state *s) { return s ? s->pos : -1; }

imi_cuda_status imi_cuda_step(imi_cuda_state *s, int32_t token, const float *embd, int want_logits) {
    if (!s) return fail(IMI_E_ARG, "null state");
    if (s->pos >= s->e->n_ctx) return fail(IMI_E_CTX_FULL, "context full (" + std::to_string(s->e->n_ctx) + ")");
    CK(cudaSetDevice(s->e->device));
    imi_cuda_state *const arr[1] = { s };
    const int w = want_logits != 0;
    return step_group(arr, 1, &token, embd, &w, false);
}

imi_cuda_status imi_cuda_step2(imi_cuda_state *a, int32_t ta, const float *ea, int la, imi_cuda_state *b, int32_t tb,
                               const float *eb, int lb) {
    if (!a || !b || a == b || a->e != b->e) return fail(IMI_E_ARG, "step2 needs two states of one engine");
    imi_cuda_engine *e = a->e;
    if (a->pos >= e->n_ctx || b->pos >= e->n_ctx) return fail(IMI_E_CTX_FULL, "context full (" + std::to_string(e->n_ctx) + ")");
    CK(cudaSetDevice(e->device));
    imi_cuda_state *const arr[2] = { a, b };
    const int32_t t[2] = { ta, tb };
    const int w[2] = { la != 0, lb != 0 };
    std::vector<float> emb;
    const float *ep = nullptr;
    if (ta < 0 || tb < 0) {
        emb.assign((size_t) 2 * e->n_embd, 0.0f);
        if (ta < 0) { if (!ea) return fail(IMI_E_ARG, "no token and no input vector"); memcpy(emb.data(), ea, (size_t) e->n_embd * 4); }
        if (tb < 0) { if (!eb) return fail(IMI_E_ARG, "no token and no input vector"); memcpy(emb.data() + e->n_embd, eb, (size_t) e->n_embd * 4); }
        ep = emb.data();
    }
    return step_group(arr, 2, t, ep, w, false);
}

imi_cuda_status imi_cuda_step_multi(imi_cuda_state *const *s, int n, const int32_t *tokens, const float *embd,
                                    const int *want_logits) {
    if (!s || n <= 0) return fail(IMI_E_ARG, "no states");
    imi_cuda_engine *e = s[0]->e;
    if (n > e->max_batch) return fail(IMI_E_ARG, "more states than max_batch");
    for (int i = 0; i < n; i++) {
        if (!s[i] || s[i]->e != e) return fail(IMI_E_ARG, "states of another engine");
        for (int j = 0; j < i; j++) if (s[j] == s[i]) return fail(IMI_E_ARG, "a state appears twice");
        if (s[i]->pos >= e->n_ctx) return fail(IMI_E_CTX_FULL, "context full (" + std::to_string(e->n_ctx) + ")");
    }
    CK(cudaSetDevice(e->device));
    for (int i0 = 0; i0 < n; i0 += e->ncmax) {   // all of them in one read when the batched path runs them
        const int m = std::min(e->ncmax, n - i0);
        std::vector<int32_t> t(m);
        for (int c = 0; c < m; c++) t[c] = tokens ? tokens[i0 + c] : -1;
        imi_cuda_status st = step_group(s + i0, m, t.data(), embd ? embd + (size_t) i0 * e->n_embd : nullptr,
                                        want_logits ? want_logits + i0 : nullptr, false);
        if (st != IMI_OK) return st;
    }
    return IMI_OK;
}

imi_cuda_status imi_cuda_step_batch(imi_cuda_state *s, const int32_t *tokens, const float *embd, int n, int want_logits,
                                    float *hidden_all) {
    if (!s || n <= 0 || (!tokens && !embd)) return fail(IMI_E_ARG, "bad step_batch arguments");
    imi_cuda_engine *e = s->e;
    const int E = e->n_embd;
    CK(cudaSetDevice(e->device));
    // imi checks the context per 64 positions and steps every group before the first that would pass n_ctx
    // (seoul.cpp:496-498); the positions of those groups are read here in chunks of up to ncmax (one table read each)
    int n_ok = 0;
    for (int g0 = 0; g0 < n; g0 += BATCH_GROUP) {
        const int gn = std::min(BATCH_GROUP, n - g0);
        if (s->pos + g0 + gn > e->n_ctx) break;
        n_ok = g0 + gn;
    }
    {
        for (int i0 = 0; i0 < n_ok; i0 += e->ncmax) {
            const int m = std::min(e->ncmax, n_ok - i0);
            imi_cuda_status st;
            if ((st = staging_wait(e)) != IMI_OK) return st;
            for (int c = 0; c < m; c++) {
                const int32_t t = tokens ? tokens[i0 + c] : -1;
                if (t >= e->n_vocab) return fail(IMI_E_ARG, "token out of range");
                if (t < 0) memcpy(e->embd_h + (size_t) c * E, embd + (size_t) (i0 + c) * E, (size_t) E * 4);
                Col k = decode_col(s, t, t < 0, c, false);
                k.hid_out = e->hid + (size_t) c * E;
                k.off = c;
                k.pos_inc = c == m - 1 ? m : 0;
                e->cols_h[c] = k;
            }
            if (!tokens) CK(cudaMemcpyAsync(e->embd, e->embd_h, (size_t) m * E * 4, cudaMemcpyHostToDevice, e->stream));
            if ((st = run_step(e, m, false, K_PREFILL, true)) != IMI_OK) return st;
            CK(cudaMemcpyAsync(s->hidden, e->hid + (size_t) (m - 1) * E, (size_t) E * 4, cudaMemcpyDeviceToDevice, e->stream));
            if (hidden_all) {
                CK(cudaMemcpyAsync(hidden_all + (size_t) i0 * E, e->hid, (size_t) m * E * 4, cudaMemcpyDeviceToHost, e->stream));
                CK(cudaStreamSynchronize(e->stream));
            }
            s->pos += m;
        }
    }
    if (n_ok < n) return fail(IMI_E_CTX_FULL, "context full (" + std::to_string(e->n_ctx) + ")");
    if (want_logits) {   // the last position's word scores (seoul.cpp:507-516)
        imi_cuda_status st;
        if ((st = staging_wait(e)) != IMI_OK) return st;
        Col k = decode_col(s, 0, false, 0, true);
        k.off = -1;
        k.pos_inc = 0;
        e->cols_h[0] = k;
        CK(cudaMemcpyAsync(e->hid, s->hidden, (size_t) E * 4, cudaMemcpyDeviceToDevice, e->stream));
        if ((st = run_step(e, 1, true, K_HEAD_ONLY, true)) != IMI_OK) return st;
    }
    return IMI_OK;
}

imi_cuda_status imi_cuda_greedy(imi_cuda_state *const *s, int n, const int32_t *tokens, int steps, int32_t *ids) {
    if (!s || n <= 0 || steps <= 0) return fail(IMI_E_ARG, "bad greedy arguments");
    imi_cuda_engine *e = s[0]->e;
    if (n > e->max_batch && n > STEP_COLS) return fail(IMI_E_ARG, "more conversations than max_batch");
    if (n > e->ncmax) {   // groups of ncmax conversations, each group all its steps (conversations are independent)
        for (int i = 0; i < n; i++)
            for (int j = 0; j < i; j++) if (s[j] == s[i]) return fail(IMI_E_ARG, "a state appears twice");
        std::vector<int32_t> part((size_t) steps * e->ncmax);
        for (int g0 = 0; g0 < n; g0 += e->ncmax) {
            const int m = std::min(e->ncmax, n - g0);
            const imi_cuda_status st = imi_cuda_greedy(s + g0, m, tokens ? tokens + g0 : nullptr, steps,
                                                       ids ? part.data() : nullptr);
            if (st != IMI_OK) return st;
            if (ids)
                for (int k = 0; k < steps; k++)
                    for (int c = 0; c < m; c++) ids[(size_t) k * n + g0 + c] = part[(size_t) k * m + c];
        }
        return IMI_OK;
    }
    for (int i = 0; i < n; i++) {
        if (!s[i] || s[i]->e != e) return fail(IMI_E_ARG, "states of another engine");
        for (int j = 0; j < i; j++) if (s[j] == s[i]) return fail(IMI_E_ARG, "a state appears twice");
        if (s[i]->pos + steps > e->n_ctx) return fail(IMI_E_CTX_FULL, "context full (" + std::to_string(e->n_ctx) + ")");
    }
    CK(cudaSetDevice(e->device));
    std::vector<int> pos0(n);
    for (int i = 0; i < n; i++) pos0[i] = s[i]->pos;
    imi_cuda_status st;
    if ((st = staging_wait(e)) != IMI_OK) return st;
    for (int c = 0; c < n; c++) e->cols_h[c] = decode_col(s[c], tokens ? tokens[c] : -2, false, c, true);
    if ((st = run_step(e, n, true, K_DECODE, true)) != IMI_OK) return st;
    for (int c = 0; c < n; c++) s[c]->pos++;
    if (steps > 1) {
        if ((st = staging_wait(e)) != IMI_OK) return st;
        for (int c = 0; c < n; c++) e->cols_h[c].token = -2;
        if ((st = run_step(e, n, true, K_DECODE, true)) != IMI_OK) return st;
        for (int c = 0; c < n; c++) s[c]->pos++;
        for (int k = 2; k < steps; k++) {
            if ((st = run_step(e, n, true, K_DECODE, false)) != IMI_OK) return st;
            for (int c = 0; c < n; c++) s[c]->pos++;
        }
    }
    if (ids) {
        std::vector<int32_t> tmp((size_t) steps);
        for (int c = 0; c < n; c++) {
            CK(cudaMemcpyAsync(tmp.data(), s[c]->picks + pos0[c], (size_t) steps * 4, cudaMemcpyDeviceToHost, e->stream));
            CK(cudaStreamSynchronize(e->stream));
            for (int k = 0; k < steps; k++) ids[(size_t) k * n + c] = tmp[k];
        }
    }
    return check_err(e);
}

imi_cuda_status imi_cuda_get_hidden(const imi_cuda_state *s, float *out) {
    if (!s || !out) return fail(IMI_E_ARG, "null argument");
    CK(cudaSetDevice(s->e->device));
    CK(cudaMemcpyAsync(out, s->hidden, (size_t) s->e->n_embd * 4, cudaMemcpyDeviceToHost, s->e->stream));
    return check_err(s->e);
}

imi_cuda_status imi_cuda_get_logits(const imi_cuda_state *s, float *out) {
    if (!s || !out) return fail(IMI_E_ARG, "null argument");
    CK(cudaSetDevice(s->e->device));
    CK(cudaMemcpyAsync(out, s->logits, (size_t) s->e->n_vocab * 4, cudaMemcpyDeviceToHost, s->e->stream));
    return check_err(s->e);
}

imi_cuda_status imi_cuda_get_argmax(const imi_cuda_state *s, int32_t *id, float *value) {
    if (!s || !id) return fail(IMI_E_ARG, "null argument");
    CK(cudaSetDevice(s->e->device));
    imi_cuda_engine *e = s->e;
    if (e->reply_gen != e->gen) {
        // the records of every conversation of the last step (when s is one of them) and the error word, in one
        // synchronisation: the next conversation's pick of the same step then needs no device round trip
        bool in_last = false;
        for (int c = 0; c < e->last_n; c++) in_last |= e->last_s[c] == s->s;
        e->reply_n = in_last ? e->last_n : 1;
        for (int c = 0; c < e->reply_n; c++) e->reply_src[c] = in_last ? e->last_s[c] : s->s;
        if (in_last && e->reply_n > 1) {   // the records gathered on the device (cols_d still holds the last step's)
            CK(launch_gather_sess(e->cols_d, e->reply_n, (uint8_t *) e->reply_d, e->stream));
            CK(cudaMemcpyAsync(e->reply_h, e->reply_d, (size_t) 32 * e->reply_n, cudaMemcpyDeviceToHost, e->stream));
        } else {
            CK(cudaMemcpyAsync(e->reply_h, s->s, sizeof(SessDev), cudaMemcpyDeviceToHost, e->stream));
        }
        const imi_cuda_status st = check_err(e);
        if (st != IMI_OK) return st;
        e->reply_gen = e->gen;
    }
    for (int c = 0; c < e->reply_n; c++)
        if (e->reply_src[c] == s->s) {
            const SessDev *h = (const SessDev *) (e->reply_h + 32 * c);
            *id = h->next_token;
            if (value) *value = h->amax_val;
            return IMI_OK;
        }
    e->reply_gen = 0;   // not among the records read (cannot happen: s was read above); read again
    return imi_cuda_get_argmax(s, id, value);
}

imi_cuda_status imi_cuda_q6k_scores(int device, const uint8_t *q6k, int rows, int cols, const float *x, float *out,
                                    int8_t *xq, float *xd, int16_t *bsums) {
    if (!q6k || !x || !out || rows <= 0 || cols <= 0 || cols % 256 || cols > 32768)
        return fail(IMI_E_ARG, "bad q6k_scores arguments (cols a multiple of 256, at most 32768)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    const int nb = cols / 256;
    const size_t wbytes = (size_t) rows * nb * 210;
    // one allocation: x | out | q8k codes | scales | code sums | the rows
    auto up = [](size_t n) { return (n + 255) / 256 * 256; };
    const size_t o_x = 0, o_out = up((size_t) cols * 4), o_q = o_out + up((size_t) rows * 4), o_d = o_q + up(cols),
                 o_b = o_d + up((size_t) nb * 4), o_w = o_b + up((size_t) nb * 32), total = o_w + wbytes;
    uint8_t *m = nullptr;
    CK(cudaMalloc(&m, total));
    cudaError_t r = cudaMemcpy(m + o_x, x, (size_t) cols * 4, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(m + o_w, q6k, wbytes, cudaMemcpyHostToDevice);
    if (r == cudaSuccess)
        r = launch_q8k_cut((const float *) (m + o_x), cols, (int8_t *) (m + o_q), (float *) (m + o_d),
                           (int16_t *) (m + o_b), 0);
    if (r == cudaSuccess)
        r = launch_q6k_scores(m + o_w, rows, nb, (const int8_t *) (m + o_q), (const float *) (m + o_d),
                              (const int16_t *) (m + o_b), (float *) (m + o_out), 0);
    if (r == cudaSuccess) r = cudaMemcpy(out, m + o_out, (size_t) rows * 4, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess && xq) r = cudaMemcpy(xq, m + o_q, cols, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess && xd) r = cudaMemcpy(xd, m + o_d, (size_t) nb * 4, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess && bsums) r = cudaMemcpy(bsums, m + o_b, (size_t) nb * 32, cudaMemcpyDeviceToHost);
    cudaFree(m);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("q6k_scores: ") + cudaGetErrorString(r));
    return IMI_OK;
}

imi_cuda_status imi_cuda_q8_cut(int device, const float *x, int n, int8_t *q, float *d, float *s) {
    if (!x || !q || !d || !s || n <= 0 || n % 32) return fail(IMI_E_ARG, "bad q8_cut arguments");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    uint8_t *m = nullptr;
    const size_t nb = (size_t) n / 32;
    CK(cudaMalloc(&m, (size_t) n * 4 + n + 8 * nb + 64));
    float *dx = (float *) m;
    int8_t *dq = (int8_t *) (m + (size_t) n * 4);
    float *dd = (float *) (m + (size_t) n * 5 + (16 - (n * 5) % 16) % 16), *ds = dd + nb;
    cudaError_t r = cudaMemcpy(dx, x, (size_t) n * 4, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = launch_q8_cut(dx, n, dq, dd, ds, 0);
    if (r == cudaSuccess) r = cudaMemcpy(q, dq, n, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess) r = cudaMemcpy(d, dd, nb * 4, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess) r = cudaMemcpy(s, ds, nb * 4, cudaMemcpyDeviceToHost);
    cudaFree(m);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("q8_cut: ") + cudaGetErrorString(r));
    return IMI_OK;
}

imi_cuda_status imi_cuda_q4_matvec(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd,
                                   const float *xs, int ncol, float *out, int32_t *dots) {
    if (!q4 || !xq || !xd || !xs || !out || rows <= 0 || cols <= 0 || cols % 256 || ncol < 1 || ncol > MV_MAX_COLS ||
        (dots && ncol != 1))
        return fail(IMI_E_ARG, "bad q4_matvec arguments (cols a multiple of 256, 1..8 inputs)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    CK(prepare_kernels());
    const int nb = cols / 32, row_bytes = nb * 18;
    std::vector<uint8_t> packed((size_t) rows * row_bytes);
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < nb; j++) {
            const uint8_t *src = q4 + ((size_t) r * nb + j) * 18;
            uint8_t *row = packed.data() + (size_t) r * row_bytes;
            memcpy(row + (size_t) nb * 16 + 2 * j, src, 2);
            memcpy(row + 16 * j, src + 2, 16);
        }
    const size_t b_w = packed.size(), b_q = (size_t) ncol * cols, b_ds = (size_t) ncol * nb * 4,
                 b_o = (size_t) ncol * rows * 4, b_dots = dots ? (size_t) rows * nb * 4 : 0;
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    uint8_t *m = nullptr;
    CK(cudaMalloc(&m, al(b_w) + al(b_q) + 2 * al(b_ds) + al(b_o) + al(b_dots) + al(sizeof(Col) * MV_MAX_COLS) + 256));
    uint8_t *p = m;
    uint8_t *dW = p; p += al(b_w);
    int8_t *dq = (int8_t *) p; p += al(b_q);
    float *dd = (float *) p; p += al(b_ds);
    float *ds = (float *) p; p += al(b_ds);
    float *dout = (float *) p; p += al(b_o);
    int32_t *ddots = dots ? (int32_t *) p : nullptr; p += al(b_dots);
    Col *dcols = (Col *) p; p += al(sizeof(Col) * MV_MAX_COLS);
    int *derr = (int *) p;
    cudaError_t r = cudaMemcpy(dW, packed.data(), b_w, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(dq, xq, b_q, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(dd, xd, b_ds, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(ds, xs, b_ds, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemset(dcols, 0, sizeof(Col) * MV_MAX_COLS + 256);
    if (r == cudaSuccess) {
        MvArgs a = {};
        a.W = dW; a.rows = rows; a.cols = cols; a.row_bytes = row_bytes; a.unit = 1;
        a.cols_d = dcols; a.ncol = ncol; a.q8_q = dq; a.q8_d = dd; a.q8_s = ds; a.dots = ddots;
        a.out = dout; a.out_stride = rows; a.err = derr; a.ring_layer = -1;
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        const int grid = std::max(1, std::min(sms, rows));
        plan_stages(a, P_Q8IN, 1, grid);
        r = launch_table(P_Q8IN, E_STORE, a, grid, 0, false);
    }
    if (r == cudaSuccess) r = cudaMemcpy(out, dout, b_o, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess && dots) r = cudaMemcpy(dots, ddots, b_dots, cudaMemcpyDeviceToHost);
    int herr = 0;
    if (r == cudaSuccess) r = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    cudaFree(m);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("q4_matvec: ") + cudaGetErrorString(r));
    if (herr) return fail(IMI_E_TIMEOUT, "q4_matvec: a device-side wait gave up");
    return IMI_OK;
}

imi_cuda_status imi_cuda_bench_matvec(int device, int rows, int cols, int ncol, int reps, float *ms, size_t *bytes) {
    if (rows <= 0 || cols <= 0 || cols % 256 || ncol < 1 || ncol > 256 || reps < 1 || !ms)
        return fail(IMI_E_ARG, "bad bench_matvec arguments (cols a multiple of 256, 1..256 inputs)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    CK(prepare_kernels());
    int sms = 148;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    const int nb = cols / 32, row_bytes = nb * 18;
    const size_t tb = (size_t) rows * row_bytes, tstride = (tb + 255) / 256 * 256, rot = (size_t) 256 << 20;
    const int copies = (int) std::max<size_t>(1, (rot + tb - 1) / tb);
    // the table (engine layout: codes, then fp16 scales) and the inputs, from a fixed xorshift sequence
    std::vector<uint8_t> host(tb);
    uint64_t x = 0x9E3779B97F4A7C15ull;
    auto next = [&]() { x ^= x << 13; x ^= x >> 7; x ^= x << 17; return x; };
    for (int r = 0; r < rows; r++) {
        uint8_t *row = host.data() + (size_t) r * row_bytes;
        for (int i = 0; i < nb * 16; i += 8) { const uint64_t v = next(); memcpy(row + i, &v, 8); }
        for (int j = 0; j < nb; j++) {   // fp16 scales in [2^-9, 2^-7): exponent 6..7, random mantissa
            const uint16_t h = (uint16_t) (((6 + (next() & 1)) << 10) | (next() & 0x3ff));
            memcpy(row + nb * 16 + 2 * j, &h, 2);
        }
    }
    std::vector<int8_t> hq((size_t) ncol * cols);
    for (auto &q : hq) q = (int8_t) ((int) (next() % 255) - 127);
    std::vector<float> hd((size_t) ncol * nb, 0.01f), hs((size_t) ncol * nb, 0.5f);
    auto al = [](size_t n) { return (n + 255) / 256 * 256; };
    // more than 8 inputs: the tensor-core read, its operands in the MMA's layout
    const bool tc = ncol > MV_MAX_COLS;
    const int G = tc_group(rows, ncol, sms), groups = (ncol + G - 1) / G;
    std::vector<uint8_t> tx;
    if (tc) tc_operands_host(hq.data(), hd.data(), hs.data(), ncol, cols, G, tx);
    const size_t tt = tc ? al(tc_tiled_bytes(rows, cols)) : 0, o_t = (size_t) copies * tstride;   // tiled copies
    const size_t o_q = o_t + (size_t) copies * tt, o_d = o_q + al(hq.size()), o_s = o_d + al(hd.size() * 4),
                 o_o = o_s + al(hs.size() * 4), o_c = o_o + al((size_t) ncol * rows * 4),
                 o_tx = o_c + al(sizeof(Col) * MV_MAX_COLS) + 256, total = o_tx + al(tx.size());
    uint8_t *m = nullptr;
    CK(cudaMalloc(&m, total));
    cudaStream_t st = nullptr;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaError_t r = cudaMemcpy(m, host.data(), tb, cudaMemcpyHostToDevice);
    for (int c = 1; c < copies && r == cudaSuccess; c++) r = cudaMemcpy(m + c * tstride, m, tb, cudaMemcpyDeviceToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(m + o_q, hq.data(), hq.size(), cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(m + o_d, hd.data(), hd.size() * 4, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(m + o_s, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemset(m + o_c, 0, al(sizeof(Col) * MV_MAX_COLS) + 256);
    if (r == cudaSuccess && tc) r = cudaMemcpy(m + o_tx, tx.data(), tx.size(), cudaMemcpyHostToDevice);
    std::vector<TcArgs> tca(tc ? copies : 0);
    for (int c = 0; c < (int) tca.size() && r == cudaSuccess; c++) {
        TcArgs &t = tca[c];
        t.wt = m + o_t + (size_t) c * tt;
        r = launch_tc_tile(m + (size_t) c * tstride, rows, cols, row_bytes, m + o_t + (size_t) c * tt, nullptr);
        t.rows = rows; t.cols = cols; t.ncol = ncol; t.G = G; t.groups = groups;
        t.xb = m + o_tx; t.out = (float *) (m + o_o); t.out_stride = rows;
        t.epi = TE_STORE; t.err = (int *) (m + o_c + al(sizeof(Col) * MV_MAX_COLS));
    }
    if (r == cudaSuccess && tc) r = cudaDeviceSynchronize();   // the tiled copies (default stream) before the reads
    if (r == cudaSuccess) r = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    // one read of all inputs from table copy k: groups of up to 8 inputs per read of the table (the small-batch
    // kernel), programmatic dependent launches one after another as the engine's step runs them
    auto read = [&](int k) -> cudaError_t {
        if (tc) {
            const int units = (rows + TC_M - 1) / TC_M * groups;
            return launch_tc_table(tca[k % copies], std::min(sms, units), st, true);
        }
        for (int c0 = 0; c0 < ncol; c0 += MV_MAX_COLS) {
            MvArgs a = {};
            a.W = m + (size_t) (k % copies) * tstride; a.rows = rows; a.cols = cols; a.row_bytes = row_bytes; a.unit = 1;
            a.cols_d = (const Col *) (m + o_c); a.ncol = std::min(MV_MAX_COLS, ncol - c0);
            a.q8_q = (const int8_t *) (m + o_q) + (size_t) c0 * cols;
            a.q8_d = (const float *) (m + o_d) + (size_t) c0 * nb;
            a.q8_s = (const float *) (m + o_s) + (size_t) c0 * nb;
            a.out = (float *) (m + o_o) + (size_t) c0 * rows; a.out_stride = rows;
            a.err = (int *) (m + o_c + al(sizeof(Col) * MV_MAX_COLS)); a.ring_layer = -1;
            const int grid = std::max(1, std::min(sms, rows));
            plan_stages(a, P_Q8IN, 1, grid);
            const cudaError_t e = launch_table(P_Q8IN, E_STORE, a, grid, st, true);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    };
    // every copy at least once per timed graph, so no read finds its table still in L2 from the previous pass
    const int nreads = std::max(reps, copies);
    if (r == cudaSuccess) r = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (r == cudaSuccess) {
        cudaError_t rc = cudaSuccess;
        for (int i = 0; i < nreads && rc == cudaSuccess; i++) rc = read(i);
        r = cudaStreamEndCapture(st, &g);
        if (rc != cudaSuccess) r = rc;
    }
    if (r == cudaSuccess) r = cudaGraphInstantiate(&ge, g, 0);
    if (r == cudaSuccess) r = cudaEventCreate(&e0);
    if (r == cudaSuccess) r = cudaEventCreate(&e1);
    if (r == cudaSuccess) r = cudaGraphLaunch(ge, st);   // untimed: first touch, code and parameters warm
    if (r == cudaSuccess) r = cudaEventRecord(e0, st);
    if (r == cudaSuccess) r = cudaGraphLaunch(ge, st);
    if (r == cudaSuccess) r = cudaEventRecord(e1, st);
    if (r == cudaSuccess) r = cudaEventSynchronize(e1);
    float t = 0;
    if (r == cudaSuccess) r = cudaEventElapsedTime(&t, e0, e1);
    int herr = 0;
    if (r == cudaSuccess) r = cudaMemcpy(&herr, m + o_c + al(sizeof(Col) * MV_MAX_COLS), 4, cudaMemcpyDeviceToHost);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (ge) cudaGraphExecDestroy(ge);
    if (g) cudaGraphDestroy(g);
    if (st) cudaStreamDestroy(st);
    cudaFree(m);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("bench_matvec: ") + cudaGetErrorString(r));
    if (herr) return fail(IMI_E_TIMEOUT, "bench_matvec: a device-side wait gave up");
    *ms = t / nreads;
    if (bytes) *bytes = tb + hq.size() + 8 * (size_t) ncol * nb + 4 * (size_t) ncol * rows;
    return IMI_OK;
}

static unsigned long long *g_tc_trace_host = nullptr;   // diagnostics: imi_cuda_trace_tc sets it for one call

imi_cuda_status imi_cuda_q4_matmul(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd,
                                   const float *xs, int ncol, float *out) {
    if (!q4 || !xq || !xd || !xs || !out || rows <= 0 || cols <= 0 || cols % 256 || ncol < 1 || ncol > 256)
        return fail(IMI_E_ARG, "bad q4_matmul arguments (cols a multiple of 256, 1..256 inputs)");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    CK(prepare_kernels());
    int sms = 148;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
    const int nb = cols / 32, row_bytes = nb * 18, G = tc_group(rows, ncol, sms), groups = (ncol + G - 1) / G;
    std::vector<uint8_t> packed((size_t) rows * row_bytes);
    for (int r = 0; r < rows; r++)
        for (int j = 0; j < nb; j++) {
            const uint8_t *src = q4 + ((size_t) r * nb + j) * 18;
            uint8_t *row = packed.data() + (size_t) r * row_bytes;
            memcpy(row + (size_t) nb * 16 + 2 * j, src, 2);
            memcpy(row + 16 * j, src + 2, 16);
        }
    std::vector<uint8_t> xb;
    tc_operands_host(xq, xd, xs, ncol, cols, G, xb);
    auto al = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t b_w = packed.size(), b_h = xb.size(), b_o = (size_t) ncol * rows * 4;
    uint8_t *m = nullptr;
    const size_t b_t = (size_t) TC_TRACE_ROWS * TC_TRACE * 8, b_wt = tc_tiled_bytes(rows, cols);
    CK(cudaMalloc(&m, al(b_w) + al(b_h) + al(b_o) + 256 + b_t + al(b_wt)));
    uint8_t *dW = m, *dh = m + al(b_w);
    float *dout = (float *) (dh + al(b_h));
    int *derr = (int *) ((uint8_t *) dout + al(b_o));
    unsigned long long *dtr = (unsigned long long *) ((uint8_t *) derr + 256);
    uint8_t *dwt = (uint8_t *) dtr + b_t;   // the table's tiled copy
    TcArgs a = {};
    if (g_tc_trace_host) {
        a.trace = dtr;
        cudaMemset(dtr, 0, b_t);
    }
    cudaError_t r = cudaMemcpy(dW, packed.data(), b_w, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemcpy(dh, xb.data(), b_h, cudaMemcpyHostToDevice);
    if (r == cudaSuccess) r = cudaMemset(derr, 0, 4);
    if (r == cudaSuccess) r = launch_tc_tile(dW, rows, cols, row_bytes, dwt, nullptr);
    if (r == cudaSuccess) {
        a.wt = dwt; a.rows = rows; a.cols = cols; a.ncol = ncol; a.G = G; a.groups = groups;
        a.xb = dh; a.out = dout; a.out_stride = rows; a.epi = TE_STORE; a.err = derr;
        const int units = (rows + TC_M - 1) / TC_M * groups;
        r = launch_tc_table(a, std::min(sms, units), 0, false);
    }
    if (r == cudaSuccess) r = cudaMemcpy(out, dout, b_o, cudaMemcpyDeviceToHost);
    if (r == cudaSuccess && g_tc_trace_host) r = cudaMemcpy(g_tc_trace_host, dtr, b_t, cudaMemcpyDeviceToHost);
    int herr = 0;
    if (r == cudaSuccess) r = cudaMemcpy(&herr, derr, 4, cudaMemcpyDeviceToHost);
    cudaFree(m);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("q4_matmul: ") + cudaGetErrorString(r));
    if (herr) return fail(IMI_E_TIMEOUT, "q4_matmul: a device-side wait gave up");
    return IMI_OK;
}

imi_cuda_status imi_cuda_trace_tc(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd,
                                  const float *xs, int ncol, float *out, unsigned long long *trace) {
    if (!trace) return fail(IMI_E_ARG, "trace is null");
    g_tc_trace_host = trace;
    const imi_cuda_status st = imi_cuda_q4_matmul(device, q4, rows, cols, xq, xd, xs, ncol, out);
    g_tc_trace_host = nullptr;
    return st;
}

// ---------------------------------------------------------------------------------------------------------------
// the same table read without allocating (imi_cuda_q4_matvec_static)
// ---------------------------------------------------------------------------------------------------------------
// Some callers must not allocate device memory while they run: cudaFree waits for every stream of the device, so a
// caller sharing the GPU with a running decode loop would stall it; a process whose HBM is already held by a memory
// pool or another framework's caching allocator may see a fresh cudaMalloc fail; and a caller on a thread with a
// fixed budget (an audio callback, an allocator hook) may not allocate at all. For them the read below keeps its
// scratch in this library's own device memory, reserved once when the library's device code is loaded into a
// context: [STATIC_HEAD: column descriptors, error flag | the repacked table, at most IMI_CUDA_STATIC_TABLE_BYTES].
namespace {
constexpr size_t STATIC_HEAD = 4096;
constexpr size_t STATIC_ERR = 2048;   // offset of the device-side error flag inside the head
constexpr int STATIC_MAX_DEVICES = 64;
static_assert(sizeof(Col) * MV_MAX_COLS <= STATIC_ERR, "column descriptors overflow the static head");
__device__ __align__(256) uint8_t g_static_scratch[STATIC_HEAD + IMI_CUDA_STATIC_TABLE_BYTES];
std::mutex g_static_mu;
// the scratch's device address, per device (null until looked up), kept for the life of the process together with the
// kernels' shared-memory limits (prepare_kernels): both belong to the device's primary context, so this entry point
// assumes that context is not reset (cudaDeviceReset) while the process uses it
uint8_t *g_static_addr[STATIC_MAX_DEVICES];

bool on_device(const void *p, int device) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) && at.device == device;
}
}  // namespace

imi_cuda_status imi_cuda_q4_matvec_static(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq,
                                          const float *xd, const float *xs, int ncol, float *out, void *stream) {
    if (!q4 || !xq || !xd || !xs || !out || rows <= 0 || cols <= 0 || cols % 256 || ncol < 1 || ncol > MV_MAX_COLS)
        return fail(IMI_E_ARG, "bad q4_matvec_static arguments (cols a multiple of 256, 1..8 inputs)");
    const int nb = cols / 32, row_bytes = nb * 18;
    const size_t table = (size_t) rows * row_bytes;
    if (table > IMI_CUDA_STATIC_TABLE_BYTES)
        return fail(IMI_E_ARG, "q4_matvec_static: the table takes " + std::to_string(table) +
                                   " bytes (rows * cols / 32 * 18); the static scratch holds at most " +
                                   std::to_string((size_t) IMI_CUDA_STATIC_TABLE_BYTES));
    if ((uintptr_t) xq % 16 || (uintptr_t) xd % 4 || (uintptr_t) xs % 4 || (uintptr_t) out % 4)
        return fail(IMI_E_ARG, "q4_matvec_static: xq must be 16-byte aligned, xd, xs and out 4-byte aligned");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= STATIC_MAX_DEVICES)
        return fail(IMI_E_NODEV, "no CUDA device");
    int prev = 0;
    CK(cudaGetDevice(&prev));
    CK(cudaSetDevice(device));
    struct Restore {
        int d;
        ~Restore() { cudaSetDevice(d); }
    } restore{ prev };
    for (const void *p : { (const void *) q4, (const void *) xq, (const void *) xd, (const void *) xs, (const void *) out })
        if (!on_device(p, device))
            return fail(IMI_E_ARG, "q4_matvec_static: every buffer must be device memory of device " + std::to_string(device));
    uint8_t *scratch = nullptr;
    {   // once per device, with that device current: the scratch's address and the kernels' shared-memory limits
        std::lock_guard<std::mutex> g(g_static_mu);
        if (!g_static_addr[device]) {
            CK(prepare_kernels());
            void *p = nullptr;
            const cudaError_t r = cudaGetSymbolAddress(&p, g_static_scratch);
            if (r != cudaSuccess || !p)
                return fail(IMI_E_CUDA, std::string("q4_matvec_static: scratch address: ") + cudaGetErrorString(r));
            g_static_addr[device] = (uint8_t *) p;
        }
        scratch = g_static_addr[device];
    }
    cudaStream_t st = (cudaStream_t) stream;
    Col *dcols = (Col *) scratch;
    int *derr = (int *) (scratch + STATIC_ERR);
    uint8_t *dW = scratch + STATIC_HEAD;
    // the descriptors and the error flag must start at zero: cleared here, on the stream, before the kernels; the
    // table area needs no clearing (the repack writes all of it before the read)
    cudaError_t r = cudaMemsetAsync(scratch, 0, STATIC_HEAD, st);
    if (r == cudaSuccess) r = launch_q4_repack(q4, rows, nb, dW, st);
    if (r == cudaSuccess) {
        MvArgs a = {};
        a.W = dW; a.rows = rows; a.cols = cols; a.row_bytes = row_bytes; a.unit = 1;
        a.cols_d = dcols; a.ncol = ncol; a.q8_q = xq; a.q8_d = xd; a.q8_s = xs;
        a.out = out; a.out_stride = rows; a.err = derr; a.ring_layer = -1;
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        const int grid = std::max(1, std::min(sms, rows));
        plan_stages(a, P_Q8IN, 1, grid);
        r = launch_table(P_Q8IN, E_STORE, a, grid, st, false);
    }
    int herr = 0;
    if (r == cudaSuccess) r = cudaMemcpyAsync(&herr, derr, 4, cudaMemcpyDeviceToHost, st);
    if (r == cudaSuccess) r = cudaStreamSynchronize(st);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("q4_matvec_static: ") + cudaGetErrorString(r));
    if (herr) return fail(IMI_E_TIMEOUT, "q4_matvec_static: a device-side wait gave up");
    return IMI_OK;
}

imi_cuda_status imi_cuda_check_wait_timeout(int device, double limit_ms) {
    if (!(limit_ms > 0.0) || limit_ms > 10000.0) return fail(IMI_E_ARG, "limit_ms must be in (0, 10000]");
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev) return fail(IMI_E_NODEV, "no CUDA device");
    CK(cudaSetDevice(device));
    int khz = 0;
    CK(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device));
    int *err = nullptr;
    CK(cudaMalloc(&err, 4));
    cudaError_t r = cudaMemset(err, 0, 4);
    if (r == cudaSuccess) r = launch_wait_check((long long) (limit_ms * khz), err, 0);
    int h = 0;
    if (r == cudaSuccess) r = cudaMemcpy(&h, err, 4, cudaMemcpyDeviceToHost);
    cudaFree(err);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("check_wait_timeout: ") + cudaGetErrorString(r));
    if (h) return fail(IMI_E_TIMEOUT, "a device-side wait gave up (code " + std::to_string(h) + ")");
    return fail(IMI_E_CUDA, "check_wait_timeout: a wait that nothing completes completed");
}

// ---- the model file's keys and tensor headers ----
struct imi_cuda_file {
    gguf_file f;
    std::map<std::pair<int64_t, uint64_t>, std::string> strs;   // 0-ended copies of the strings asked for
    std::map<int64_t, std::vector<const uint8_t *>> str_at;     // string arrays: where each element starts
    std::mutex mu;
};

imi_cuda_status imi_cuda_file_open(const char *path, imi_cuda_file **out) {
    if (!path || !out) return fail(IMI_E_ARG, "null argument");
    *out = nullptr;
    std::unique_ptr<imi_cuda_file> h(new imi_cuda_file);
    if (!h->f.open(path)) return fail(IMI_E_FILE, h->f.error);
    *out = h.release();
    return IMI_OK;
}
void imi_cuda_file_close(imi_cuda_file *f) { delete f; }
int64_t imi_cuda_file_find_key(const imi_cuda_file *f, const char *key) {
    if (!f || !key) return -1;
    for (size_t k = 0; k < f->f.values.size(); k++)
        if (f->f.values[k].key == key) return (int64_t) k;
    return -1;
}
int64_t imi_cuda_file_n_keys(const imi_cuda_file *f) { return f ? (int64_t) f->f.values.size() : 0; }
static const gguf_value *file_value(const imi_cuda_file *f, int64_t k) {
    return f && k >= 0 && k < (int64_t) f->f.values.size() ? &f->f.values[(size_t) k] : nullptr;
}
const char *imi_cuda_file_key_name(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v ? v->key.c_str() : nullptr;
}
int imi_cuda_file_key_type(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v ? v->type : -1;
}
const void *imi_cuda_file_key_data(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v && v->type != 8 && v->type != 9 ? v->val : nullptr;
}
// a GGUF string (u64 length, bytes) at p as a 0-ended copy kept with the file
static const char *file_str(const imi_cuda_file *f, int64_t k, uint64_t i, const uint8_t *p) {
    imi_cuda_file *m = const_cast<imi_cuda_file *>(f);
    std::lock_guard<std::mutex> g(m->mu);
    auto it = m->strs.find({ k, i });
    if (it == m->strs.end()) {
        uint64_t n;
        memcpy(&n, p, 8);
        it = m->strs.emplace(std::make_pair(k, i), std::string((const char *) p + 8, (size_t) n)).first;
    }
    return it->second.c_str();
}
const char *imi_cuda_file_key_str(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v && v->type == 8 ? file_str(f, k, UINT64_MAX, v->val) : nullptr;
}
int imi_cuda_file_arr_type(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v && v->type == 9 ? v->arr_type : -1;
}
uint64_t imi_cuda_file_arr_n(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v && v->type == 9 ? v->arr_n : 0;
}
const void *imi_cuda_file_arr_data(const imi_cuda_file *f, int64_t k) {
    const gguf_value *v = file_value(f, k);
    return v && v->type == 9 && v->arr_type != 8 ? v->arr : nullptr;
}
const char *imi_cuda_file_arr_str(const imi_cuda_file *f, int64_t k, uint64_t i) {
    const gguf_value *v = file_value(f, k);
    if (!v || v->type != 9 || v->arr_type != 8 || i >= v->arr_n) return nullptr;
    const uint8_t *p = nullptr;
    {   // strings lie one after another: index the array once
        imi_cuda_file *m = const_cast<imi_cuda_file *>(f);
        std::lock_guard<std::mutex> g(m->mu);
        auto &at = m->str_at[k];
        if (at.empty()) {
            at.reserve(v->arr_n);
            const uint8_t *q = v->arr;
            for (uint64_t j = 0; j < v->arr_n; j++) {
                at.push_back(q);
                uint64_t n;
                memcpy(&n, q, 8);
                q += 8 + n;
            }
        }
        p = at[i];
    }
    return file_str(f, k, i, p);
}
int imi_cuda_file_tensor(const imi_cuda_file *f, const char *name, int *type, int64_t ne[4], const void **data,
                         size_t *nbytes) {
    if (!f || !name) return -1;
    const gguf_tensor *t = f->f.tensor(name);
    if (!t) return -1;
    if (type) *type = t->type;
    if (ne)
        for (int d = 0; d < 4; d++) ne[d] = t->ne[d];
    if (data) *data = t->data;
    if (nbytes) *nbytes = t->nbytes;
    return 0;
}

void *imi_cuda_stream(const imi_cuda_engine *e) { return e ? (void *) e->stream : nullptr; }

float imi_cuda_last_step_ms(const imi_cuda_engine *e) {
    if (!e || !e->timed) return 0.0f;
    cudaSetDevice(e->device);
    float ms = 0.0f;
    if (cudaEventSynchronize(e->t1) != cudaSuccess || cudaEventElapsedTime(&ms, e->t0, e->t1) != cudaSuccess) {
        cudaGetLastError();
        return 0.0f;
    }
    return ms;
}

int imi_cuda_launches_per_step(const imi_cuda_engine *e, int n, int want_logits) {
    if (!e || n <= 0) return 0;
    if (n > STEP_COLS && e->tc_batch) {   // the batched path: a preparation launch before every table read
        const int groups = (n + e->ncmax - 1) / e->ncmax;
        int per = 0;
        for (auto &L : e->layers) per += L.conv ? 8 : 9;
        return groups * (per + (want_logits ? 2 : 1));
    }
    const int groups = (n + STEP_COLS - 1) / STEP_COLS;
    int per = 0;
    for (auto &L : e->layers) per += L.conv ? 4 : 5;
    // + the word table (or the final norm without scores); a Q6_K word table takes the final norm and its own read
    return groups * (per + 1 + (e->tok_q6k && want_logits ? 1 : 0));
}

int imi_cuda_launches_per_batch(const imi_cuda_engine *e, int n, int want_logits) {
    if (!e || n <= 0) return 0;
    int reads = 0, launches = 0;
    for (int i0 = 0; i0 < n; i0 += e->ncmax) {
        const int m = std::min(e->ncmax, n - i0);
        int per = 1;   // one read of m positions: its layers, then the final norm
        if (m > STEP_COLS)
            for (auto &L : e->layers) per += L.conv ? 8 : 10;   // a preparation per table; K/V write and attention
        else
            for (auto &L : e->layers) per += L.conv ? 4 : 6;
        launches += per;
        reads++;
    }
    (void) reads;
    return launches + (want_logits ? (e->tok_q6k ? 2 : 1) : 0);
}

imi_cuda_status imi_cuda_bench_tables(imi_cuda_engine *e, int ncol, int reps, float *ms, size_t *bytes) {
    if (!e || ncol < 1 || ncol > e->ncmax || reps < 1 || !ms) return fail(IMI_E_ARG, "bad bench_tables arguments");
    CK(cudaSetDevice(e->device));
    std::vector<const TableRef *> ws;
    for (auto &L : e->layers)
        for (const TableRef *t : { &L.in_proj, &L.out_proj, &L.qkvg, &L.o, &L.gate_up, &L.down })
            if (t->rows) ws.push_back(t);
    size_t b = 0;
    for (auto *t : ws) b += (size_t) t->rows * t->row_bytes;
    if (bytes) *bytes = b;
    // inputs: the act scratch (zeros after allocation is fine: the integer work does not depend on values)
    CK(cudaMemsetAsync(e->X, 0, (size_t) (2 * e->n_embd + e->big_n + e->n_embd + e->n_head * e->head_dim + e->n_ff) * 4 * STEP_COLS, e->stream));
    auto pass = [&]() -> cudaError_t {
        for (auto *t : ws) {
            if (ncol > STEP_COLS) {   // the tensor-core batched read (operands as left in its buffers; outputs to X)
                const cudaError_t r = tc_read(e, *t, ncol, TE_STORE, e->X, t->rows);
                if (r != cudaSuccess) return r;
                continue;
            }
            MvArgs a = {};
            a.cols_d = e->cols_d; a.ncol = ncol; a.eps = e->eps; a.n_embd = e->n_embd; a.ring_layer = -1;
            a.err = e->err; a.q8_q = e->qa_q; a.q8_d = e->qa_d; a.q8_s = e->qa_s; a.out = e->big; a.out_stride = 0;
            cudaError_t r = table_launch(e, *t, P_Q8IN, E_STORE, a);   // codes given: big holds >= 2 n_ff floats
            if (r != cudaSuccess) return r;
        }
        return cudaSuccess;
    };
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    CK(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
    const cudaError_t r = pass();
    const cudaError_t r2 = cudaStreamEndCapture(e->stream, &g);
    if (r != cudaSuccess || r2 != cudaSuccess) { if (g) cudaGraphDestroy(g); return fail(IMI_E_CUDA, "bench_tables capture"); }
    const cudaError_t r3 = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (r3 != cudaSuccess) return fail(IMI_E_CUDA, "bench_tables instantiate");
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaGraphLaunch(ge, e->stream));
    CK(cudaEventRecord(e0, e->stream));
    for (int i = 0; i < reps; i++) CK(cudaGraphLaunch(ge, e->stream));
    CK(cudaEventRecord(e1, e->stream));
    CK(cudaEventSynchronize(e1));
    float t = 0;
    CK(cudaEventElapsedTime(&t, e0, e1));
    *ms = t / reps;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(ge);
    return check_err(e);
}

imi_cuda_status imi_cuda_trace_table(imi_cuda_engine *e, int layer, int which, int ncol, unsigned long long *trace,
                                     int *grid) {
    if (!e || !trace || !grid || layer < 0 || layer >= e->n_layer || which < 0 || which > 3 || ncol < 1 ||
        ncol > STEP_COLS)
        return fail(IMI_E_ARG, "bad trace_table arguments");
    CK(cudaSetDevice(e->device));
    const LayerRef &L = e->layers[layer];
    const TableRef *t = which == 0 ? (L.conv ? &L.in_proj : &L.qkvg) : which == 1 ? (L.conv ? &L.out_proj : &L.o)
                        : which == 2 ? &L.gate_up : &L.down;
    if ((size_t) (t->rows) > (size_t) e->big_n * STEP_COLS) return fail(IMI_E_ARG, "table too tall for the scratch");
    MvArgs a = {};
    a.cols_d = e->cols_d; a.ncol = ncol; a.eps = e->eps; a.n_embd = e->n_embd; a.ring_layer = -1;
    a.err = e->err; a.q8_q = e->qa_q; a.q8_d = e->qa_d; a.q8_s = e->qa_s; a.out = e->big; a.out_stride = 0;
    const int epi = E_STORE;   // the output stage of the traced read: a plain store (same table bytes, same phases)
    const int g = std::max(1, std::min(e->sm_count, t->rows));
    unsigned long long *d = nullptr;
    CK(cudaMalloc(&d, (size_t) g * MV_TRACE * 8));
    CK(cudaMemsetAsync(d, 0, (size_t) g * MV_TRACE * 8, e->stream));
    a.trace = d;
    a.W = e->w + t->off; a.rows = t->rows; a.cols = t->cols; a.row_bytes = t->row_bytes;
    a.has_m = t->has_m ? 1 : 0;
    a.unit = epi == E_SILU ? 2 : 1;
    plan_stages(a, P_Q8IN, 1, g);
    cudaError_t r = launch_table(P_Q8IN, epi, a, g, e->stream, false);
    if (r == cudaSuccess) r = cudaMemcpyAsync(trace, d, (size_t) g * MV_TRACE * 8, cudaMemcpyDeviceToHost, e->stream);
    if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
    cudaFree(d);
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("trace_table: ") + cudaGetErrorString(r));
    *grid = g;
    return check_err(e);
}

namespace {
struct StateImage {
    int32_t magic, version, pos, n_attn, n_ctx, kvd, n_conv, d_conv, n_embd, n_vocab, next_pick;
};
size_t image_bytes(const imi_cuda_engine *e, int pos) {
    const size_t kvd = (size_t) e->n_head_kv * e->head_dim;
    return sizeof(StateImage) + 2 * (size_t) e->n_attn * pos * kvd * 2 + (size_t) e->n_conv * e->d_conv * e->n_embd * 4 +
           (size_t) e->n_embd * 4 + (size_t) e->n_vocab * 4;
}
}  // namespace

imi_cuda_status imi_cuda_state_save(const imi_cuda_state *s, void *buf, size_t cap, size_t *size) {
    if (!s || !size) return fail(IMI_E_ARG, "null argument");
    const imi_cuda_engine *e = s->e;
    const size_t need = image_bytes(e, s->pos);
    *size = need;
    if (!buf) return IMI_OK;
    if (cap < need) return fail(IMI_E_ARG, "buffer too small for the state image");
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->stream));
    SessDev sd;
    CK(cudaMemcpy(&sd, s->s, sizeof sd, cudaMemcpyDeviceToHost));
    if (sd.pos != s->pos)
        return fail(IMI_E_CUDA, "device position " + std::to_string(sd.pos) + " disagrees with " + std::to_string(s->pos));
    const int kvd = e->n_head_kv * e->head_dim, R = e->d_conv + 1, E = e->n_embd, pos = s->pos;
    StateImage h = { 0x53494d49, 1, pos, e->n_attn, e->n_ctx, kvd, e->n_conv, e->d_conv, E, e->n_vocab, sd.next_token };
    uint8_t *o = (uint8_t *) buf;
    memcpy(o, &h, sizeof h);
    o += sizeof h;
    // the image keeps imi's layout, [layer][position][kv head][D]; the caches are [layer][kv head][position][D]
    const int D = e->head_dim, nkv = e->n_head_kv;
    for (const __half *cache : { s->kc, s->vc })
        for (int a = 0; a < e->n_attn; a++) {
            for (int g = 0; g < nkv && pos > 0; g++)
                CK(cudaMemcpy2D(o + (size_t) g * D * 2, (size_t) kvd * 2, cache + ((size_t) a * nkv + g) * e->n_ctx * D,
                                (size_t) D * 2, (size_t) D * 2, (size_t) pos, cudaMemcpyDeviceToHost));
            o += (size_t) pos * kvd * 2;
        }
    for (int l = 0; l < e->n_conv; l++)
        for (int k = 0; k < e->d_conv; k++) {   // tap k holds position pos - d_conv + k (zero before position 0)
            const int slot = (((pos - e->d_conv + k) % R) + R) % R;
            CK(cudaMemcpy(o, s->ring + ((size_t) l * R + slot) * E, (size_t) E * 4, cudaMemcpyDeviceToHost));
            o += (size_t) E * 4;
        }
    CK(cudaMemcpy(o, s->hidden, (size_t) E * 4, cudaMemcpyDeviceToHost));
    o += (size_t) E * 4;
    CK(cudaMemcpy(o, s->logits, (size_t) e->n_vocab * 4, cudaMemcpyDeviceToHost));
    return IMI_OK;
}

imi_cuda_status imi_cuda_state_load(imi_cuda_state *s, const void *buf, size_t size) {
    if (!s || !buf || size < sizeof(StateImage)) return fail(IMI_E_ARG, "bad state image");
    imi_cuda_engine *e = s->e;
    e->gen++;
    StateImage h;
    memcpy(&h, buf, sizeof h);
    const int kvd = e->n_head_kv * e->head_dim, R = e->d_conv + 1, E = e->n_embd;
    if (h.magic != 0x53494d49 || h.version != 1 || h.n_attn != e->n_attn || h.kvd != kvd || h.n_conv != e->n_conv ||
        h.d_conv != e->d_conv || h.n_embd != E || h.n_vocab != e->n_vocab || h.pos < 0 || h.pos > e->n_ctx ||
        size < image_bytes(e, h.pos))
        return fail(IMI_E_FORMAT, "state image does not fit this engine");
    CK(cudaSetDevice(e->device));
    CK(cudaStreamSynchronize(e->stream));
    const uint8_t *i = (const uint8_t *) buf + sizeof h;
    const int D = e->head_dim, nkv = e->n_head_kv;   // image [layer][position][kv head][D] -> caches [layer][kv head][position][D]
    for (__half *cache : { s->kc, s->vc })
        for (int a = 0; a < e->n_attn; a++) {
            for (int g = 0; g < nkv && h.pos > 0; g++)
                CK(cudaMemcpy2D(cache + ((size_t) a * nkv + g) * e->n_ctx * D, (size_t) D * 2, i + (size_t) g * D * 2,
                                (size_t) kvd * 2, (size_t) D * 2, (size_t) h.pos, cudaMemcpyHostToDevice));
            i += (size_t) h.pos * kvd * 2;
        }
    CK(cudaMemset(s->ring, 0, (size_t) e->n_conv * R * E * 4));
    for (int l = 0; l < e->n_conv; l++)
        for (int k = 0; k < e->d_conv; k++) {
            const int slot = (((h.pos - e->d_conv + k) % R) + R) % R;
            CK(cudaMemcpy(s->ring + ((size_t) l * R + slot) * E, i, (size_t) E * 4, cudaMemcpyHostToDevice));
            i += (size_t) E * 4;
        }
    CK(cudaMemcpy(s->hidden, i, (size_t) E * 4, cudaMemcpyHostToDevice));
    i += (size_t) E * 4;
    CK(cudaMemcpy(s->logits, i, (size_t) e->n_vocab * 4, cudaMemcpyHostToDevice));
    SessDev sd = {};
    sd.pos = h.pos;
    sd.next_token = h.next_pick;
    CK(cudaMemcpy(s->s, &sd, sizeof sd, cudaMemcpyHostToDevice));
    s->pos = h.pos;
    return IMI_OK;
}

imi_cuda_status imi_cuda_trace_step(imi_cuda_state *s, int32_t token, int want_logits, unsigned long long *out,
                                    int max_launches, int *kinds, int *grids, int *n) {
    if (!s || !out || !kinds || !grids || !n || max_launches <= 0) return fail(IMI_E_ARG, "bad trace_step arguments");
    imi_cuda_engine *e = s->e;
    if (s->pos >= e->n_ctx) return fail(IMI_E_CTX_FULL, "context full");
    if (token < 0 || token >= e->n_vocab) return fail(IMI_E_ARG, "token out of range");
    CK(cudaSetDevice(e->device));
    imi_cuda_status st;
    if ((st = staging_wait(e)) != IMI_OK) return st;
    const size_t per = (size_t) e->sm_count * MV_TRACE;
    CK(cudaMalloc(&e->trace_buf, per * max_launches * 8));
    CK(cudaMemsetAsync(e->trace_buf, 0, per * max_launches * 8, e->stream));
    e->trace_n = 0;
    e->trace_max = max_launches;
    e->trace_kind.clear();
    e->trace_grid.clear();
    e->cols_h[0] = decode_col(s, token, false, 0, want_logits != 0);
    e->gen++;
    CK(cudaMemcpyAsync(e->cols_d, e->cols_h, sizeof(Col), cudaMemcpyHostToDevice, e->stream));
    cudaError_t r = enqueue_step(e, 1, want_logits != 0, K_DECODE);
    if (r == cudaSuccess) r = cudaMemcpyAsync(out, e->trace_buf, per * e->trace_n * 8, cudaMemcpyDeviceToHost, e->stream);
    if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
    cudaFree(e->trace_buf);
    e->trace_buf = nullptr;
    if (r != cudaSuccess) return fail(IMI_E_CUDA, std::string("trace_step: ") + cudaGetErrorString(r));
    *n = e->trace_n;
    for (int i = 0; i < e->trace_n; i++) { kinds[i] = e->trace_kind[i]; grids[i] = e->trace_grid[i]; }
    s->pos++;
    return check_err(e);
}

}  // extern "C"

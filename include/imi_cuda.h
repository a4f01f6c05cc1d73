/* imi_cuda.h - C-ABI of the B200 decode engine for imi's brain token loop (the Seoul / LFM3 hybrid backbone).
 *
 * This is the drop-in boundary for imi's brain (reference: imi/core/seoul.h, struct imi_seoul). Plain pointers and
 * sizes only; every call returns an imi_cuda_status and leaves a message for imi_cuda_error(). There is no CPU
 * fallback: without a usable CUDA device every compute call fails with IMI_E_NODEV / IMI_E_CUDA.
 *
 * Model: one engine = one GGUF model resident on one GPU (imi_seoul::load, seoul.cpp:93-186).
 * State: one conversation (attention caches, conv memory, position, latest hidden/logits) resident on the same GPU
 *        (imi_seoul_state, seoul.h:21-26). The engine itself holds no conversation; imi_seoul's "own" conversation is a
 *        state the C++ wrapper (imi_seoul_cuda.h) creates.
 * Step semantics, float order and outputs follow imi_seoul exactly; see each entry point for the reference line. */
#ifndef IMI_CUDA_H
#define IMI_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct imi_cuda_engine imi_cuda_engine;
typedef struct imi_cuda_state imi_cuda_state;

typedef enum {
    IMI_OK = 0,
    IMI_E_ARG = 1,       /* bad argument (null pointer, token out of range, n <= 0, states of another engine) */
    IMI_E_FILE = 2,      /* GGUF file missing or unreadable (imi: load() returns false, seoul.cpp:94) */
    IMI_E_FORMAT = 3,    /* a tensor is missing or has a type/shape the kernels do not read (seoul.cpp:96,162) */
    IMI_E_CTX_FULL = 4,  /* position would pass n_ctx: nothing is stepped (imi prints "context full", seoul.cpp:353) */
    IMI_E_CUDA = 5,      /* a CUDA call failed */
    IMI_E_NOMEM = 6,     /* device (or pinned host) allocation failed */
    IMI_E_TIMEOUT = 7,   /* a bounded device-side wait gave up (the kernel returned; the context stays usable) */
    IMI_E_NODEV = 8      /* no CUDA device with the requested index */
} imi_cuda_status;

typedef struct {
    int n_embd, n_vocab, n_ctx, n_layer, n_attn, n_head, n_head_kv, head_dim, n_ff, d_conv, n_swa, max_batch;
    size_t weight_bytes;   /* bytes of layer tables + word table + small parameters on the device */
    size_t state_bytes;    /* device bytes of one conversation state */
    int cols_per_read;     /* conversations (or prefill positions) one read of the tables serves at most: 8 on the
                              small-batch kernel; up to 256 (max(max_batch, 128)) on the tensor cores, which every
                              Q4_0 model uses above 8 */
} imi_cuda_info;

/* Last error message of this thread (never NULL). */
const char *imi_cuda_error(void);

/* Load a GGUF model onto CUDA device `device` (replaces imi_seoul::load(path, threads, ctx_len), seoul.cpp:93).
 * n_ctx: positions per conversation; max_batch: most conversations stepped together by imi_cuda_step_multi.
 * An engine and its states are used by one host thread at a time: they share the engine's stream, its staging
 * buffers and its read-back buffer.
 * Device memory budget: when the environment variable IMI_CUDA_MAX_DEVICE_BYTES is set (bytes), the engine and all
 * its states together allocate at most that much; a load or a new state beyond it fails with IMI_E_NOMEM (for a GPU
 * shared with other work). */
imi_cuda_status imi_cuda_load(const char *gguf_path, int device, int n_ctx, int max_batch, imi_cuda_engine **out);
void imi_cuda_free(imi_cuda_engine *e);                                     /* ~imi_seoul, seoul.cpp:687-689 */
imi_cuda_status imi_cuda_get_info(const imi_cuda_engine *e, imi_cuda_info *out);

/* A fresh conversation sized like the engine's (imi_seoul::new_state, seoul.cpp:193-201): position 0, zero conv memory. */
imi_cuda_status imi_cuda_state_new(imi_cuda_engine *e, imi_cuda_state **out);
void imi_cuda_state_free(imi_cuda_state *s);
/* Position 0 and zero conv memory (imi_seoul::reset, seoul.cpp:188-191). */
imi_cuda_status imi_cuda_state_reset(imi_cuda_state *s);
int imi_cuda_state_pos(const imi_cuda_state *s);                            /* imi_seoul::pos */

/* One position (imi_seoul::step, seoul.cpp:352-357): token >= 0 reads the word table row, else embd[n_embd] is the
 * input vector. want_logits adds the word scores (and the greedy pick). IMI_E_CTX_FULL if pos >= n_ctx. */
imi_cuda_status imi_cuda_step(imi_cuda_state *s, int32_t token, const float *embd, int want_logits);

/* Two conversations one position each, every table read once for both (imi_seoul::step2, seoul.cpp:208-220).
 * Each gets exactly the numbers its own imi_cuda_step would give. */
imi_cuda_status imi_cuda_step2(imi_cuda_state *a, int32_t token_a, const float *embd_a, int logits_a,
                               imi_cuda_state *b, int32_t token_b, const float *embd_b, int logits_b);

/* n distinct conversations of one engine, one position each, one table read for all (n <= max_batch): the
 * generalisation of step2 to the multi-session case. tokens[i] (or embd + i*n_embd when tokens is NULL or
 * tokens[i] < 0), want_logits[i] (NULL = all). */
imi_cuda_status imi_cuda_step_multi(imi_cuda_state *const *s, int n, const int32_t *tokens, const float *embd,
                                    const int *want_logits);

/* Read n positions of one conversation (imi_seoul::step_batch, seoul.cpp:490-517): tokens[n], or embd[n][n_embd].
 * hidden and (if want_logits) logits are the last position's; hidden_all[n][n_embd] (host, optional) receives every
 * position's hidden state. Positions are read in chunks; IMI_E_CTX_FULL (nothing more stepped) when a chunk would
 * pass n_ctx, as seoul.cpp:498. */
imi_cuda_status imi_cuda_step_batch(imi_cuda_state *s, const int32_t *tokens, const float *embd, int n,
                                    int want_logits, float *hidden_all);

/* Greedy decode on the device: `steps` positions for each of n conversations (n <= max(max_batch, 8)), each step's
 * input being the previous step's pick (the caller loop of imi/core/hear.cpp:65-72 without a stop word). The first
 * step reads tokens[i] (or, when tokens is NULL, each conversation's last pick). ids[steps][n] receives every pick.
 * Logits of the last step stay readable. */
imi_cuda_status imi_cuda_greedy(imi_cuda_state *const *s, int n, const int32_t *tokens, int steps, int32_t *ids);

/* Checkpoint / resume of one conversation (the content of imi_seoul_state, seoul.h:21-26) as a host byte image:
 *   int32 magic 0x53494d49 ("IMIS"), version 1, pos, n_attn, n_ctx, kv_dim, n_conv, d_conv, n_embd, n_vocab, next_pick;
 *   K cache [n_attn][pos][kv_dim] fp16, V cache likewise (positions 0..pos-1 only);
 *   conv memory [n_conv][d_conv][n_embd] fp32, oldest first (imi's layout, seoul.h:47);
 *   hidden [n_embd] fp32, logits [n_vocab] fp32.
 * save: buf NULL -> *size receives the bytes needed; else the image is written (cap >= that size).
 * load: into a state of an engine with the same shape and an n_ctx >= the image's pos. */
imi_cuda_status imi_cuda_state_save(const imi_cuda_state *s, void *buf, size_t cap, size_t *size);
imi_cuda_status imi_cuda_state_load(imi_cuda_state *s, const void *buf, size_t size);

/* The latest outputs of a conversation (imi_seoul::hidden / ::logits, seoul.h:51): host copies. */
imi_cuda_status imi_cuda_get_hidden(const imi_cuda_state *s, float *out /* n_embd */);
imi_cuda_status imi_cuda_get_logits(const imi_cuda_state *s, float *out /* n_vocab */);
/* The greedy pick of the latest step with logits: first maximum, lowest id on ties (imi/core/hear.cpp:67-68). */
imi_cuda_status imi_cuda_get_argmax(const imi_cuda_state *s, int32_t *id, float *value);

/* ---- the model file's keys and tensor headers (host only; imi_file, imi/model.h:17-36) ----
 * The GGUF file memory-mapped by the library's own reader, for callers that read keys beside the brain (the
 * tokenizer reads the word list from the same file: imi_words::load(brain.f), flow.cpp:49). Value types are GGUF's
 * (4 u32, 5 i32, 6 f32, 7 bool, 8 string, 9 array, 10 u64, ...). Pointers stay valid until imi_cuda_file_close. */
typedef struct imi_cuda_file imi_cuda_file;
imi_cuda_status imi_cuda_file_open(const char *path, imi_cuda_file **out);
void imi_cuda_file_close(imi_cuda_file *f);
int64_t imi_cuda_file_find_key(const imi_cuda_file *f, const char *key);              /* -1 when absent */
int64_t imi_cuda_file_n_keys(const imi_cuda_file *f);
const char *imi_cuda_file_key_name(const imi_cuda_file *f, int64_t k);
int imi_cuda_file_key_type(const imi_cuda_file *f, int64_t k);
const void *imi_cuda_file_key_data(const imi_cuda_file *f, int64_t k);                  /* a scalar's bytes */
const char *imi_cuda_file_key_str(const imi_cuda_file *f, int64_t k);                   /* a string (copy, 0-ended) */
int imi_cuda_file_arr_type(const imi_cuda_file *f, int64_t k);
uint64_t imi_cuda_file_arr_n(const imi_cuda_file *f, int64_t k);
const void *imi_cuda_file_arr_data(const imi_cuda_file *f, int64_t k);                  /* fixed-size elements */
const char *imi_cuda_file_arr_str(const imi_cuda_file *f, int64_t k, uint64_t i);       /* string element i */
/* a tensor's header: 0 and its GGML type, shape (fastest first), bytes in the map; -1 when absent */
int imi_cuda_file_tensor(const imi_cuda_file *f, const char *name, int *type, int64_t ne[4], const void **data,
                         size_t *nbytes);

/* ---- measurement ---- */

/* The CUDA stream (cudaStream_t) every launch of this engine goes to, for callers that time on the device. */
void *imi_cuda_stream(const imi_cuda_engine *e);
/* Milliseconds on the device of the engine's last step (the last read of its tables with everything around it:
 * every launch of one imi_cuda_step / step2 / step_multi group / step_batch chunk), waiting for it to finish; 0 if
 * none ran. The C++ wrapper adds it to imi_seoul::t_tables after each step. */
float imi_cuda_last_step_ms(const imi_cuda_engine *e);
/* Kernel launches of one step of n conversations (with or without word scores). */
int imi_cuda_launches_per_step(const imi_cuda_engine *e, int n, int want_logits);
/* Kernel launches of one imi_cuda_step_batch of n positions (with or without the last position's word scores). */
int imi_cuda_launches_per_batch(const imi_cuda_engine *e, int n, int want_logits);
/* Every layer table read back to back with ncol (1..cols_per_read) inputs riding each read, as imi_seoul::bench_tables
 * (seoul.cpp:657-685): *ms = mean milliseconds per pass over `reps` passes (after one untimed pass), *bytes = table
 * bytes read per pass. */
imi_cuda_status imi_cuda_bench_tables(imi_cuda_engine *e, int ncol, int reps, float *ms, size_t *bytes);

/* Diagnostics: read table `which` (0 in_proj/qkvg, 1 out_proj/o, 2 gate_up, 3 down) of layer `layer`
 * once, alone, with ncol inputs, and return per-CTA phase timestamps in ns: trace[cta][16] (0 start, 1 after the
 * dependency wait, 2 after input preparation, 3+s after stage s's integer phase, 14 end of the float chains).
 * *grid receives the number of CTAs; trace must hold 148*16 values on a B200. */
imi_cuda_status imi_cuda_trace_table(imi_cuda_engine *e, int layer, int which, int ncol, unsigned long long *trace,
                                     int *grid);

/* Diagnostics: one decode step of `s` (token given) launched directly (not from a graph) with every launch writing
 * per-CTA phase timestamps (ns): out[launch][n_sm][16] as in imi_cuda_trace_table (final norm: 0 start, 1 after the
 * dependency wait, 14 end; attention at head_dim 64 adds 2 query and this position's K/V made, 3 scores, 4
 * probabilities, 5 P.V done, 6 the first K/V copies issued, 7 / 8 the first / last K tile landed, 9 / 10 the first /
 * last V tile landed). kinds[launch]: 10*input+output kind of a table read, 100 attention, 101 final norm;
 * grids[launch]: CTAs. *n receives the number of launches (at most max_launches). */
imi_cuda_status imi_cuda_trace_step(imi_cuda_state *s, int32_t token, int want_logits, unsigned long long *out,
                                    int max_launches, int *kinds, int *grids, int *n);

/* Diagnostics: the failure path of the engine's bounded device waits (every wait on a weight stage gives up after
 * about one second and reports IMI_E_TIMEOUT instead of hanging). One CTA waits on an mbarrier that nothing completes,
 * with a limit of limit_ms milliseconds at the device's clock; the wait gives up, the kernel sets the error flag and
 * returns. Returns IMI_E_TIMEOUT when the wait gave up as designed (the context stays usable), IMI_OK never. */
imi_cuda_status imi_cuda_check_wait_timeout(int device, double limit_ms);

/* ---- kernel level (known-answer tests and the isolated table sweep) ---- */

/* Cut x[n] to 8-bit per 32 values on the device (imi_q8::from, tables.cpp:100-109 with imi_cut32, vec.h:47-77):
 * q[n] int8 codes, d[n/32] scales, s[n/32] = d * sum(q). Host pointers. */
imi_cuda_status imi_cuda_q8_cut(int device, const float *x, int n, int8_t *q, float *d, float *s);

/* Word scores of a Q6_K table (the product's own word-table format: rows of 210-byte blocks per 256 values) for one
 * float input x[cols], on the device: the input cut per 256 values as imi_q8k::from (tables.cpp:200-213), then every
 * row as imi_q6k_row (tables.cpp:235-278, the AVX2 order) -> out[rows]. The cut can be returned too (xq[cols],
 * xd[cols/256], bsums[cols/16]; each may be NULL). cols a multiple of 256, at most 32768; host pointers. The kernel
 * level of the Q6_K word table, which the engine also reads inside its steps when a file carries one. */
imi_cuda_status imi_cuda_q6k_scores(int device, const uint8_t *q6k, int rows, int cols, const float *x, float *out,
                                    int8_t *xq, float *xd, int16_t *bsums);

/* A Q4_0 table (GGUF rows of 18-byte blocks, rows x cols) times ncol 8-bit inputs (xq[ncol][cols], xd/xs[ncol][cols/32])
 * on the device with imi's 4-bit kernel semantics (imi_q4_group / imi_q4_group2 / imi_q4_group_batch,
 * tables.cpp:127-177,419-477): out[ncol][rows]. Host pointers; block_dots (optional, ncol == 1) receives the integer
 * dot of every (row, 32-block) pair [rows][cols/32]. */
imi_cuda_status imi_cuda_q4_matvec(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq,
                                   const float *xd, const float *xs, int ncol, float *out, int32_t *block_dots);

/* The same table read for many inputs on the tensor cores (the batched read of imi_q8b + imi_q4_group_batch,
 * tables.cpp:405-477): ncol 1..256 inputs, each block's integer dot by a tcgen05 MMA (8-bit codes, int32, exact), imi's float
 * chains per (row, input) in block order; results as imi_cuda_q4_matvec gives them. Host pointers. */
imi_cuda_status imi_cuda_q4_matmul(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq,
                                   const float *xd, const float *xs, int ncol, float *out);

/* Diagnostics: imi_cuda_q4_matmul with CTA 0's timeline of the tensor-core read in ns, trace[9][64]: 0 stage copies
 * issued, 1 (unused, 0), 2 stage done by the last epilogue warp, 3 block's MMA issued, 4 block's dots awaited by the
 * epilogue, 5 block's chains done, 6 block's dots in registers, 7 stage's copies seen by the MMA warp, 8 stage's TMEM
 * slot free for the MMA warp (stages and blocks counted from the CTA's first unit); trace holds 9 * 64 values. */
imi_cuda_status imi_cuda_trace_tc(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq, const float *xd,
                                  const float *xs, int ncol, float *out, unsigned long long *trace);

/* The isolated table read timed on the device (the configs[4] sweep; imi/kernels/q4x2_bench.cpp's measurement): a
 * rows x cols Q4_0 table (random codes and scales, the engine's row layout) times ncol 8-bit inputs, `reps` reads after
 * one untimed pass, CUDA events on one stream. The table is replicated in device memory until the copies pass 256 MB
 * and the reads rotate through all of them (at least `reps` reads, at least one per copy), so every read comes from
 * HBM (L2 holds 126 MB). *ms = mean milliseconds per
 * read of all ncol inputs; *bytes = algorithmic bytes per read: the table once, the inputs' codes and scales, the
 * outputs. ncol 1..256; cols a multiple of 256. */
imi_cuda_status imi_cuda_bench_matvec(int device, int rows, int cols, int ncol, int reps, float *ms, size_t *bytes);

/* ---- without allocation ---- */

/* No counterpart in the reference (imi's own path has no device memory): imi_cuda_q4_matvec on device buffers that
 * allocates nothing. It exists for callers that must not allocate device memory while they run: cudaFree waits for
 * every stream of the device (a caller sharing the GPU with a running decode loop would stall it), a cudaMalloc may
 * fail once a memory pool or another framework's caching allocator holds the free memory, and some callers run where
 * allocating is not allowed at all (a real-time audio callback, an allocator hook).
 *
 * q4: the table as GGUF Q4_0 rows (rows x cols, 18-byte blocks); xq[ncol][cols] (16-byte aligned), xd, xs[ncol][cols/32]
 * and out[ncol][rows]: all device memory of `device`; results as imi_cuda_q4_matvec gives them. stream: a cudaStream_t
 * of that device (NULL: the default stream); the call returns once its work on that stream is done.
 * Scratch: one static device array of this library per device (IMI_CUDA_STATIC_TABLE_BYTES for the table in the
 * kernels' row layout, plus 4 KiB). The call clears what must start at zero (the column descriptors and the error
 * flag) on the stream itself, so nothing needs to be zero beforehand. A table above IMI_CUDA_STATIC_TABLE_BYTES
 * (rows * cols / 32 * 18 bytes) is refused with IMI_E_ARG.
 * The first call on a device looks the scratch address up (cudaGetSymbolAddress, with that device current) and sets
 * the kernels' shared-memory limits; both are kept for the life of the process, which assumes the device's primary
 * context is not reset (cudaDeviceReset) in between. The scratch is shared: two calls on the same device that overlap in time (from two host threads,
 * or on two streams) race on it and corrupt each other's results; callers serialise them. */
#define IMI_CUDA_STATIC_TABLE_BYTES 16777216u
imi_cuda_status imi_cuda_q4_matvec_static(int device, const uint8_t *q4, int rows, int cols, const int8_t *xq,
                                          const float *xd, const float *xs, int ncol, float *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif

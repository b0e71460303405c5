/* d3s.h - C ABI of the B200 token sampler (temperature -> top-k -> top-p ->
 * exponential-race draw) that replaces drama3-mlx's src/sampling.c.
 *
 * Paths in citations are relative to the drama3-mlx project root.
 *
 * Semantics (identical to the CPU oracle in oracle/, bit for bit):
 *   k = min(top_k, V); T = max(temperature, 1e-5); q = logits / T;
 *   lse = max(q) + log(sum exp(q - max q)) over the whole row;
 *   top k by (q desc, id asc); cum_r = inclusive float sum of exp(q_r - lse);
 *   rank r > 0 is dropped when cum_r > top_p; survivors are re-softmaxed;
 *   the winner is the first rank with the largest p_r / -log(1 - u_r).
 *   u [N, k] comes from MLX's threefry key sequence, as mlx_random_uniform
 *   would draw it (src/sampling.c:179-209, src/mlxu.c:769-774).
 *
 * Ids are positions into the last axis (int32), as the reference returns them.
 * Every entry point returns D3S_OK (0) or a negative D3S_ERR_* code and never
 * exits the process (the reference calls die() -> exit(1), src/mlxu.c:28-36);
 * d3s_last_error() holds the message for the calling thread.
 * Device pointers are CUDA device memory of the context's device; `stream` is
 * a cudaStream_t (NULL = the legacy default stream). Calls on device pointers
 * are asynchronous on `stream`.
 */
#ifndef D3S_H
#define D3S_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define D3S_VERSION 1

#if defined(__GNUC__)
#define D3S_API __attribute__((visibility("default")))
#else
#define D3S_API
#endif

/* status codes */
#define D3S_OK 0
#define D3S_ERR_ARG -1          /* bad argument (null pointer, size, dtype, top_k < 1, ...) */
#define D3S_ERR_CUDA -2         /* a CUDA runtime call failed */
#define D3S_ERR_NONFINITE -3    /* a row's scaled logits were NaN / +inf / all -inf (sync calls) */
#define D3S_ERR_UNSUPPORTED -4  /* a size beyond the documented limits */
#define D3S_ERR_NOMEM -5        /* device or host allocation failed */

/* logits element types */
#define D3S_F32 0
#define D3S_BF16 1

/* per-row status values (d3s_request.status) */
#define D3S_ROW_OK 0
#define D3S_ROW_NONFINITE 1
#define D3S_ROW_BADPARAM 2

/* noise sources (d3s_request.noise) */
#define D3S_NOISE_KEY 0    /* one key for the batch: u = uniform(key, [N, k]) */
#define D3S_NOISE_SEEDS 1  /* row r draws as d3_sample(row r, seeds[r]) would */
#define D3S_NOISE_GIVEN 2  /* u given: sample_with_noise */
#define D3S_NOISE_KEYS 3   /* row r draws u [1, k] from its own subkey keys[r * ld_keys] */

/* limits */
#define D3S_MAX_V 131072      /* the full-row sum's fixed point holds V <= 2^17 */
#define D3S_MAX_K 16384       /* k = min(top_k, V) */

/* The RNG state: one threefry-2x32 key, a plain serialisable pair of words.
 * This is MLX's random key (mlx/random.cpp): key(seed) = {seed >> 32, seed}. */
typedef struct {
  uint32_t k[2];
} d3s_key;

typedef struct d3s_ctx d3s_ctx;

D3S_API int d3s_version(void);
D3S_API const char *d3s_last_error(void);

/* ---- keys (host-side; no device work) ---- */

/* random::key(seed). */
D3S_API int d3s_key_from_seed(uint64_t seed, d3s_key *out);
/* random::split(key) -> (k0, k1). */
D3S_API int d3s_key_split(const d3s_key *key, d3s_key *k0, d3s_key *k1);
/* m_seed (src/mlxu.c:769) -> mlx_random_seed: state = key(seed). state NULL
 * seeds the library's global key, as MLX's global key sequence. */
D3S_API int d3s_seed(d3s_key *state, uint64_t seed);
/* The global key sequence's next(): (state, sub) = split(state); NULL = global. */
D3S_API int d3s_next_key(d3s_key *state, d3s_key *sub);

/* ---- context ---- */

/* A context owns the device id, the kernels' device scratch (per-row records
 * passed between the streaming and the selection kernel, the hand-off list of
 * rows for the wide path) and staging buffers for the host-pointer entry points. */
D3S_API int d3s_ctx_create(int device, d3s_ctx **out);
D3S_API void d3s_ctx_destroy(d3s_ctx *ctx);
/* Pre-size the context's device scratch (about 2.1 KB of row records plus a
 * 4-byte hand-off slot per row) for requests of up to max_rows rows.
 * d3s_sample grows it on demand with cudaMalloc, which a CUDA graph capture
 * cannot contain: reserve before capturing. */
D3S_API int d3s_ctx_reserve(d3s_ctx *ctx, int64_t max_rows);

/* ---- the reference's internal API (src/model.h:169-176) ---- */

/* sample_noise (src/sampling.c:179-192): u_dev [rows, k], k = min(top_k, V),
 * drawn from state (NULL = global key), which advances by one split. */
D3S_API int d3s_sample_noise(d3s_ctx *ctx, d3s_key *state, int rows, int V, int top_k, float *u_dev,
                     void *stream);

/* sample_with_noise (src/sampling.c:194-203): logits_dev [N, ld] (dtype),
 * u_dev [N, ld_u] of which the first k columns are used; ids_dev [N]. */
D3S_API int d3s_sample_with_noise(d3s_ctx *ctx, const void *logits_dev, int dtype, int N, int V,
                          int64_t ld, const float *u_dev, int k, int64_t ld_u, float temperature,
                          float top_p, int32_t *ids_dev, void *stream);

/* sample_top_k_top_p (src/sampling.c:205-209): one split of state (NULL =
 * global key), u = uniform(sub, [N, k]) generated inside the kernel. */
D3S_API int d3s_sample_top_k_top_p(d3s_ctx *ctx, const void *logits_dev, int dtype, int N, int V,
                           int64_t ld, float temperature, int top_k, float top_p,
                           d3s_key *state, int32_t *ids_dev, void *stream);

/* ---- batched engine (all of the above lower to this) ---- */

typedef struct {
  const void *logits;         /* [N, ld] device */
  int32_t dtype;              /* D3S_F32 / D3S_BF16 */
  int32_t N, V;
  int64_t ld;                 /* elements between rows, >= V */
  float temperature, top_p;   /* used when the matching *_rows pointer is NULL */
  int32_t top_k;
  const float *temperature_rows; /* [N] device, optional */
  const float *top_p_rows;       /* [N] device, optional */
  const int32_t *top_k_rows;     /* [N] device, optional (not with D3S_NOISE_KEY) */
  int32_t noise;              /* D3S_NOISE_* */
  d3s_key key;                /* D3S_NOISE_KEY: the subkey that draws u [N, k] */
  const uint64_t *seeds;      /* D3S_NOISE_SEEDS: [N] device */
  const float *u;             /* D3S_NOISE_GIVEN: [N, ld_u] device */
  int64_t ld_u;
  int32_t *ids;               /* [N] device, required; -1 for a flagged row */
  int32_t *status;            /* [N] device, optional: D3S_ROW_* */
  int32_t *kept;              /* [N] device, optional: survivors of the top-p cut */
  float *probs;               /* [N, ld_out] device, optional: race probabilities by rank */
  int32_t *topk_ids;          /* [N, ld_out] device, optional: ids by rank */
  int64_t ld_out;
  const d3s_key *keys;        /* D3S_NOISE_KEYS: [N * ld_keys] device, 8-byte aligned */
  int64_t ld_keys;            /* keys between rows (0 means 1) */
  int32_t *finite;            /* [N] device, optional: 1 when every logit of the row is
                                 finite (the guard of src/generate.c:92), else 0 */
} d3s_request;

D3S_API int d3s_sample(d3s_ctx *ctx, const d3s_request *req, void *stream);

/* Synchronise the context's device and report a failure the kernels recorded
 * (a bounded wait that gave up); clears it. D3S_OK when none. */
D3S_API int d3s_ctx_check(d3s_ctx *ctx);

/* Test hooks (no counterpart in the reference): y_dev = f(x_dev) with the
 * kernels' own arithmetic; op 0 = exp, 1 = log, 2 = the full-row-sum term
 * exp(max(x, -86)), 3 = x / param by the per-row reciprocal path, 4 = the
 * special-function unit's 2^x that the approximate full-row sum uses. */
D3S_API int d3s_debug_math(d3s_ctx *ctx, int op, const float *x_dev, float *y_dev, int64_t n,
                           float param, void *stream);
/* Test hook (no counterpart in the reference): which kernel samples the
 * batches above the small-batch path (N > 512), process-wide: 0 = the usual
 * choice, 1 = the four-warp streaming stats kernel + the select kernel, 3 =
 * the row-warp kernel (one warp per row), 4 = the one-warp streaming stats
 * kernel + the select kernel. A path that cannot take the request
 * falls back to the usual one. Results are identical on every path; tests use
 * it to check each of them. */
D3S_API int d3s_debug_force_path(int path);
/* Counts float bit patterns x in [lo, hi) (step `step`) with |x| in
 * [2^-100, 2^60], the reciprocal path's exact range, whose quotient x / T differs from the IEEE quotient, for each of
 * T_dev[nT]; adds to *bad_dev (device), last failing (x, T) in example_dev[2]. */
D3S_API int d3s_debug_div_check(d3s_ctx *ctx, const float *T_dev, int nT, uint64_t lo,
                                uint64_t hi, uint64_t step, unsigned long long *bad_dev,
                                float *example_dev, void *stream);

/* ---- batched sampling without allocation ---- */

/* Rows a d3s_sample_rows_static call may hold (about 8.6 MB of device scratch
 * that every GPU loading this library keeps until the process exits). */
#define D3S_STATIC_MAX_ROWS 4096

/* No counterpart in the reference. For callers that cannot allocate device
 * memory while they sample: a serving engine that budgets every device byte
 * up front and forbids allocation once it serves, or a real-time audio thread
 * that cannot wait on cudaMalloc's implicit device synchronisation.
 * Same results as d3s_sample with D3S_NOISE_SEEDS and per-row temperature,
 * top_p and top_k (all device arrays of N, as are the logits and ids); no
 * context is needed. Its scratch is one fixed array in the library shared by
 * every call: N above D3S_STATIC_MAX_ROWS is rejected (D3S_ERR_UNSUPPORTED),
 * and two calls whose kernels overlap on the GPU (different streams without an
 * ordering between them) race on it. The first call on each device looks up
 * the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture. Nothing is allocated, on any call.
 * A kernel that gives up a bounded wait (a row copy that never completed)
 * records it in the array's error word and leaves rows' ids unwritten; the
 * word stays set across calls until d3s_static_check reads it. */
D3S_API int d3s_sample_rows_static(const void *logits_dev, int dtype, int N, int V, int64_t ld,
                                   const float *temperature_dev, const float *top_p_dev,
                                   const int32_t *top_k_dev, const uint64_t *seeds_dev,
                                   int32_t *ids_dev, void *stream);

/* No counterpart in the reference. Waits for the work queued on `stream`,
 * then reads and clears the error word of d3s_sample_rows_static's scratch on
 * the current device: D3S_OK when no call since the last check gave up a
 * wait, else D3S_ERR_CUDA (the ids of the calls since the last check are
 * undefined). Allocates nothing. */
D3S_API int d3s_static_check(void *stream);

/* Test hook (no counterpart in the reference): stores `value` in the error
 * word that d3s_static_check reads, on the current device, ordered on
 * `stream`, so a test can see a recorded failure reported without stalling a
 * copy. */
D3S_API int d3s_static_debug_set_error(int32_t value, void *stream);

/* ---- rows sharded over the GPUs of a node: the gather of ids to rank 0 ---- */

/* No single counterpart in the reference (it samples on one device); this is
 * the id gather that sharding the rows over G GPUs needs, one process per GPU.
 * Rank r samples rows [r N / G, (r + 1) N / G) of an N-row batch and its
 * sampler writes their ids straight into rank 0's result (a CUDA IPC mapping
 * of rank 0's buffer, plain stores over NVLink), so no collective runs after
 * the sampler; a counter in rank 0's memory, raised by each rank after its
 * sampler (release at system scope) and waited on by rank 0 (acquire, with a
 * 5 s limit that sets the gather's error word instead of hanging), marks the
 * step complete. The result has `slots` (>= 2) slots, step s in slot
 * s mod slots: a rank writes step s only after rank 0 released step
 * s - slots, so the ranks may run up to slots - 1 steps ahead of rank 0's
 * gather.
 * Use: every rank d3s_gather_create; rank 0 d3s_gather_export, the 64-byte
 * handle passed to the other ranks by the caller's own channel, which call
 * d3s_gather_attach. Then per step s = 0, 1, 2, ... on every rank:
 * d3s_gather_begin on the sampler's stream (it waits there until the slot is
 * free and gives the ids pointer for this rank's rows), the sampler with
 * req.ids = that pointer, then d3s_gather_end on a stream ordered after the
 * sampler (the same one, or a side stream that waited for an event of it, so
 * the signal / wait overlaps the next step's sampling); rank 0 reads the N ids
 * of step s at the result pointer d3s_gather_end gave, after it on that
 * stream, then calls d3s_gather_release there. Rank 0's own sampler does not
 * wait for a free slot: its release of step s - slots must come before its
 * sampler of step s in stream order. */
#define D3S_GATHER_HANDLE_BYTES 64
typedef struct d3s_gather d3s_gather;
D3S_API int d3s_gather_create(int device, int world, int rank, int64_t rows, int slots,
                              d3s_gather **out);
D3S_API int d3s_gather_export(d3s_gather *g, void *handle);
D3S_API int d3s_gather_attach(d3s_gather *g, const void *handle);
D3S_API int d3s_gather_begin(d3s_gather *g, int64_t step, int32_t **ids_dev, void *stream);
D3S_API int d3s_gather_end(d3s_gather *g, int64_t step, int32_t **result_dev, void *stream);
D3S_API int d3s_gather_release(d3s_gather *g, int64_t step, void *stream);
/* A start line on `stream` (no counterpart in the reference: it lines up the
 * ranks' GPUs, for timing): every rank's stream stops here until every rank's
 * stream has reached its `line`-th start line (line = 1, 2, ... on every rank),
 * so work queued after it starts on all GPUs together, whenever each host
 * queued it. The wait gives up after 5 s and records it for d3s_gather_check. */
D3S_API int d3s_gather_line_up(d3s_gather *g, int64_t line, void *stream);
/* Rank 0: copy the N ids of `step` (after d3s_gather_end) to dst_dev, on `stream`. */
D3S_API int d3s_gather_copy_result(d3s_gather *g, int64_t step, int32_t *dst_dev, void *stream);
/* Waits for `stream`; D3S_ERR_CUDA (and clears it) when a wait of this rank
 * gave up since the last check. */
D3S_API int d3s_gather_check(d3s_gather *g, void *stream);
D3S_API void d3s_gather_destroy(d3s_gather *g);

/* ---- one decode frame: tower_decode_step's draws (src/tower.c:405-452) ---- */

/* Advance S streams' key states (device [S], 8-byte aligned) by n splits each,
 * as n calls of the key sequence's next(), writing the subkeys in draw order
 * to sub_dev[s * ld_sub + i]. A frame of tower_decode_step takes
 * n = 2 + (n_codebooks - 1): main, retry, then one per codebook head
 * (src/tower.c:417-424). */
D3S_API int d3s_keys_next(d3s_ctx *ctx, d3s_key *state_dev, int S, int n, d3s_key *sub_dev,
                          int64_t ld_sub, void *stream);

#define D3S_RAS_WINDOW 16      /* main tokens a frame is checked against (src/generate.h:11) */
#define D3S_FRAME_EOS 1        /* flags: the frame's main token is eos_id */
#define D3S_FRAME_NONFINITE 2  /* the logits row holds NaN or +-inf (src/generate.c:92) */
#define D3S_FRAME_RETRY 4      /* the RAS retry token replaced a repeated semantic token */

typedef struct {
  const void *logits;          /* [S, ld] device: backbone audio logits, index 0 = eos,
                                  i >= 1 = semantic_start + i - 1 */
  int32_t dtype, S, V;
  int64_t ld;
  float temperature, top_p;    /* SamplingParams (src/model.h:146-150) of the main draw */
  int32_t top_k;
  const d3s_key *keys;         /* device, 8-byte aligned: stream s's frame subkeys at
                                  keys[s * ld_keys + i], i = 0 main, 1 retry */
  int64_t ld_keys;
  int32_t *history;            /* [S, D3S_RAS_WINDOW] device: last main tokens, oldest first */
  int32_t *hist_len;           /* [S] device: valid history entries per stream */
  int32_t semantic_start, code_vocab, eos_id;  /* model config (src/model.h:27-29) */
  int32_t update_history;      /* 1: append each main token to its window (src/generate.c:97-100) */
  int32_t *main_tok;           /* [S] device: codes[0], -1 when a draw was flagged */
  int32_t *c0;                 /* [S] device: codes[1] = clip(main - semantic_start, 0, code_vocab - 1) */
  int32_t *flags;              /* [S] device, optional: D3S_FRAME_* bits */
} d3s_frame_request;

/* The main and the retry draw of S streams from one pass of kernels (rows s
 * and S + s of one batch read logits row s), then candidate_token, the
 * repetition check, c0 and the flags (src/tower.c:425-437). The codebook
 * heads of the frame are plain d3s_sample calls with D3S_NOISE_KEYS and
 * keys = sub + 2 + j, ld_keys = n. */
D3S_API int d3s_frame_main(d3s_ctx *ctx, const d3s_frame_request *req, void *stream);

/* Host: the codes of a take as a .npy file, as npy_write_codes writes them
 * (src/npy.c:98-129, src/generate.c:162-168). frames is [n_frames, width]
 * int32 host memory, one sampled frame row per decode step (column 0 the main
 * token, columns 1..n_codebooks the codes: c0 then the heads); the file holds
 * codes[k][t] = frames[t][1 + k] as little-endian int64, shape
 * (n_codebooks, n_frames). */
D3S_API int d3s_codes_write_npy(const char *path, const int32_t *frames, int n_frames, int width,
                                int n_codebooks);

/* ---- the lm_head projection in front of the sampler ---- */

/* backbone_audio_logits -> m_linear (src/backbone.c:1213, src/mlxu.c:442-496):
 * logits_dev[b, v] = bf16(sum_d h_dev[b, d] * W_dev[v, d]) with fp32
 * accumulation and a round-to-nearest bf16 result, as the reference's GEMV
 * writes bf16 logits (src/mlxu.c:397). h [B, D], W [V, D] (the restricted
 * lm_head_audio [4097, 2048], src/model.h:71) and logits [B, ld_logits] are
 * bf16 device arrays with 16-byte aligned rows (D, ld_h, ld_w multiples of 8).
 * B <= 8 runs a CUDA-core GEMV; larger B a tcgen05 tensor-core GEMM. The sum
 * order differs from MLX's, so logits can differ from the reference's by one
 * bf16 rounding step where the fp32 sum lies next to a rounding boundary. */
D3S_API int d3s_lmhead(d3s_ctx *ctx, const void *h_dev, int64_t ld_h, const void *W_dev,
                       int64_t ld_w, int B, int V, int D, void *logits_dev, int64_t ld_logits,
                       void *stream);

/* The fused prologue: d3s_lmhead into req->logits (bf16, [req->N = B,
 * req->ld], V = req->V), then d3s_sample(req) on the same stream. */
D3S_API int d3s_lmhead_sample(d3s_ctx *ctx, const void *h_dev, int64_t ld_h, const void *W_dev,
                              int64_t ld_w, int D, const d3s_request *req, void *stream);

/* ---- the reference's test C-ABI (src/testapi.c:155-166) ---- */

/* Host logits [N, V] f32 -> host ids [N]: seeds the global key with `seed`,
 * then sample_top_k_top_p. Synchronous. A failure writes -1 ids and sets
 * d3s_last_error(); d3s_last_status() returns the code of the last d3_sample. */
D3S_API void d3_sample(const float *logits, int N, int V, float temperature, int top_k, float top_p,
               unsigned long long seed, int *out);
D3S_API int d3s_last_status(void);

#ifdef __cplusplus
}
#endif

#endif

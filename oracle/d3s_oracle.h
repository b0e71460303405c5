/* d3s_oracle.h - CPU restatement of drama3-mlx's token sampler.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA sampler in
 * drama3-mlx_b200/csrc and the timed CPU baseline of bench.py. Nothing on the
 * product path links, loads or calls it.
 *
 * What it restates (paths relative to the drama3-mlx project root):
 *   - src/sampling.c:22-49   sample_fn: temperature divide, top-k, full-row
 *                            log-sum-exp, inclusive cumsum, top-p drop rule,
 *                            masked softmax, exponential-race argmax.
 *   - src/sampling.c:53-140  drama3_sample (Metal): its top-k selection order
 *                            (per-simdgroup argmax rounds + 32-way merge) and its
 *                            first-strictly-greater race loop.
 *   - src/sampling.c:179-209 sample_noise / sample_with_noise /
 *                            sample_top_k_top_p: k = min(top_k, V), the
 *                            MIN_TEMPERATURE clamp, one uniform [N, k] per call.
 *   - src/mlxu.c:769-774     m_seed / m_uniform -> MLX random::seed / uniform.
 *   - src/testapi.c:155-166  d3_sample.
 *
 * Parity status: the Threefry-2x32-20 block is pinned to the published
 * Random123 known-answer vectors and to JAX's documented split of key 0 (MLX
 * uses the same counter layout). MLX's bits/uniform layout (odd counts, the
 * u32 -> float mapping) is restated from MLX 0.32.3's published source
 * behaviour and is UNPINNED here: MLX cannot run in this container and the
 * reference's own tests hold no golden ids or uniforms.
 *
 * Floating-point conventions shared with the CUDA kernels (all IEEE binary32,
 * round-to-nearest-even, no contraction: build with -ffp-contract=off):
 *   - exp and log are d3o_exp / d3o_log below (Cody-Waite reduction + a
 *     degree-6 polynomial / atanh series), not libm, so the CPU and GPU agree bit for bit.
 *   - the full-row sum of exp(q - max) is taken as 256 strided partials
 *     (partial p sums elements p, p+256, ... in order, in float), each partial
 *     truncated to a 2^-46 fixed-point uint64 and the partials added exactly.
 *     Each term is exp(max(q - max, -86)): below -86 a term is far under the
 *     fixed point's resolution, and the floor keeps exp's scale normal.
 *   - the row maximum ignores the sign of zero (-0 and +0 compare equal, as in
 *     every comparison of the path); top-k order is (value desc, id asc).
 */
#ifndef D3S_ORACLE_H
#define D3S_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define D3O_F32 0
#define D3O_BF16 1
#define D3O_MIN_TEMPERATURE 1e-5f
#define D3O_PARTIALS 256

/* ---- random numbers ---- */
void d3o_threefry2x32(const uint32_t key[2], const uint32_t ctr[2], uint32_t out[2]);
void d3o_key_from_seed(uint64_t seed, uint32_t key[2]);
void d3o_split(const uint32_t key[2], uint32_t k0[2], uint32_t k1[2]);
/* global-key step: (state, sub) = split(state); returns sub */
void d3o_next_key(uint32_t state[2], uint32_t sub[2]);
uint32_t d3o_bits_word(const uint32_t key[2], uint64_t n, uint64_t f);
void d3o_bits(const uint32_t key[2], uint64_t n, uint32_t *out);
float d3o_bits_to_uniform(uint32_t b);
void d3o_uniform(const uint32_t key[2], uint64_t n, float *out);

/* ---- math ---- */
float d3o_exp(float x);
float d3o_log(float x);
void d3o_exp_array(const float *x, float *y, int64_t n);
void d3o_log_array(const float *x, float *y, int64_t n);
/* the full-row-sum term: exp(max(d, -86)) */
void d3o_term_array(const float *x, float *y, int64_t n);

/* ---- sampler ---- */
typedef struct {
  float gmax;       /* max of logits / T */
  float lse;        /* gmax + log(sum) */
  uint64_t sum_fixed; /* the 2^-46 fixed-point full-row sum */
  int kept;         /* survivors of the top-p cut (a prefix of the top k) */
  int choice;       /* rank that won the race */
  float cum_margin; /* min |cum_r - top_p| over the ranks the cut examined */
  float race_gap;   /* best score minus the runner-up score (kept ranks) */
  int bad;          /* 1 = the row's scaled logits are not finite (NaN, +inf, all -inf) */
} d3o_diag;

/* One row: x [V] logits (float), u [k] uniforms. Returns the sampled position
 * in [0, V), or -1 for a non-finite row. topk_ids / probs [k] (optional) get the
 * ranked ids and the race probabilities (0 for dropped ranks). */
int d3o_sample_row(const float *x, int V, float temperature, float top_p, int k,
                   const float *u, int32_t *topk_ids, float *probs, d3o_diag *diag);

/* Test support: the inclusive cumsums cum_r (r < k) that sample_fn compares
 * with top_p (src/sampling.c:39-43), without the cut, for a finite row.
 * Returns 0, or -1 for a non-finite row. */
int d3o_row_cums(const float *x, int V, float temperature, int k, float *cums);

/* Test support: the largest relative error of d3o_exp against double exp over
 * every float in [lo, hi] (lo <= hi <= 0, results normal), and the number of
 * adjacent floats a < b in [lo, hi] (0 < lo) with d3o_log(b) < d3o_log(a). */
double d3o_exp_max_relerr(float lo, float hi);
int64_t d3o_log_nonmonotone(float lo, float hi);

/* Top k of q [V] in the order of the Metal kernel's selection + merge
 * (src/sampling.c:93-121). vals / ids [k]. */
void d3o_topk_metal_order(const float *q, int V, int k, float *vals, int32_t *ids);
/* Top k of q [V] by (value desc, id asc), the stable-sort order. */
void d3o_topk_stable(const float *q, int V, int k, float *vals, int32_t *ids);

/* sample_with_noise over logits [N, ld] (dtype D3O_F32 / D3O_BF16), u [N, k].
 * Returns the number of non-finite rows (their ids are -1). */
int d3o_sample_with_noise(const void *logits, int dtype, int N, int V, int64_t ld,
                          const float *u, int k, float temperature, float top_p,
                          int32_t *ids, int nthreads);

/* sample_top_k_top_p on a key state: one split, u = uniform(sub, N*k). */
int d3o_sample_top_k_top_p(uint32_t state[2], const void *logits, int dtype, int N, int V,
                           int64_t ld, float temperature, int top_k, float top_p,
                           int32_t *ids, int nthreads);

/* d3_sample (src/testapi.c:155-166): seed, then sample_top_k_top_p. */
void d3o_d3_sample(const float *logits, int N, int V, float temperature, int top_k,
                   float top_p, uint64_t seed, int32_t *out);

/* Per-row parameters and seeds: row r is sampled as d3_sample(row r, seeds[r])
 * would sample it. Null arrays fall back to the scalar values. Returns the
 * number of rows flagged (non-finite logits or top_k < 1); their ids are -1. */
int d3o_sample_rows(const void *logits, int dtype, int N, int V, int64_t ld,
                    const float *temperature, const float *top_p, const int32_t *top_k,
                    const uint64_t *seeds, float temperature_all, float top_p_all,
                    int top_k_all, uint64_t seed_all, int32_t *ids, int nthreads);

/* Frame key order of tower_decode_step (src/tower.c:417-424): n_heads + 2
 * uniform draws from the global state, in order. ks[i] = k of draw i.
 * Writes the concatenated uniforms into u (sum of ks floats). */
void d3o_frame_noise(uint32_t state[2], int n_draws, const int *ks, float *u);

/* Per-row keys: row r draws u [1, k] from keys[2 * r * ld_keys ..] (a
 * stream's own subkey, as sample_noise(1, V, top_k) on that stream's key
 * sequence would). Null parameter arrays fall back to the scalars. Returns the
 * number of flagged rows (ids -1). */
int d3o_sample_rows_keys(const void *logits, int dtype, int N, int V, int64_t ld,
                         const float *temperature, const float *top_p, const int32_t *top_k,
                         float temperature_all, float top_p_all, int top_k_all,
                         const uint32_t *keys, int64_t ld_keys, int32_t *ids, int nthreads);

/* The sampling part of tower_decode_step (src/tower.c:405-433) for one
 * stream: the main draw (user T / top_p / top_k, key_main), the retry draw
 * (RAS: T 1.0, top_p 0.95, top_k 30, key_retry, src/tower.c:14-16), both on the
 * same backbone logits row; candidate_token maps index 0 to eos_id and i >= 1
 * to semantic_start + i - 1; a semantic first token found among the
 * hist_len history tokens is replaced by the retry token. Writes the frame's
 * main token, c0 = clip(main - semantic_start, 0, code_vocab - 1) and flags
 * (D3O_FRAME_*). A row with non-finite logits (the reference's die() at
 * src/generate.c:92) gets main -1, c0 0 and the NONFINITE flag. */
#define D3O_RAS_TEMPERATURE 1.0f
#define D3O_RAS_TOP_P 0.95f
#define D3O_RAS_TOP_K 30
#define D3O_RAS_WINDOW 16
#define D3O_FRAME_EOS 1
#define D3O_FRAME_NONFINITE 2
#define D3O_FRAME_RETRY 4
void d3o_frame_main(const void *logits, int dtype, int V, float temperature, float top_p,
                    int top_k, const uint32_t key_main[2], const uint32_t key_retry[2],
                    const int32_t *history, int hist_len, int semantic_start, int code_vocab,
                    int eos_id, int32_t *main_tok, int32_t *c0, int32_t *flags);

/* The history step of the decode loop (src/generate.c:97-100): append tok to
 * the window of the last D3O_RAS_WINDOW main tokens, dropping the oldest when
 * full. */
void d3o_history_push(int32_t *history, int *hist_len, int32_t tok);

#ifdef __cplusplus
}
#endif

#endif

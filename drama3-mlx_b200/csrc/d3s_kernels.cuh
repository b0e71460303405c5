// d3s_kernels.cuh - kernel arguments and launch interface of the sampler.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "d3s.h"

namespace d3s {

// Kernel arguments (passed by value). Mirrors d3s_request plus scratch.
struct KArgs {
  const void *logits;
  int64_t ld;
  int dtype;
  int N, V;
  float T, top_p;
  int top_k;
  const float *T_rows;
  const float *p_rows;
  const int32_t *k_rows;
  int noise;
  uint2 key;
  const uint64_t *seeds;
  const float *u;
  int64_t ld_u;
  int32_t *ids;
  int32_t *status;
  int32_t *kept;
  float *probs;
  int32_t *topk_ids;
  int64_t ld_out;
  const uint2 *keys;  // D3S_NOISE_KEYS: row r's key at keys[r * ld_keys]
  int64_t ld_keys;
  int32_t *finite;    // optional: 1 when every logit of the row is finite
  int row_period;     // > 0: row r reads logits row r % row_period (draws sharing logits)
  // scratch (device): rows the fast kernel hands to the wide kernel, the
  // count of those rows, and the wide kernel's completion counter.
  int32_t *deferred;
  uint32_t *deferred_n;
  uint32_t *wide_done;
  int64_t deferred_cap;  // entries of `deferred`; hand-offs beyond it flag the row
  int32_t *error;        // set to 1 when a bounded wait gives up
  // batches of one CTA per row: leave the rows handed on (no id written) on
  // the list for a later launch_handoff instead of launching the wide kernel
  int skip_handoff;
  // batches of one CTA per row: the logits are host memory mapped into the
  // device (zero-copy): each CTA loads its row with plain loads, no bulk copy
  int direct;
  // the row-independent part of the approximate full-row sum's relative error
  // bound (set by the launcher of the approximate-sum kernels)
  float approx_c0;
  // zero-copy one-row calls: set to 1 (in mapped host memory) once every
  // result of the launch is written, so the host can poll it instead of
  // waiting for the stream
  int32_t *done_flag;
};

// Per-row results the stats kernel passes to the select kernel. The header
// (dense, one per row): the row max in q, the candidate count and the four
// warps' 2^-46 fixed-point partial sums. The candidates, as raw (x bits, id)
// pairs in no particular order (the select kernel divides and keys them), live
// in a separate slab.
struct alignas(16) RowHead {
  float gmax;
  int done;    // 1: the stats kernel already wrote the row's result (or handed it on)
  int cnt;     // candidates (the first min(cnt, 256) are stored)
  int approx;  // 1: sum[] holds the SFU-exp2 approximation of the full-row sum
  unsigned long long sum[4];
};
struct alignas(16) RowCands {
  unsigned long long cand[256];
};

// Device scratch a launch needs: N RowHeads and RowCands, `deferred` N int32; counters holds 3
// uint32 that must be zero before the first launch: the hand-off count and the
// wide kernel's completion count (the wide kernel re-zeroes both), and the
// error word (cleared by the host when it reads it).
struct Scratch {
  int32_t *deferred = nullptr;
  uint32_t *counters = nullptr;
  int64_t capacity = 0;
  RowHead *heads = nullptr;  // one per row of the largest request so far
  RowCands *cands = nullptr;
  int64_t rec_capacity = 0;
};

// Raise fn's dynamic shared-memory limit to smem once per device and return its
// blocks per SM for (threads, smem), cached; 0 when an attribute call failed.
int prepare_launch(const void *fn, int threads, size_t smem);

// Test hook: which kernel takes the batches above the small-batch path
// (0 = the usual choice, 1 = stats + select pair, 3 = row-warp).
void set_force_path(int path);

// Launch the sampler for one request. Validates sizes; returns D3S_* status.
int launch_sample(const KArgs &a, const Scratch &s, cudaStream_t stream);
// The wide kernel over the hand-off list (rows a launch with skip_handoff left
// there), on the same request.
int launch_handoff(const KArgs &a, cudaStream_t stream);

// One decode frame's main + retry draws for S streams (d3s_frame_request).
struct FrameArgs {
  int S;
  float temperature, top_p;
  int top_k;
  const uint2 *keys;
  int64_t ld_keys;
  int32_t *history;
  int32_t *hist_len;
  int semantic_start, code_vocab, eos_id, update_history;
  int32_t *main_tok, *c0, *flags;
};
// Device arrays of 2S entries (rows [0, S) main, [S, 2S) retry).
struct FrameScratch {
  float *T = nullptr, *p = nullptr;
  int32_t *k = nullptr, *ids = nullptr, *finite = nullptr;
  uint2 *keys = nullptr;
  int64_t capacity = 0;  // streams
};
// `a` carries the logits (logits, dtype, V, ld) and the scratch pointers.
int launch_frame(const FrameArgs &f, const FrameScratch &fs, KArgs a, const Scratch &sc,
                 cudaStream_t stream);
// The lm_head projection: out[b, v] = bf16(h[b, :] . W[v, :]), fp32 accumulate.
// h [B, D], W [V, D], out [B, ld_out], all bf16 device memory, rows 16-byte
// aligned (ld and D multiples of 8).
constexpr int kGemvMaxB = 8;  // batch rows up to which the CUDA-core GEMV runs
struct LmArgs {
  const void *h;
  int64_t ld_h;
  const void *W;
  int64_t ld_w;
  int B, V, D;
  void *out;
  int64_t ld_out;
  int32_t *error;  // bit 1 set when a bounded wait in the GEMM gave up
};
int launch_lmhead(const LmArgs &a, cudaStream_t stream);

// Advance S key states by n splits each; subkeys at sub[s * ld_sub + i].
int launch_keys_next(uint2 *state, int S, int n, uint2 *sub, int64_t ld_sub, cudaStream_t stream);

// Record an error message for d3s_last_error() on this thread; returns code.
int set_error(int code, const char *msg);

// Draw u [rows, k] = uniform(key, rows * k) (sample_noise).
int launch_uniform(uint2 key, int rows, int k, float *u, cudaStream_t stream);

// Debug: y = exp_full(x) (op 0), log_full(x) (op 1), exp_term(x) (op 2), the
// per-row-reciprocal quotient x / T (op 3) or the SFU's 2^x (op 4) on device.
int launch_math(int op, const float *x, float *y, int64_t n, float T, cudaStream_t stream);

// Debug: count x in [lo, hi) (float bit patterns, step `step`, within the
// reciprocal path's range) whose reciprocal-path quotient x / T differs from the
// IEEE quotient, for each T of Ts[nT]; adds to *bad, last failure in example[2].
int launch_div_check(const float *Ts, int nT, uint64_t lo, uint64_t hi, uint64_t step,
                     unsigned long long *bad, float *example, cudaStream_t stream);

}  // namespace d3s

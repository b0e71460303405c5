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
  // scratch (device): rows the fast kernel hands to the wide kernel, the
  // count of those rows, and the wide kernel's completion counter.
  int32_t *deferred;
  uint32_t *deferred_n;
  uint32_t *wide_done;
  int64_t deferred_cap;  // entries of `deferred`; hand-offs beyond it flag the row
};

// Device scratch a launch needs: `deferred` holds N int32, counters 2 uint32
// that must be zero before the first launch (the wide kernel re-zeroes them).
struct Scratch {
  int32_t *deferred = nullptr;
  uint32_t *counters = nullptr;
  int64_t capacity = 0;
};

// Launch the sampler for one request. Validates sizes; returns D3S_* status.
int launch_sample(const KArgs &a, const Scratch &s, cudaStream_t stream);

// Draw u [rows, k] = uniform(key, rows * k) (sample_noise).
int launch_uniform(uint2 key, int rows, int k, float *u, cudaStream_t stream);

// Debug: y = exp_full(x) (op 0), log_full(x) (op 1), exp_term(x) (op 2) on device.
int launch_math(int op, const float *x, float *y, int64_t n, cudaStream_t stream);

}  // namespace d3s

// d3s_kernels.cu - the sampler kernels for sm_100a.
//
// Reference: src/sampling.c:22-49 (sample_fn, the semantics), src/sampling.c:53-140
// (drama3_sample, the Metal kernel it replaces), src/sampling.c:179-209 (noise and
// dispatch). Paths are relative to the drama3-mlx project root.
//
// Layout: one CTA of 256 threads per row, persistent over rows. Thread t owns
// the row's elements t, t + 256, t + 512, ... (coalesced loads), which are
// exactly the elements of full-row-sum partial t, so the partial is a
// sequential float sum inside one thread. The fast kernel keeps the row in
// registers (V <= 8192, k <= 256); the wide kernel streams the row from global
// memory for larger V or k.
//
// Per row: q = x / T (IEEE divide) and its max (one warp redux + 8-way smem);
// partial sums of exp(q - max) in float, truncated to 2^-46 fixed point and
// summed exactly (two 32-bit warp reduxes); a candidate threshold (the
// ceil(k/8)-th largest thread max of each warp, min over warps) that at least
// k elements reach; the candidates are ranked by counting in shared memory; a
// single warp then runs the sequential cumsum, drop rule, softmax and the
// exponential race with an in-kernel threefry uniform.
#include <algorithm>

#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

namespace d3s {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kCandCap = 1024;
constexpr int kFastMaxK = 256;
constexpr int kFastMaxV = 32 * kThreads;
constexpr unsigned kFull = 0xffffffffu;

template <bool BF16>
__device__ __forceinline__ float load_x(const void *base, int64_t i) {
  if constexpr (BF16) {
    const unsigned short h = __ldg(reinterpret_cast<const unsigned short *>(base) + i);
    return __uint_as_float((unsigned)h << 16);
  } else {
    return __ldg(reinterpret_cast<const float *>(base) + i);
  }
}

template <bool BF16>
__device__ __forceinline__ const void *row_base(const KArgs &a, int row) {
  const int64_t off = (int64_t)row * a.ld;
  if constexpr (BF16)
    return reinterpret_cast<const unsigned short *>(a.logits) + off;
  else
    return reinterpret_cast<const float *>(a.logits) + off;
}

struct RowP {
  float T, p;
  int k;
};

// Per-row parameters: the MIN_TEMPERATURE clamp (src/sampling.c:195) and
// k = min(top_k, V) (src/sampling.c:207). NaN temperature or top_k < 1 flag the row.
__device__ __forceinline__ int row_params(const KArgs &a, int row, RowP &rp) {
  const float T = a.T_rows ? a.T_rows[row] : a.T;
  const float p = a.p_rows ? a.p_rows[row] : a.top_p;
  const int tk = a.k_rows ? a.k_rows[row] : a.top_k;
  if (tk < 1 || T != T) return D3S_ROW_BADPARAM;
  const int k = min(tk, a.V);
  if (k > D3S_MAX_K) return D3S_ROW_BADPARAM;
  rp.T = T < kMinTemperature ? kMinTemperature : T;
  rp.p = p;
  rp.k = k;
  return D3S_ROW_OK;
}

__device__ __forceinline__ void flag_row(const KArgs &a, int row, int code) {
  a.ids[row] = -1;
  if (a.status) a.status[row] = code;
  if (a.kept) a.kept[row] = 0;
}

__device__ __forceinline__ uint2 row_key(const KArgs &a, int row) {
  return a.noise == D3S_NOISE_SEEDS ? seed_subkey(a.seeds[row]) : a.key;
}

// u for (row, rank r): the word of the [N, k] (one key) or [1, k] (per-row seed)
// uniform array that sample_top_k_top_p / d3_sample would draw.
__device__ __forceinline__ float row_uniform(const KArgs &a, int row, int k, int r, uint2 key) {
  if (a.noise == D3S_NOISE_GIVEN) return a.u[(int64_t)row * a.ld_u + r];
  const bool one = a.noise == D3S_NOISE_KEY;
  const uint64_t n = one ? (uint64_t)a.N * (uint64_t)k : (uint64_t)k;
  const uint64_t f = one ? (uint64_t)row * (uint64_t)k + (uint64_t)r : (uint64_t)r;
  return bits_to_uniform(bits_word(key, n, f));
}

// The serial end of a row, run by one warp: sorted[k] holds the top-k keys in
// rank order, scr[k] is scratch. Inclusive cumsum of exp(v - lse) in rank
// order (src/sampling.c:39, :126-127), drop when cum > top_p at rank > 0
// (:40-43, :128), softmax over the survivors with a 1/sum multiply (:44,
// :129-134), race p / -log(1 - u) with the first strictly greater score
// winning (:45-47, :135-137).
__device__ void sample_tail(const KArgs &a, int row, const unsigned long long *sorted, float *scr,
                            int k, float lse, float top_p, int lane) {
  for (int r = lane; r < k; r += 32) scr[r] = exp_full(__fsub_rn(cand_value(sorted[r]), lse));
  __syncwarp();
  int kept = k;
  if (lane == 0) {
    float cum = 0.0f;
    for (int r = 0; r < k; ++r) {
      cum = __fadd_rn(cum, scr[r]);
      if (r > 0 && cum > top_p) {
        kept = r;
        break;
      }
    }
  }
  kept = __shfl_sync(kFull, kept, 0);
  __syncwarp();
  const float top = cand_value(sorted[0]);
  for (int r = lane; r < kept; r += 32) scr[r] = exp_full(__fsub_rn(cand_value(sorted[r]), top));
  __syncwarp();
  float inv = 0.0f;
  if (lane == 0) {
    float sum = 0.0f;
    for (int r = 0; r < kept; ++r) sum = __fadd_rn(sum, scr[r]);
    inv = __fdiv_rn(1.0f, sum);
  }
  inv = __shfl_sync(kFull, inv, 0);
  const uint2 key = a.noise == D3S_NOISE_GIVEN ? make_uint2(0u, 0u) : row_key(a, row);
  float best = -1.0f;
  int best_r = 0;
  for (int r = lane; r < k; r += 32) {
    const float p = r < kept ? __fmul_rn(scr[r], inv) : 0.0f;
    const float u = row_uniform(a, row, k, r, key);
    const float noise = -log_full(__fsub_rn(1.0f, u));
    const float score = __fdiv_rn(p, noise);
    if (a.probs) a.probs[(int64_t)row * a.ld_out + r] = p;
    if (a.topk_ids) a.topk_ids[(int64_t)row * a.ld_out + r] = cand_id(sorted[r]);
    if (score > best) {
      best = score;
      best_r = r;
    }
  }
  const float wbest = warp_max(best);
  const unsigned choice = __reduce_min_sync(kFull, best == wbest ? (unsigned)best_r : 0xffffffffu);
  if (lane == 0) {
    a.ids[row] = cand_id(sorted[choice]);
    if (a.status) a.status[row] = D3S_ROW_OK;
    if (a.kept) a.kept[row] = kept;
  }
}

struct FastSmem {
  float red_max[kWarps];
  float red_tau[kWarps];
  unsigned long long red_sum[kWarps];
  int red_cnt[2][kWarps];
  unsigned cand_n;
  unsigned long long cand[kCandCap];
  unsigned long long sorted[kFastMaxK];
  float scr[kFastMaxK];
};

// Sum of the 2^-46 fixed-point partials of one warp (each < 2^51): the low 26
// and high 25 bits are reduced separately so 32-bit reduxes cannot overflow.
__device__ __forceinline__ unsigned long long warp_sum_fixed(unsigned long long fx) {
  unsigned lo = (unsigned)(fx & ((1ull << 26) - 1));
  unsigned hi = (unsigned)(fx >> 26);
  lo = __reduce_add_sync(kFull, lo);
  hi = __reduce_add_sync(kFull, hi);
  return ((unsigned long long)hi << 26) + lo;
}

// The r-th largest of the warp's 32 values (-inf when fewer than r are finite).
__device__ __forceinline__ float warp_rth_largest(float v, int r) {
  int cnt = 0;
  for (;;) {
    const float mx = warp_max(v);
    cnt += __popc(__ballot_sync(kFull, v == mx));
    if (cnt >= r || mx == -f_inf()) return mx;
    if (v == mx) v = -f_inf();
  }
}

template <int J, bool BF16>
__global__ void __launch_bounds__(kThreads) sample_fast_kernel(const KArgs a) {
  __shared__ FastSmem sm;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int V = a.V;
  if (t == 0) sm.cand_n = 0;
  __syncthreads();
  for (int row = blockIdx.x; row < a.N; row += gridDim.x) {
    RowP rp;
    const int pst = row_params(a, row, rp);
    if (pst != D3S_ROW_OK) {
      if (t == 0) flag_row(a, row, pst);
      continue;
    }
    if (rp.k > kFastMaxK) {  // handed to the wide kernel
      if (t == 0) {
        const unsigned pos = atomicAdd(a.deferred_n, 1u);
        if (pos < (unsigned long long)a.deferred_cap)
          a.deferred[pos] = row;
        else
          flag_row(a, row, D3S_ROW_BADPARAM);
      }
      continue;
    }
    const void *base = row_base<BF16>(a, row);
    // ---- q = x / T and the row max ----
    float q[J];
    float m = -f_inf();
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = t + kThreads * j;
      const float x = i < V ? load_x<BF16>(base, i) : -f_inf();
      q[j] = __fdiv_rn(x, rp.T);
      m = max_nan(m, q[j]);
    }
    const float wm = warp_max_nan(m);
    if (lane == 0) sm.red_max[w] = wm;
    __syncthreads();
    float gmax = sm.red_max[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) gmax = max_nan(gmax, sm.red_max[i]);
    if (!(fabsf(gmax) < f_inf())) {  // NaN, +inf, or every value -inf
      if (t == 0) flag_row(a, row, D3S_ROW_NONFINITE);
      __syncthreads();
      continue;
    }
    // ---- partial t of the full-row sum (padding terms are exactly 0) ----
    float s = 0.0f;
    const float2 mg = make_float2(-gmax, -gmax);
#pragma unroll
    for (int j = 0; j + 1 < J; j += 2) {
      const float2 e = exp_term2(__fadd2_rn(make_float2(q[j], q[j + 1]), mg));
      s = __fadd_rn(s, e.x);
      s = __fadd_rn(s, e.y);
    }
    if (J & 1) s = __fadd_rn(s, exp_term(__fsub_rn(q[J - 1], gmax)));
    const unsigned long long wsum = warp_sum_fixed(__float2ull_rz(__fmul_rn(s, 0x1p46f)));
    const float tau_w = warp_rth_largest(m, (rp.k + kWarps - 1) / kWarps);
    if (lane == 0) {
      sm.red_sum[w] = wsum;
      sm.red_tau[w] = tau_w;
    }
    __syncthreads();
    unsigned long long S = 0;
    float tau = f_inf();
#pragma unroll
    for (int i = 0; i < kWarps; ++i) {
      S += sm.red_sum[i];
      tau = fminf(tau, sm.red_tau[i]);
    }
    const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
    // ---- candidates: every element >= tau (at least k of them) ----
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = t + kThreads * j;
      if (i < V && q[j] >= tau) {
        const unsigned pos = atomicAdd(&sm.cand_n, 1u);
        if (pos < kCandCap) sm.cand[pos] = cand_key(q[j], (uint32_t)i);
      }
    }
    __syncthreads();
    unsigned C = sm.cand_n;
    if (C > kCandCap) {
      // Too many (ties): find the k-th largest key exactly by bisection on the
      // 64-bit (value, id) key, then take exactly the k keys at or above it.
      unsigned long long P = 0;
      for (int b = 63; b >= 0; --b) {
        const unsigned long long trial = P | (1ull << b);
        int c = 0;
#pragma unroll
        for (int j = 0; j < J; ++j) {
          const int i = t + kThreads * j;
          c += (i < V && cand_key(q[j], (uint32_t)i) >= trial) ? 1 : 0;
        }
        c = __reduce_add_sync(kFull, c);
        if (lane == 0) sm.red_cnt[b & 1][w] = c;
        __syncthreads();
        int tot = 0;
#pragma unroll
        for (int i = 0; i < kWarps; ++i) tot += sm.red_cnt[b & 1][i];
        if (tot >= rp.k) P = trial;
      }
      if (t == 0) sm.cand_n = 0;
      __syncthreads();
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int i = t + kThreads * j;
        if (i < V) {
          const unsigned long long key = cand_key(q[j], (uint32_t)i);
          if (key >= P) sm.cand[atomicAdd(&sm.cand_n, 1u)] = key;
        }
      }
      __syncthreads();
      C = (unsigned)rp.k;
    }
    // ---- rank the candidates by counting; keys are unique ----
    for (unsigned c = t; c < C; c += kThreads) {
      const unsigned long long kc = sm.cand[c];
      unsigned rank = 0;
      for (unsigned c2 = 0; c2 < C; ++c2) rank += sm.cand[c2] > kc ? 1u : 0u;
      if (rank < (unsigned)rp.k) sm.sorted[rank] = kc;
    }
    __syncthreads();
    if (w == 0) {
      if (lane == 0) sm.cand_n = 0;
      sample_tail(a, row, sm.sorted, sm.scr, rp.k, lse, rp.p, lane);
    }
  }
}

// Wide path: any V <= D3S_MAX_V and k <= D3S_MAX_K. The row is re-read from
// global memory (L2) in each pass; selection is the exact bisection on the
// 64-bit key, then a bitonic sort of the k winners in shared memory.
template <bool BF16>
__global__ void __launch_bounds__(kThreads) sample_wide_kernel(const KArgs a, int use_list,
                                                                int kcap) {
  extern __shared__ unsigned long long keys[];  // [pow2 >= kcap] keys, then float scr[kcap]
  __shared__ float red_max[kWarps];
  __shared__ unsigned long long red_sum[kWarps];
  __shared__ int red_cnt[2][kWarps];
  __shared__ unsigned gather_n;
  int kp_cap = 1;
  while (kp_cap < kcap) kp_cap <<= 1;
  float *scr = reinterpret_cast<float *>(keys + kp_cap);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int V = a.V;
  const unsigned nrows =
      use_list ? (unsigned)min((long long)*((volatile uint32_t *)a.deferred_n), (long long)a.deferred_cap)
               : (unsigned)a.N;
  for (unsigned idx = blockIdx.x; idx < nrows; idx += gridDim.x) {
    const int row = use_list ? a.deferred[idx] : (int)idx;
    RowP rp;
    const int pst = row_params(a, row, rp);
    if (pst != D3S_ROW_OK || rp.k > kcap) {
      if (t == 0) flag_row(a, row, D3S_ROW_BADPARAM);
      continue;
    }
    const int k = rp.k;
    int kp = 1;
    while (kp < k) kp <<= 1;
    const void *base = row_base<BF16>(a, row);
    float m = -f_inf();
    for (int i = t; i < V; i += kThreads) m = max_nan(m, __fdiv_rn(load_x<BF16>(base, i), rp.T));
    const float wm = warp_max_nan(m);
    if (lane == 0) red_max[w] = wm;
    __syncthreads();
    float gmax = red_max[0];
#pragma unroll
    for (int i = 1; i < kWarps; ++i) gmax = max_nan(gmax, red_max[i]);
    if (!(fabsf(gmax) < f_inf())) {
      if (t == 0) flag_row(a, row, D3S_ROW_NONFINITE);
      __syncthreads();
      continue;
    }
    float s = 0.0f;
    for (int i = t; i < V; i += kThreads)
      s = __fadd_rn(s, exp_term(__fsub_rn(__fdiv_rn(load_x<BF16>(base, i), rp.T), gmax)));
    const unsigned long long wsum = warp_sum_fixed(__float2ull_rz(__fmul_rn(s, 0x1p46f)));
    if (lane == 0) red_sum[w] = wsum;
    __syncthreads();
    unsigned long long S = 0;
#pragma unroll
    for (int i = 0; i < kWarps; ++i) S += red_sum[i];
    const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
    unsigned long long P = 0;
    for (int b = 63; b >= 0; --b) {
      const unsigned long long trial = P | (1ull << b);
      int c = 0;
      for (int i = t; i < V; i += kThreads)
        c += cand_key(__fdiv_rn(load_x<BF16>(base, i), rp.T), (uint32_t)i) >= trial ? 1 : 0;
      c = __reduce_add_sync(kFull, c);
      if (lane == 0) red_cnt[b & 1][w] = c;
      __syncthreads();
      int tot = 0;
#pragma unroll
      for (int i = 0; i < kWarps; ++i) tot += red_cnt[b & 1][i];
      if (tot >= k) P = trial;
    }
    if (t == 0) gather_n = 0;
    __syncthreads();
    for (int i = t; i < V; i += kThreads) {
      const unsigned long long key = cand_key(__fdiv_rn(load_x<BF16>(base, i), rp.T), (uint32_t)i);
      if (key >= P) keys[atomicAdd(&gather_n, 1u)] = key;
    }
    for (int i = k + t; i < kp; i += kThreads) keys[i] = 0ull;
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= kp; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = t; i < (kp >> 1); i += kThreads) {
          const int lo = 2 * stride * (i / stride) + (i % stride);
          const int hi = lo + stride;
          const bool desc = (lo & size) == 0;
          const unsigned long long x = keys[lo], y = keys[hi];
          if (desc ? (x < y) : (x > y)) {
            keys[lo] = y;
            keys[hi] = x;
          }
        }
        __syncthreads();
      }
    }
    if (w == 0) sample_tail(a, row, keys, scr, k, lse, rp.p, lane);
    __syncthreads();
  }
  if (use_list) {
    // The last CTA to finish re-zeroes the hand-off counters for the next launch:
    // every CTA has read deferred_n before it counts itself done.
    __syncthreads();
    if (t == 0) {
      __threadfence();
      const unsigned d = atomicAdd(a.wide_done, 1u);
      if (d == gridDim.x - 1) {
        *a.deferred_n = 0u;
        *a.wide_done = 0u;
        __threadfence();
      }
    }
  }
}

__global__ void uniform_kernel(uint2 key, uint64_t n, float *u) {
  for (uint64_t f = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n;
       f += (uint64_t)gridDim.x * blockDim.x)
    u[f] = bits_to_uniform(bits_word(key, n, f));
}

__global__ void math_kernel(int op, const float *x, float *y, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    y[i] = op == 0 ? exp_full(v) : (op == 1 ? log_full(v) : exp_term(v));
  }
}

// ---- launch helpers ----

using FastFn = void (*)(const KArgs);

template <bool BF16>
FastFn pick_fast(int J) {
  switch (J) {
    case 1: return sample_fast_kernel<1, BF16>;
    case 2: return sample_fast_kernel<2, BF16>;
    case 4: return sample_fast_kernel<4, BF16>;
    case 8: return sample_fast_kernel<8, BF16>;
    case 16: return sample_fast_kernel<16, BF16>;
    case 17: return sample_fast_kernel<17, BF16>;
    case 24: return sample_fast_kernel<24, BF16>;
    case 32: return sample_fast_kernel<32, BF16>;
    default: return nullptr;
  }
}

int pick_J(int V) {
  const int need = (V + kThreads - 1) / kThreads;
  static const int Js[] = {1, 2, 4, 8, 16, 17, 24, 32};
  for (int J : Js)
    if (J >= need) return J;
  return 0;
}

struct DevInfo {
  int dev = -1;
  int sms = 0;
};

int device_sms() {
  static thread_local DevInfo cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cache.dev != dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cache.dev = dev;
    cache.sms = sms;
  }
  return cache.sms;
}

int occupancy(const void *fn, size_t smem) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, kThreads, smem) != cudaSuccess)
    return 1;
  return std::max(blocks, 1);
}

size_t wide_smem(int kcap) {
  int kp = 1;
  while (kp < kcap) kp <<= 1;
  return (size_t)kp * sizeof(unsigned long long) + (size_t)kcap * sizeof(float);
}

template <bool BF16>
int launch_wide(const KArgs &a, int use_list, int kcap, cudaStream_t st) {
  const size_t smem = wide_smem(kcap);
  auto fn = sample_wide_kernel<BF16>;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return D3S_ERR_CUDA;
  const int sms = device_sms();
  int grid = sms * occupancy((const void *)fn, smem);
  if (!use_list) grid = std::min(grid, a.N);
  if (grid < 1) grid = 1;
  fn<<<grid, kThreads, smem, st>>>(a, use_list, kcap);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

template <bool BF16>
int launch_typed(const KArgs &a, const Scratch &s, cudaStream_t st) {
  const bool scalar_k = a.k_rows == nullptr;
  const int J = a.V <= kFastMaxV ? pick_J(a.V) : 0;
  const int kscalar = std::min(a.top_k, a.V);
  if (J == 0 || (scalar_k && kscalar > kFastMaxK))
    return launch_wide<BF16>(a, 0, scalar_k ? kscalar : D3S_MAX_K, st);
  if (!scalar_k && (!s.deferred || !s.counters || s.capacity < a.N)) return D3S_ERR_ARG;
  FastFn fn = pick_fast<BF16>(J);
  const int sms = device_sms();
  if (sms <= 0) return D3S_ERR_CUDA;
  const int grid = std::max(1, std::min(a.N, sms * occupancy((const void *)fn, 0)));
  fn<<<grid, kThreads, 0, st>>>(a);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  if (!scalar_k) return launch_wide<BF16>(a, 1, D3S_MAX_K, st);
  return D3S_OK;
}

}  // namespace

int launch_sample(const KArgs &a, const Scratch &s, cudaStream_t st) {
  if (a.N == 0) return D3S_OK;
  return a.dtype == D3S_BF16 ? launch_typed<true>(a, s, st) : launch_typed<false>(a, s, st);
}

int launch_uniform(uint2 key, int rows, int k, float *u, cudaStream_t st) {
  const uint64_t n = (uint64_t)rows * (uint64_t)k;
  if (n == 0) return D3S_OK;
  const int sms = device_sms();
  const int grid = (int)std::min<uint64_t>((n + 255) / 256, (uint64_t)std::max(sms, 1) * 8);
  uniform_kernel<<<grid, 256, 0, st>>>(key, n, u);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

int launch_math(int op, const float *x, float *y, int64_t n, cudaStream_t st) {
  if (n == 0) return D3S_OK;
  const int sms = device_sms();
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)std::max(sms, 1) * 16);
  math_kernel<<<grid, 256, 0, st>>>(op, x, y, n);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

}  // namespace d3s

// d3s_kernels.cu - the sampler kernels for sm_100a.
//
// Reference: src/sampling.c:22-49 (sample_fn, the semantics), src/sampling.c:53-140
// (drama3_sample, the Metal kernel it replaces), src/sampling.c:179-209 (noise and
// dispatch). Paths are relative to the drama3-mlx project root.
//
// Fast kernel (V <= 8192, k <= 256): persistent CTAs of 4 warps, one row at a
// time per CTA. Each row is fetched by a 1-D bulk copy (cp.async.bulk, the TMA
// engine) into a shared-memory stage, `stages` rows ahead, completing on an
// mbarrier; thread t owns full-row-sum partials t and t + 128 (elements
// p, p + 256, p + 512, ... of partial p), so each partial is a sequential float
// sum inside one thread, and the two partials run as one packed fp32x2 chain.
// Per row: the row max and |x| range (warp redux + 4-way smem), q = x / T by a
// per-row reciprocal with one correction step (exactly the IEEE quotient when
// the row is in range, else the IEEE divide per element), the partial sums of
// exp(q - max) in 2^-46 fixed point summed exactly, a candidate threshold that
// at least k elements reach, a warp bitonic sort of the candidates, and one
// warp's serial tail: cumsum, drop rule, softmax, exponential race with an
// in-kernel threefry uniform.
//
// Wide kernel (any V <= 131072, k <= 16384): one CTA per row, the row re-read
// from global memory (L2) in each pass, selection by exact bisection on the
// 64-bit (value, id) key, bitonic sort of the k winners in shared memory.
#include <algorithm>

#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

namespace d3s {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kPartials = 256;
constexpr int kCandCap = 256;    // fast kernel candidate buffer
constexpr int kSortMax = 256;    // warp bitonic sort up to 8 keys per lane
constexpr int kFastMaxK = 256;
constexpr int kFastW = 4;        // warps per CTA in the fast kernel
constexpr int kFastThreads = 32 * kFastW;
constexpr int kFastPP = kPartials / kFastThreads;  // partials per thread (2)
constexpr int kFastMaxV = 32 * kPartials;          // 8192
constexpr int kMaxStages = 4;
constexpr int kWideThreads = 256;
constexpr int kWideWarps = kWideThreads / 32;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// ---- PTX wrappers: mbarrier, 1-D bulk copy, bounded waits ----

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait for an mbarrier phase with a time limit; false = gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

// ---- loads and per-row parameters ----

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
__device__ __forceinline__ float lds_x(const unsigned char *base, int i) {
  if constexpr (BF16)
    return __uint_as_float((unsigned)reinterpret_cast<const unsigned short *>(base)[i] << 16);
  else
    return reinterpret_cast<const float *>(base)[i];
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

// q = x / T, correctly rounded, from rT = RN(1/T): q0 = RN(x rT) is within an
// ulp, the residual x - q0 T is exact, and one fused correction gives RN(x / T)
// (Markstein, IBM J. Res. Dev. 34(1), 1990). Valid while quotients and
// residuals stay normal: the caller checks the row's |x| range and T.
__device__ __forceinline__ float2 div_rows2(float2 x, float2 rT, float2 mT) {
  const float2 q0 = __fmul2_rn(x, rT);
  const float2 e = __ffma2_rn(q0, mT, x);
  return __ffma2_rn(e, rT, q0);
}
__device__ __forceinline__ float div_rows(float x, float rT, float mT) {
  const float q0 = __fmul_rn(x, rT);
  const float e = __fmaf_rn(q0, mT, x);
  return __fmaf_rn(e, rT, q0);
}
// Range in which div_rows is exact: nonzero |x| in [2^-60, 2^60], T in [2^-20, 2^20].
__device__ __forceinline__ bool div_rows_ok(float amin, float amax, float T) {
  return amin >= 0x1p-60f && amax <= 0x1p60f && T >= 0x1p-20f && T <= 0x1p20f;
}

// ---- warp helpers ----

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  const unsigned lo = __shfl_xor_sync(kFull, (unsigned)v, m);
  const unsigned hi = __shfl_xor_sync(kFull, (unsigned)(v >> 32), m);
  return ((unsigned long long)hi << 32) | lo;
}

// Sum of the 2^-46 fixed-point partial sums of one warp (each lane's value
// < 2^52): the low 26 and high bits are reduced separately so the 32-bit
// reduxes cannot overflow.
__device__ __forceinline__ unsigned long long warp_sum_fixed(unsigned long long fx) {
  unsigned lo = (unsigned)(fx & ((1ull << 26) - 1));
  unsigned hi = (unsigned)(fx >> 26);
  lo = __reduce_add_sync(kFull, lo);
  hi = __reduce_add_sync(kFull, hi);
  return ((unsigned long long)hi << 26) + lo;
}

// The r-th largest of the warp's 32 * M values (v[M] per lane; -inf when fewer
// than r are finite). Each round removes every copy of the current maximum.
template <int M>
__device__ __forceinline__ float warp_rth_largest(float (&v)[M], int r) {
  int cnt = 0;
  for (;;) {
    float m = v[0];
#pragma unroll
    for (int i = 1; i < M; ++i) m = fmaxf(m, v[i]);
    const float mx = warp_max(m);
#pragma unroll
    for (int i = 0; i < M; ++i) cnt += __popc(__ballot_sync(kFull, v[i] == mx));
    if (cnt >= r || mx == -f_inf()) return mx;
#pragma unroll
    for (int i = 0; i < M; ++i) v[i] = v[i] == mx ? -f_inf() : v[i];
  }
}

// Bitonic sort of 32 * S keys held as v[s] = element lane + 32 s, descending.
template <int S>
__device__ __forceinline__ void warp_sort_desc(unsigned long long (&v)[S], int lane) {
  constexpr int n = 32 * S;
#pragma unroll
  for (int size = 2; size <= n; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride >= 32) {
        const int ss = stride / 32;
#pragma unroll
        for (int s = 0; s < S; ++s) {
          if ((s & ss) == 0) {
            const bool desc = ((lane + 32 * s) & size) == 0;
            const unsigned long long x = v[s], y = v[s | ss];
            const bool swap = desc ? (x < y) : (x > y);
            v[s] = swap ? y : x;
            v[s | ss] = swap ? x : y;
          }
        }
      } else {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const unsigned long long o = shfl_xor_u64(v[s], stride);
          const bool desc = ((lane + 32 * s) & size) == 0;
          const bool lower = (lane & stride) == 0;
          const bool keep_max = lower == desc;
          const unsigned long long mx = v[s] > o ? v[s] : o, mn = v[s] > o ? o : v[s];
          v[s] = keep_max ? mx : mn;
        }
      }
    }
  }
}

// Sort keys[0..C) (C <= 32 S) descending in place with one warp; pads with 0.
template <int S>
__device__ __forceinline__ void warp_sort_smem(unsigned long long *keys, int C, int lane) {
  unsigned long long v[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int e = lane + 32 * s;
    v[s] = e < C ? keys[e] : 0ull;
  }
  __syncwarp();
  warp_sort_desc<S>(v, lane);
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int e = lane + 32 * s;
    if (e < C) keys[e] = v[s];
  }
  __syncwarp();
}

__device__ __forceinline__ void warp_sort_any(unsigned long long *keys, int C, int lane) {
  if (C <= 32)
    warp_sort_smem<1>(keys, C, lane);
  else if (C <= 64)
    warp_sort_smem<2>(keys, C, lane);
  else if (C <= 128)
    warp_sort_smem<4>(keys, C, lane);
  else
    warp_sort_smem<8>(keys, C, lane);
}

// The serial end of a row, run by one warp: sorted[k] holds the top-k keys in
// rank order, scr[k] is scratch. Inclusive cumsum of exp(v - lse) in rank
// order (src/sampling.c:39, :126-127), drop when cum > top_p at rank > 0
// (:40-43, :128), softmax over the survivors with a 1/sum multiply (:44,
// :129-134), race p / -log(1 - u) where the first strictly greater score wins
// (:45-47, :135-137). Survivors form a prefix of the ranks and every survivor's
// score is positive unless its noise is -0, so the dropped ranks (p = 0, score
// 0 or NaN) are only drawn when no survivor scored above 0.
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
  for (int r = lane; r < kept; r += 32) {
    const float p = __fmul_rn(scr[r], inv);
    const float noise = -log_full(__fsub_rn(1.0f, row_uniform(a, row, k, r, key)));
    const float score = __fdiv_rn(p, noise);
    if (a.probs) a.probs[(int64_t)row * a.ld_out + r] = p;
    if (score > best) {
      best = score;
      best_r = r;
    }
  }
  float wbest = warp_max(best);
  if (!(wbest > 0.0f)) {
    for (int r = kept + lane; r < k; r += 32) {
      const float noise = -log_full(__fsub_rn(1.0f, row_uniform(a, row, k, r, key)));
      const float score = __fdiv_rn(0.0f, noise);
      if (score > best) {
        best = score;
        best_r = r;
      }
    }
    wbest = warp_max(best);
  }
  if (a.probs)
    for (int r = kept + lane; r < k; r += 32) a.probs[(int64_t)row * a.ld_out + r] = 0.0f;
  if (a.topk_ids)
    for (int r = lane; r < k; r += 32) a.topk_ids[(int64_t)row * a.ld_out + r] = cand_id(sorted[r]);
  const unsigned choice = __reduce_min_sync(kFull, best == wbest ? (unsigned)best_r : 0xffffffffu);
  if (lane == 0) {
    a.ids[row] = cand_id(sorted[choice]);
    if (a.status) a.status[row] = D3S_ROW_OK;
    if (a.kept) a.kept[row] = kept;
  }
}

// ---- fast kernel ----

struct alignas(16) FastSmem {
  uint64_t mbar[kMaxStages];
  float red_max[kFastW];
  float red_amax[kFastW];
  float red_amin[kFastW];
  float red_tau[kFastW];
  unsigned long long red_sum[kFastW];
  int red_cnt[2][kFastW];
  unsigned cand_n[2];  // by row parity: row it+1's counter is cleared during row it
  unsigned long long cand[kCandCap];
  float scr[kCandCap];
};

// Issue the bulk copy of row `row` into stage s: the 16-byte-aligned span that
// covers the row (a copy must start and end on 16-byte boundaries).
template <int ESZ>
__device__ __forceinline__ void issue_row(const KArgs &a, int row, unsigned char *stage,
                                          uint64_t *bar) {
  const uintptr_t start = (uintptr_t)a.logits + (uintptr_t)row * (uintptr_t)a.ld * ESZ;
  const uintptr_t lo = start & ~(uintptr_t)15;
  const uintptr_t hi = (start + (uintptr_t)a.V * ESZ + 15) & ~(uintptr_t)15;
  const uint32_t bytes = (uint32_t)(hi - lo);
  mbar_expect_tx(bar, bytes);
  bulk_g2s(stage, reinterpret_cast<const void *>(lo), bytes, bar);
}

template <int JJ, bool BF16>
__global__ void __launch_bounds__(kFastThreads) sample_fast_kernel(const KArgs a, int stages,
                                                                    int span) {
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ FastSmem sm;
  constexpr int PP = kFastPP;
  constexpr int NT = kFastThreads;
  constexpr int ESZ = BF16 ? 2 : 4;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int V = a.V;
  if (t == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&sm.mbar[s], 1);
    sm.cand_n[0] = 0;
    sm.cand_n[1] = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (t == 0)
    for (int s = 0; s < stages; ++s) {
      const int r = blockIdx.x + s * gridDim.x;
      if (r < a.N) issue_row<ESZ>(a, r, dsm + (size_t)s * span, &sm.mbar[s]);
    }
  int it = 0;
  bool failed = false;
  for (;; ++it) {
    const int row = blockIdx.x + it * gridDim.x;
    if (row >= a.N) break;
    const int s = it % stages;
    const bool ok = mbar_wait_bounded(&sm.mbar[s], (uint32_t)(it / stages) & 1u);
    const unsigned char *rb =
        dsm + (size_t)s * span +
        (((uintptr_t)a.logits + (uintptr_t)row * (uintptr_t)a.ld * ESZ) & 15);
    // ---- the row into registers; its max and |x| range ----
    float q[PP][JJ];
    float pm[PP];
    float amax = 0.0f, amin = f_inf();
#pragma unroll
    for (int m = 0; m < PP; ++m) {
      pm[m] = -f_inf();
#pragma unroll
      for (int j = 0; j < JJ; ++j) {
        const int i = t + NT * m + kPartials * j;
        const bool valid = ok && i < V;
        const float v = valid ? lds_x<BF16>(rb, i) : -f_inf();
        q[m][j] = v;
        pm[m] = max_nan(pm[m], v);
        if (valid) {
          amax = fmaxf(amax, fabsf(v));
          amin = fminf(amin, fabsf(v));
        }
      }
    }
    {
      const float wm = warp_max_nan(max_nan(pm[0], pm[PP - 1]));
      const float wa = warp_max(amax);
      const float wi = -warp_max(-amin);
      if (lane == 0) {
        sm.red_max[w] = wm;
        sm.red_amax[w] = wa;
        sm.red_amin[w] = wi;
      }
    }
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    if (t == 0 && row + stages * (int)gridDim.x < a.N) {  // the stage is free: refill it
      fence_proxy_async();
      issue_row<ESZ>(a, row + stages * gridDim.x, dsm + (size_t)s * span, &sm.mbar[s]);
    }
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
    float xmax = sm.red_max[0], xamax = sm.red_amax[0], xamin = sm.red_amin[0];
#pragma unroll
    for (int i = 1; i < kFastW; ++i) {
      xmax = max_nan(xmax, sm.red_max[i]);
      xamax = fmaxf(xamax, sm.red_amax[i]);
      xamin = fminf(xamin, sm.red_amin[i]);
    }
    const float gmax = __fdiv_rn(xmax, rp.T);  // max(x / T) = RN(max(x) / T): RN is monotone
    if (!(fabsf(gmax) < f_inf())) {             // NaN, +inf, or every value -inf
      if (t == 0) flag_row(a, row, D3S_ROW_NONFINITE);
      __syncthreads();
      continue;
    }
    // ---- q = x / T ----
    if (div_rows_ok(xamin, xamax, rp.T)) {
      const float rT = __frcp_rn(rp.T);
      const float2 rT2 = make_float2(rT, rT), mT2 = make_float2(-rp.T, -rp.T);
#pragma unroll
      for (int j = 0; j < JJ; ++j) {
        const float2 r2 = div_rows2(make_float2(q[0][j], q[PP - 1][j]), rT2, mT2);
        q[0][j] = r2.x;
        q[PP - 1][j] = r2.y;
      }
#pragma unroll
      for (int m = 0; m < PP; ++m)  // padding past V stays -inf (only the last column has any)
        if (t + NT * m + kPartials * (JJ - 1) >= V) q[m][JJ - 1] = -f_inf();
    } else {
#pragma unroll
      for (int m = 0; m < PP; ++m)
#pragma unroll
        for (int j = 0; j < JJ; ++j) q[m][j] = __fdiv_rn(q[m][j], rp.T);
    }
    float pq[PP];
#pragma unroll
    for (int m = 0; m < PP; ++m) pq[m] = __fdiv_rn(pm[m], rp.T);
    // ---- partials t and t + 128 of the full-row sum, one packed chain ----
    float2 s2 = make_float2(0.0f, 0.0f);
    const float2 mg = make_float2(-gmax, -gmax);
#pragma unroll
    for (int j = 0; j < JJ; ++j)
      s2 = __fadd2_rn(s2, exp_term2(__fadd2_rn(make_float2(q[0][j], q[PP - 1][j]), mg)));
    const unsigned long long fx =
        __float2ull_rz(__fmul_rn(s2.x, 0x1p46f)) + __float2ull_rz(__fmul_rn(s2.y, 0x1p46f));
    const unsigned long long wsum = warp_sum_fixed(fx);
    // candidate threshold: each warp's ceil(k/4)-th largest partial max, min over warps
    const float tau_w = warp_rth_largest<PP>(pq, (rp.k + kFastW - 1) / kFastW);
    if (lane == 0) {
      sm.red_sum[w] = wsum;
      sm.red_tau[w] = tau_w;
    }
    if (t == 0) sm.cand_n[(it + 1) & 1] = 0;
    __syncthreads();
    unsigned long long S = 0;
    float tau = f_inf();
#pragma unroll
    for (int i = 0; i < kFastW; ++i) {
      S += sm.red_sum[i];
      tau = fminf(tau, sm.red_tau[i]);
    }
    const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
    // ---- candidates: every element >= tau (at least k of them) ----
    unsigned *cn = &sm.cand_n[it & 1];
#pragma unroll
    for (int m = 0; m < PP; ++m)
#pragma unroll
      for (int j = 0; j < JJ; ++j) {
        const int i = t + NT * m + kPartials * j;
        if (i < V && q[m][j] >= tau) {
          const unsigned pos = atomicAdd(cn, 1u);
          if (pos < kCandCap) sm.cand[pos] = cand_key(q[m][j], (uint32_t)i);
        }
      }
    __syncthreads();
    unsigned C = *cn;
    if (C > kSortMax) {
      // Too many at the threshold (ties): the k-th largest key exactly, by
      // bisection on the 64-bit (value, id) key; then exactly the k keys above it.
      unsigned long long P = 0;
      for (int b = 63; b >= 0; --b) {
        const unsigned long long trial = P | (1ull << b);
        int c = 0;
#pragma unroll
        for (int m = 0; m < PP; ++m)
#pragma unroll
          for (int j = 0; j < JJ; ++j) {
            const int i = t + NT * m + kPartials * j;
            c += (i < V && cand_key(q[m][j], (uint32_t)i) >= trial) ? 1 : 0;
          }
        c = __reduce_add_sync(kFull, c);
        if (lane == 0) sm.red_cnt[b & 1][w] = c;
        __syncthreads();
        int tot = 0;
#pragma unroll
        for (int i = 0; i < kFastW; ++i) tot += sm.red_cnt[b & 1][i];
        if (tot >= rp.k) P = trial;
      }
      if (t == 0) *cn = 0;
      __syncthreads();
#pragma unroll
      for (int m = 0; m < PP; ++m)
#pragma unroll
        for (int j = 0; j < JJ; ++j) {
          const int i = t + NT * m + kPartials * j;
          if (i < V) {
            const unsigned long long key = cand_key(q[m][j], (uint32_t)i);
            if (key >= P) sm.cand[atomicAdd(cn, 1u)] = key;
          }
        }
      __syncthreads();
      C = (unsigned)rp.k;
    }
    if (w == 0) {
      warp_sort_any(sm.cand, (int)C, lane);
      sample_tail(a, row, sm.cand, sm.scr, rp.k, lse, rp.p, lane);
    }
  }
  if (failed) {
    // A bulk copy did not complete in time: record it, then wait (bounded) for
    // this CTA's copies still in flight before the shared memory goes away.
    if (t == 0) {
      atomicOr(a.error, 1);
      for (int i = it; i < it + stages; ++i) {
        if (blockIdx.x + i * (int)gridDim.x >= a.N) break;
        if (!mbar_wait_bounded(&sm.mbar[i % stages], (uint32_t)(i / stages) & 1u)) break;
      }
    }
  }
}

// ---- wide kernel ----

template <bool BF16>
__global__ void __launch_bounds__(kWideThreads) sample_wide_kernel(const KArgs a, int use_list,
                                                                    int kcap) {
  extern __shared__ unsigned long long keys[];  // [pow2 >= kcap] keys, then float scr[kcap]
  __shared__ float red_max[kWideWarps];
  __shared__ unsigned long long red_sum[kWideWarps];
  __shared__ int red_cnt[2][kWideWarps];
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
    for (int i = t; i < V; i += kWideThreads) m = max_nan(m, __fdiv_rn(load_x<BF16>(base, i), rp.T));
    const float wm = warp_max_nan(m);
    if (lane == 0) red_max[w] = wm;
    __syncthreads();
    float gmax = red_max[0];
#pragma unroll
    for (int i = 1; i < kWideWarps; ++i) gmax = max_nan(gmax, red_max[i]);
    if (!(fabsf(gmax) < f_inf())) {
      if (t == 0) flag_row(a, row, D3S_ROW_NONFINITE);
      __syncthreads();
      continue;
    }
    float s = 0.0f;
    for (int i = t; i < V; i += kWideThreads)
      s = __fadd_rn(s, exp_term(__fsub_rn(__fdiv_rn(load_x<BF16>(base, i), rp.T), gmax)));
    const unsigned long long wsum = warp_sum_fixed(__float2ull_rz(__fmul_rn(s, 0x1p46f)));
    if (lane == 0) red_sum[w] = wsum;
    __syncthreads();
    unsigned long long S = 0;
#pragma unroll
    for (int i = 0; i < kWideWarps; ++i) S += red_sum[i];
    const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
    unsigned long long P = 0;
    for (int b = 63; b >= 0; --b) {
      const unsigned long long trial = P | (1ull << b);
      int c = 0;
      for (int i = t; i < V; i += kWideThreads)
        c += cand_key(__fdiv_rn(load_x<BF16>(base, i), rp.T), (uint32_t)i) >= trial ? 1 : 0;
      c = __reduce_add_sync(kFull, c);
      if (lane == 0) red_cnt[b & 1][w] = c;
      __syncthreads();
      int tot = 0;
#pragma unroll
      for (int i = 0; i < kWideWarps; ++i) tot += red_cnt[b & 1][i];
      if (tot >= k) P = trial;
    }
    if (t == 0) gather_n = 0;
    __syncthreads();
    for (int i = t; i < V; i += kWideThreads) {
      const unsigned long long key = cand_key(__fdiv_rn(load_x<BF16>(base, i), rp.T), (uint32_t)i);
      if (key >= P) keys[atomicAdd(&gather_n, 1u)] = key;
    }
    for (int i = k + t; i < kp; i += kWideThreads) keys[i] = 0ull;
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= kp; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = t; i < (kp >> 1); i += kWideThreads) {
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

__global__ void math_kernel(int op, const float *x, float *y, int64_t n, float T) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    float r;
    switch (op) {
      case 0: r = exp_full(v); break;
      case 1: r = log_full(v); break;
      case 2: r = exp_term(v); break;
      default: r = div_rows(v, __frcp_rn(T), -T); break;
    }
    y[i] = r;
  }
}

// Counts x (every float bit pattern from lo, step `step`) whose div_rows(x, T)
// differs from the IEEE quotient, for x in div_rows' valid range.
__global__ void div_check_kernel(const float *Ts, int nT, uint64_t lo, uint64_t hi, uint64_t step,
                                 unsigned long long *bad, float *example) {
  const uint64_t n = (hi - lo + step - 1) / step;
  for (int ti = 0; ti < nT; ++ti) {
    const float T = Ts[ti];
    const float rT = __frcp_rn(T), mT = -T;
    unsigned long long local = 0;
    for (uint64_t f = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n;
         f += (uint64_t)gridDim.x * blockDim.x) {
      const float x = __uint_as_float((uint32_t)(lo + f * step));
      const float ax = fabsf(x);
      if (!(ax >= 0x1p-60f && ax <= 0x1p60f)) continue;
      const float q = div_rows(x, rT, mT), ref = __fdiv_rn(x, T);
      if (__float_as_uint(q) != __float_as_uint(ref)) {
        ++local;
        example[0] = x;
        example[1] = T;
      }
    }
    if (local) atomicAdd(bad, local);
  }
}

// ---- launch helpers ----

using FastFn = void (*)(const KArgs, int, int);

template <bool BF16>
FastFn pick_fast(int J) {
  switch (J) {
    case 1: return sample_fast_kernel<1, BF16>;
    case 2: return sample_fast_kernel<2, BF16>;
    case 4: return sample_fast_kernel<4, BF16>;
    case 8: return sample_fast_kernel<8, BF16>;
    case 12: return sample_fast_kernel<12, BF16>;
    case 16: return sample_fast_kernel<16, BF16>;
    case 17: return sample_fast_kernel<17, BF16>;
    case 24: return sample_fast_kernel<24, BF16>;
    case 32: return sample_fast_kernel<32, BF16>;
    default: return nullptr;
  }
}

int pick_J(int V) {
  const int need = (V + kPartials - 1) / kPartials;
  static const int Js[] = {1, 2, 4, 8, 12, 16, 17, 24, 32};
  for (int J : Js)
    if (J >= need) return J;
  return 0;
}

int device_sms() {
  static thread_local int cached_dev = -1, cached_sms = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cached_dev != dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    cached_dev = dev;
    cached_sms = sms;
  }
  return cached_sms;
}

int occupancy(const void *fn, int threads, size_t smem) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, threads, smem) != cudaSuccess)
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
  int grid = sms * occupancy((const void *)fn, kWideThreads, smem);
  if (!use_list) grid = std::min(grid, a.N);
  if (grid < 1) grid = 1;
  fn<<<grid, kWideThreads, smem, st>>>(a, use_list, kcap);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

template <bool BF16>
int launch_fast(const KArgs &a, int J, cudaStream_t st) {
  constexpr int esz = BF16 ? 2 : 4;
  const int span = ((a.V * esz + 15) / 16) * 16 + 16;
  int stages = BF16 ? 3 : 2;
  while (stages > 2 && (size_t)stages * span > 64 * 1024) --stages;
  const size_t smem = (size_t)stages * span;
  FastFn fn = pick_fast<BF16>(J);
  if (!fn) return D3S_ERR_ARG;
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return D3S_ERR_CUDA;
  const int sms = device_sms();
  if (sms <= 0) return D3S_ERR_CUDA;
  const int grid = std::max(1, std::min(a.N, sms * occupancy((const void *)fn, kFastThreads, smem)));
  fn<<<grid, kFastThreads, smem, st>>>(a, stages, span);
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
  const int rc = launch_fast<BF16>(a, J, st);
  if (rc != D3S_OK) return rc;
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

int launch_math(int op, const float *x, float *y, int64_t n, float T, cudaStream_t st) {
  if (n == 0) return D3S_OK;
  const int sms = device_sms();
  const int grid = (int)std::min<int64_t>((n + 255) / 256, (int64_t)std::max(sms, 1) * 16);
  math_kernel<<<grid, 256, 0, st>>>(op, x, y, n, T);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

int launch_div_check(const float *Ts, int nT, uint64_t lo, uint64_t hi, uint64_t step,
                     unsigned long long *bad, float *example, cudaStream_t st) {
  const int sms = device_sms();
  div_check_kernel<<<std::max(sms, 1) * 8, 256, 0, st>>>(Ts, nT, lo, hi, step, bad, example);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

}  // namespace d3s

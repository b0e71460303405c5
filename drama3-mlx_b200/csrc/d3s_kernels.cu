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
#include <atomic>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

namespace d3s {
namespace {

constexpr unsigned kFull = 0xffffffffu;
constexpr int kPartials = 256;
constexpr int kCandCap = 256;    // fast kernel candidate buffer
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

// The logits row a (virtual) row reads: draws that share logits (the main and
// the retry draw of a frame) are rows r and r + row_period of one request.
__device__ __forceinline__ int64_t phys_row(const KArgs &a, int row) {
  return a.row_period > 0 ? (int64_t)(row % a.row_period) : (int64_t)row;
}

template <bool BF16>
__device__ __forceinline__ const void *row_base(const KArgs &a, int row) {
  const int64_t off = phys_row(a, row) * a.ld;
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
  if (a.noise == D3S_NOISE_SEEDS) return seed_subkey(a.seeds[row]);
  if (a.noise == D3S_NOISE_KEYS) return a.keys[(int64_t)row * a.ld_keys];
  return a.key;
}

// u for (row, rank r): the word of the [N, k] (one key) or [1, k] (per-row seed)
// uniform array that sample_top_k_top_p / d3_sample would draw.
__device__ __forceinline__ float row_uniform(const KArgs &a, int row, int k, int r, uint2 key) {
  if (a.noise == D3S_NOISE_GIVEN) return a.u[(int64_t)row * a.ld_u + r];
  const bool one = a.noise == D3S_NOISE_KEY;
  const uint64_t n = one ? (uint64_t)a.N * (uint64_t)k : (uint64_t)k;
  const uint64_t f = one ? (uint64_t)row * (uint64_t)k + (uint64_t)r : (uint64_t)r;
  return bits_to_uniform(bits_word1(key, n, f));
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
// Rows on which div_rows gives every quotient that can matter exactly. The
// reciprocal step is exact for |x| in [2^-100, 2^60] with T in [2^-17, 2^20]
// (checked over every float x for a set of T by the tests). Smaller nonzero
// |x| may be off by an ulp, but with |max| >= 2^-40 their term is exp(-max)
// (|q| < 2^-83 is below half an ulp of max) and with |tau| >= 2^-60 they are
// never a boundary candidate; candidate keys themselves use the IEEE divide.
__device__ __forceinline__ bool div_rows_ok(float xmin, float xmax, float T, float gmax,
                                            float tau) {
  return fmaxf(fabsf(xmin), fabsf(xmax)) <= 0x1p60f && T >= 0x1p-17f && T <= 0x1p20f &&
         fabsf(gmax) >= 0x1p-40f && fabsf(tau) >= 0x1p-60f;
}

// ---- warp helpers ----

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

// How the tail reads the ranked candidates. Ranks64: the top k as 64-bit
// (value, id) keys. Ranks32: the top k as 32-bit value keys (okey of q) in
// rank order; the id of a rank is looked up among the row's candidates by the
// whole warp (ties in value keep their ids in increasing order, so the rank
// r that is the m-th of the ranks holding its key is the m-th smallest id of the
// candidates with that key).
struct Ranks64 {
  static constexpr bool kPerRankIds = true;
  const unsigned long long *s;
  __device__ __forceinline__ float value(int r) const { return cand_value(s[r]); }
  __device__ __forceinline__ int32_t id(int r, int) const { return cand_id(s[r]); }
};

struct Ranks32 {
  static constexpr bool kPerRankIds = false;
  const uint32_t *s;                // top k, rank order
  const uint32_t *keys;             // every candidate's key, list order
  int C;
  const unsigned long long *cs;     // raw candidates: the first kStageCands
  const unsigned long long *slab;   // all of them
  int staged;                       // how many cs holds
  __device__ __forceinline__ float value(int r) const { return okey_to_float(s[r]); }
  // called by every lane of the warp
  __device__ __forceinline__ int32_t id(int r, int lane) const {
    const uint32_t K = s[r];
    int m = 0;  // ranks before r with the same key (they sit just before it)
    for (int b = 0; b < r; b += 32) {
      const int q = b + lane;
      m += __popc(__ballot_sync(kFull, q < r && s[q] == K));
    }
    unsigned total = 0u;
    int first = -1;
    for (int b = 0; b < C; b += 32) {
      const int e = b + lane;
      const unsigned bal = __ballot_sync(kFull, e < C && keys[e] == K);
      if (first < 0 && bal) first = b + __ffs(bal) - 1;
      total += __popc(bal);
    }
    auto raw_id = [&](int e) {
      return (uint32_t)(e < staged ? cs[e] : slab[e]);
    };
    if (total == 1u) return (int32_t)raw_id(first);
    // ties: the m-th smallest id of the candidates with key K
    uint32_t taken = 0u, id = 0u;
    for (int t = 0; t <= m; ++t) {
      uint32_t mine = 0xFFFFFFFFu;
      for (int e = lane; e < C; e += 32)
        if (keys[e] == K) {
          const uint32_t v = raw_id(e);
          if ((t == 0 || v > taken) && v < mine) mine = v;
        }
      id = __reduce_min_sync(kFull, mine);
      taken = id;
    }
    return (int32_t)id;
  }
};

// The serial end of a row, run by one warp: R gives the top k in rank order
// (values and ids), scr (>= k + 4 floats, 16-byte aligned) is scratch, key draws
// the row's uniforms. Inclusive cumsum of exp(v - lse) in rank order
// (src/sampling.c:39, :126-127), drop when cum > top_p at rank > 0 (:40-43,
// :128), softmax over the survivors with a 1/sum multiply (:44, :129-134), race
// p / -log(1 - u) where the first strictly greater score wins (:45-47,
// :135-137). The two sequential sums run identically on every lane (broadcast
// reads, four ranks per load). Survivors are a prefix of the ranks and every
// survivor's score is positive unless its noise is -0, so the dropped ranks
// (p = 0, score 0 or NaN) are drawn only when no survivor scored above 0.
//
// lse is known to lie in [lse_lo, lse_hi] (equal bounds: lse is exact). With
// an interval, the cut is found with lse_hi and then certified for every lse in
// it: terms under a smaller lse are larger (exp's relative error, below
// 2^-23.6, bounds how far a rounded exp can break that order), so the cut rank
// must still pass top_p under lse_hi less a rounding margin, and the rank before
// it must stay at or below top_p under lse_lo plus that margin. Returns false,
// having written nothing, when the cut cannot be certified; the caller then
// computes the exact lse and calls again.
template <class Ranks>
__device__ __forceinline__ bool sample_tail_r(const KArgs &a, int row, uint2 key, const Ranks &R,
                                              float *scr, int k, float lse_lo, float lse_hi,
                                              float top_p, int lane) {
  const bool exact = __float_as_uint(lse_lo) == __float_as_uint(lse_hi);
  // e_r = exp(v_r - lse_hi) (exact: under the exact lse), zero past k up to the
  // next multiple of 4 (adding +0 leaves every running sum unchanged)
  const int k4 = (k + 3) & ~3;
  float lsum = 0.0f;
  for (int r = lane; r < k4; r += 32) {
    const float e = r < k ? exp_nonpos(__fsub_rn(R.value(r), lse_hi)) : 0.0f;
    scr[r] = e;
    lsum = __fadd_rn(lsum, e);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) lsum = __fadd_rn(lsum, __shfl_xor_sync(kFull, lsum, o));
  __syncwarp();
  // Under an interval, a term under lse_lo is at most F times the same rank's
  // term under lse_hi plus 0.75 2^-24: F covers exp(lse_hi - lse_lo) and exp's
  // error at both ends; the arguments' roundings (|y| 2^-24 each, y = v - lse
  // <= 0) move a term e^y by at most 2 |y| e^y 2^-24 <= (2 / e) 2^-24. A wide
  // interval (above 2^-14) gets no bound: F = inf, and any cut it needs is left
  // to the exact sum.
  float F = 1.0f;
  if (!exact) {
    const float d = __fsub_ru(lse_hi, lse_lo);
    F = d <= 0x1p-14f ? __fadd_ru(1.0f, __fadd_ru(__fmul_ru(d, 1.0001f), 0x1p-22f)) : f_inf();
  }
  // Any-order sum of the k terms: a sequential sum of nonnegative terms differs
  // from it by at most 2 (k - 1) 2^-24 relative (< 3.1e-5 for k <= 256). When
  // even that bound stays <= top_p, no prefix sum can exceed top_p: nothing is
  // cut. (Under an interval, for the terms under lse_lo, the largest.)
  const float lsum_lo = exact ? lsum : __fmaf_ru(F, lsum, (float)k * 0x1p-24f);
  int kept = k;
  if (!(__fmul_ru(lsum_lo, 1.0001f) <= top_p)) {
    // cum_r = e_0 + ... + e_r in rank order; the first r > 0 with cum_r > top_p
    // is the cut. Four ranks per step: the running sums, then one test. before
    // is the sum of ranks 0 .. kept - 1 (all k when nothing is cut).
    float cum = 0.0f, cut = 0.0f, before = 0.0f;
    bool found = false;
    for (int r0 = 0; r0 < k; r0 += 4) {
      const float4 e4 = *reinterpret_cast<const float4 *>(scr + r0);
      const float c0 = __fadd_rn(cum, e4.x), c1 = __fadd_rn(c0, e4.y);
      const float c2 = __fadd_rn(c1, e4.z), c3 = __fadd_rn(c2, e4.w);
      const bool h0 = r0 > 0 && c0 > top_p;  // rank 0 is never dropped
      if (h0 || c1 > top_p || c2 > top_p || c3 > top_p) {
        kept = h0 ? r0 : (c1 > top_p ? r0 + 1 : (c2 > top_p ? r0 + 2 : r0 + 3));
        cut = h0 ? c0 : (c1 > top_p ? c1 : (c2 > top_p ? c2 : c3));
        before = h0 ? cum : (c1 > top_p ? c0 : (c2 > top_p ? c1 : c2));
        found = true;
        break;
      }
      cum = c3;
    }
    if (!found) before = cum;
    if (!exact) {
      // margin: two sequential sums of <= kept + 1 terms (kept 2^-24 each),
      // exp's order error (2.9 2^-24 for its error below 2^-23.5) and the
      // product's rounding; the sum under lse_lo, bounded from the one under
      // lse_hi, takes two more sequential-sum errors
      const float mu = __fmul_rn((float)(2 * kept + 6), 0x1p-24f);
      if (kept < k && !(__fmul_rn(cut, 1.0f - mu) > top_p)) return false;
      const float before_lo = __fmaf_ru(F, before, (float)kept * 0x1.8p-25f);
      const float mu2 = __fmul_rn((float)(4 * kept + 8), 0x1p-24f);
      if (kept >= 2 && !(__fmul_ru(before_lo, 1.0f + mu2) <= top_p)) return false;
    }
  }
  __syncwarp();
  const float top = R.value(0);
  const int kept4 = (kept + 3) & ~3;
  for (int r = lane; r < kept4; r += 32)
    scr[r] = r < kept ? exp_nonpos(__fsub_rn(R.value(r), top)) : 0.0f;
  __syncwarp();
  float sum = 0.0f;
  for (int r0 = 0; r0 < kept; r0 += 4) {
    const float4 e4 = *reinterpret_cast<const float4 *>(scr + r0);
    sum = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(sum, e4.x), e4.y), e4.z), e4.w);
  }
  const float inv = __fdiv_rn(1.0f, sum);
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
  if constexpr (Ranks::kPerRankIds) {
    if (a.topk_ids)
      for (int r = lane; r < k; r += 32) a.topk_ids[(int64_t)row * a.ld_out + r] = R.id(r, lane);
  }
  const unsigned choice = __reduce_min_sync(kFull, best == wbest ? (unsigned)best_r : 0xffffffffu);
  const int32_t chosen = R.id((int)choice, lane);
  if (lane == 0) {
    a.ids[row] = chosen;
    if (a.status) a.status[row] = D3S_ROW_OK;
    if (a.kept) a.kept[row] = kept;
  }
  return true;
}

__device__ __forceinline__ bool sample_tail(const KArgs &a, int row, uint2 key,
                                            const unsigned long long *sorted, float *scr, int k,
                                            float lse_lo, float lse_hi, float top_p, int lane) {
  return sample_tail_r(a, row, key, Ranks64{sorted}, scr, k, lse_lo, lse_hi, top_p, lane);
}

// Sum over the warp of each lane's fixed-point total (< 2^55): three 21/21/22-bit
// pieces, each summed exactly by a 32-bit redux.
__device__ __forceinline__ unsigned long long warp_sum_u64(unsigned long long v) {
  const unsigned p0 = __reduce_add_sync(kFull, (unsigned)(v & 0x1FFFFFu));
  const unsigned p1 = __reduce_add_sync(kFull, (unsigned)((v >> 21) & 0x1FFFFFu));
  const unsigned p2 = __reduce_add_sync(kFull, (unsigned)(v >> 42));
  return (unsigned long long)p0 + ((unsigned long long)p1 << 21) + ((unsigned long long)p2 << 42);
}

// The lse bracket of one row from its header, computed by one thread. For a
// row of the approximate stats, S (2^-46 fixed point) is the SFU's exp2 of
// RN(x c + g) with c = RN(log2(e) / T) and g = RN(-xmax c). With G = |max x / T|,
// first-order error analysis bounds |S_exact - S| / S by
// 2^-24 (3 G + 5 ln V + n_p + L + 1) + e_exp + e_ex2: the quotients' and
// differences' roundings (2G + 2 ln V for the exact sum, G + 3 ln V for the
// approximate one, ln V bounding the entropy-weighted |x/T - max|), sequential
// sums of n_p (the exact partials) and L (the approximate accumulators) terms,
// exp's relative error (below 2^-23.5) and ex2.approx's (below 2^-22.5; both
// checked by the tests). approx_bound_c0 (c0) rounds the row-independent part
// up; the row's part is 3.1 G 2^-24. The exact lse = RN(gmax + log(RN(S_exact)
// 2^-46)) is then bracketed by the same expression at the bracket's ends: RN
// and log are monotone there (log is checked over every float in [1, 16384) by
// the tests), and the exact S is at least 2^46. Rows of the exact stats get
// their exact lse twice.
__device__ __forceinline__ void row_lse(const RowHead &H, float c0, float &lse_lo, float &lse_hi) {
  unsigned long long S = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) S += H.sum[i];
  if (H.approx) {
    const float delta = __fmaf_ru(0x1.8cccccp-23f, fabsf(H.gmax), c0);
    const float lo = __fmul_rd(__fmul_rd(__ull2float_rd(S), __fsub_rd(1.0f, delta)), 0x1p-46f);
    const float hi = __fmul_ru(__fmul_ru(__ull2float_ru(S), __fadd_ru(1.0f, delta)), 0x1p-46f);
    lse_lo = __fadd_rn(H.gmax, log_full(fmaxf(lo, 1.0f)));
    lse_hi = __fadd_rn(H.gmax, log_full(hi));
  } else {
    lse_lo = __fadd_rn(H.gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
    lse_hi = lse_lo;
  }
}

// Per-row parameters as stored (read one row ahead of use).
struct RawP {
  float T, p;
  int tk;
  unsigned long long seed;
};

__device__ __forceinline__ RawP load_raw(const KArgs &a, int row) {
  RawP r;
  r.T = a.T_rows ? a.T_rows[row] : a.T;
  r.p = a.p_rows ? a.p_rows[row] : a.top_p;
  r.tk = a.k_rows ? a.k_rows[row] : a.top_k;
  r.seed = 0ull;
  if (a.noise == D3S_NOISE_SEEDS) {
    r.seed = a.seeds[row];
  } else if (a.noise == D3S_NOISE_KEYS) {
    const uint2 k = a.keys[(int64_t)row * a.ld_keys];
    r.seed = ((unsigned long long)k.y << 32) | k.x;
  }
  return r;
}

// The key that draws the row's uniforms, from its stored parameters (called by
// every lane of a warp).
__device__ __forceinline__ uint2 raw_key(const KArgs &a, const RawP &r, int lane) {
  if (a.noise == D3S_NOISE_SEEDS) return seed_subkey_warp(r.seed, lane);
  if (a.noise == D3S_NOISE_KEYS) return make_uint2((unsigned)r.seed, (unsigned)(r.seed >> 32));
  return a.key;
}

__device__ __forceinline__ int resolve(const KArgs &a, const RawP &r, RowP &rp) {
  if (r.tk < 1 || r.T != r.T) return D3S_ROW_BADPARAM;
  const int k = min(r.tk, a.V);
  if (k > D3S_MAX_K) return D3S_ROW_BADPARAM;
  rp.T = r.T < kMinTemperature ? kMinTemperature : r.T;
  rp.p = r.p;
  rp.k = k;
  return D3S_ROW_OK;
}

// ---- stats kernel (K1): the streaming pass over the rows ----

constexpr int kStatMinBlocks = 6;

struct alignas(16) StatSmem {
  uint64_t mbar[kMaxStages];
  unsigned stage_done[kMaxStages];  // warps finished with the stage's row
  unsigned cand_n[kMaxStages];      // candidates of the stage's row so far
  float red_max[2][kFastW];         // by row parity, so no barrier is needed between rows
  float red_min[2][kFastW];
  float red_tau[2][kFastW];
};

// L2 policy for the logits stream: read once, so evict it first and keep the
// row records the select kernel reads next.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// Issue the bulk copy of row `row` into a stage: the 16-byte-aligned span that
// covers the row (a copy must start and end on 16-byte boundaries).
template <int ESZ>
__device__ __forceinline__ void issue_row(const KArgs &a, int row, unsigned char *stage,
                                          uint64_t *bar, uint64_t pol) {
  const uintptr_t start = (uintptr_t)a.logits + (uintptr_t)phys_row(a, row) * (uintptr_t)a.ld * ESZ;
  const uintptr_t lo = start & ~(uintptr_t)15;
  const uintptr_t hi = (start + (uintptr_t)a.V * ESZ + 15) & ~(uintptr_t)15;
  const uint32_t bytes = (uint32_t)(hi - lo);
  mbar_expect_tx(bar, bytes);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(stage)),
      "l"(lo), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
      : "memory");
}

__device__ __forceinline__ void defer_row(const KArgs &a, int row) {
  const unsigned pos = atomicAdd(a.deferred_n, 1u);
  if (pos < (unsigned long long)a.deferred_cap)
    a.deferred[pos] = row;
  else
    flag_row(a, row, D3S_ROW_BADPARAM);
}
// Hand a row whose top-p cut the approximate sum could not certify to the wide
// kernel, which recomputes the exact full-row sum with a whole CTA and then
// samples the row from its stored candidates. Stored as -(row + 1).
__device__ __forceinline__ void defer_row_exact_sum(const KArgs &a, int row) {
  const unsigned pos = atomicAdd(a.deferred_n, 1u);
  if (pos < (unsigned long long)a.deferred_cap)
    a.deferred[pos] = -(row + 1);
  else
    flag_row(a, row, D3S_ROW_BADPARAM);
}

// A candidate as the stats kernel stores it: x's bits above its id. The select
// kernel turns it into the (value, id) key of q = x / T (IEEE divide).
__device__ __forceinline__ unsigned long long raw_cand(float x, uint32_t id) {
  return ((unsigned long long)__float_as_uint(x) << 32) | id;
}
__device__ __forceinline__ unsigned long long raw_to_key(unsigned long long r, float T) {
  return cand_key(__fdiv_rn(__uint_as_float((uint32_t)(r >> 32)), T), (uint32_t)r);
}

// 32-bit mask of the predicate x >= y (NaN compares false): all ones or zero.
__device__ __forceinline__ uint32_t ge_mask(float x, float y) {
  uint32_t m;
  asm("set.ge.u32.f32 %0, %1, %2;" : "=r"(m) : "f"(x), "f"(y));
  return m;
}

// The rest of a row once its max and threshold are known: q = x / T in place
// (per-row reciprocal when the range allows, IEEE divide otherwise), the two
// packed partial sums of exp(q - max) in fixed point, and every element >= tau
// written as a raw (x, id) candidate into the row's list: one bit per element in two
// 32-bit words (x: partial t, y: partial t + 128; bit j = column j), one warp
// prefix sum, then a short loop over the set bits that re-reads x from the
// stage. q2[j] holds elements t + 256 j (x) and
// t + 128 + 256 j (y) as one register pair, the operand of the packed ops.
template <int JJ, bool CLAMP, bool EXACT>
__device__ __forceinline__ void sum_and_mask(const float2 (&q2)[JJ], float gmax, float tau, int t,
                                             int V, float2 &s2, uint32_t &bx, uint32_t &by) {
  constexpr int NT = kFastThreads;
  static_assert(JJ <= 32, "one mask word per partial");
  const float2 mg = make_float2(-gmax, -gmax);
#pragma unroll
  for (int j = 0; j < JJ; ++j) {
    float2 e = exp_term2<CLAMP>(__fadd2_rn(q2[j], mg));
    uint32_t mx = ge_mask(q2[j].x, tau), my = ge_mask(q2[j].y, tau);
    if (!(EXACT && j < JJ - 1)) {  // a column that can run past V: padding adds exactly 0
      if (t + kPartials * j >= V) {
        e.x = 0.0f;
        mx = 0u;
      }
      if (t + NT + kPartials * j >= V) {
        e.y = 0.0f;
        my = 0u;
      }
    }
    s2 = __fadd2_rn(s2, e);
    bx |= mx & (1u << j);
    by |= my & (1u << j);
  }
}

// The end of a row's stats once its sums and candidate bits are known: the
// warp's fixed-point sum into the header, the candidates (every set bit j of bx
// / by: element t + 256 j / t + 128 + 256 j) as raw (x, id) pairs into the
// row's list at positions from one warp scan and one shared atomic per warp.
template <bool BF16>
__device__ __forceinline__ void stats_finish(RowHead &H, RowCands &Cs, unsigned *cand_n,
                                             const unsigned char *rb, float2 s2, uint32_t bx,
                                             uint32_t by, float gmax, int approx, int t, int lane,
                                             int w) {
  constexpr int NT = kFastThreads;
  const unsigned long long wsum = warp_sum_fixed(__float2ull_rz(__fmul_rn(s2.x, 0x1p46f)) +
                                                 __float2ull_rz(__fmul_rn(s2.y, 0x1p46f)));
  const int mine = __popc(bx) + __popc(by);
  int incl = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int o = __shfl_up_sync(kFull, incl, d);
    if (lane >= d) incl += o;
  }
  // this warp's span of the row's list: one shared-memory atomic per warp
  unsigned base = 0;
  if (lane == 31 && incl > 0) base = atomicAdd(cand_n, (unsigned)incl);
  base = __shfl_sync(kFull, base, 31);
  int pos = (int)base + incl - mine;
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    uint32_t bits = m ? by : bx;
    while (bits) {
      const int j = __ffs(bits) - 1;
      bits &= bits - 1;
      const int i = t + NT * m + kPartials * j;
      // the raw candidate (x, id); the select kernel divides and keys it
      if (pos < kCandCap) Cs.cand[pos] = raw_cand(lds_x<BF16>(rb, i), (uint32_t)i);
      ++pos;
    }
  }
  if (lane == 31) H.sum[w] = wsum;
  if (t == 0) {
    H.gmax = gmax;
    H.done = 0;
    H.approx = approx;
  }
}

template <int JJ, bool BF16, bool EXACT>
__device__ __forceinline__ void stats_row(const KArgs &a, RowHead &H, RowCands &Cs,
                                          unsigned *cand_n, const unsigned char *rb,
                                          float2 (&q2)[JJ], float T, float rT, float gmax,
                                          float tau, float xminq, bool fast, int t, int lane, int w) {
  const int V = a.V;
  if (fast) {
    const float2 rT2 = make_float2(rT, rT), mT2 = make_float2(-T, -T);
#pragma unroll
    for (int j = 0; j < JJ; ++j) q2[j] = div_rows2(q2[j], rT2, mT2);
  } else {
#pragma unroll
    for (int j = 0; j < JJ; ++j) q2[j] = make_float2(__fdiv_rn(q2[j].x, T), __fdiv_rn(q2[j].y, T));
  }
  float2 s2 = make_float2(0.0f, 0.0f);
  uint32_t bx = 0u, by = 0u;
  // every term's d >= the row's smallest d: when that is >= -86 the floor is a no-op
  if (__fsub_rn(xminq, gmax) >= kTermFloor)
    sum_and_mask<JJ, false, EXACT>(q2, gmax, tau, t, V, s2, bx, by);
  else
    sum_and_mask<JJ, true, EXACT>(q2, gmax, tau, t, V, s2, bx, by);
  stats_finish<BF16>(H, Cs, cand_n, rb, s2, bx, by, gmax, 0, t, lane, w);
}

// The approximate row stats: each term 2^(x c + g) by the SFU (c = RN(log2(e)
// / T), g = RN(-xmax c)), no division, no floor; candidates are the x above
// tau_lo, a threshold just under the x-domain threshold, low enough that no x
// at or below it can have a quotient reaching RN(taux / T) (so every element of
// the top k is a candidate: the select step divides and keys them exactly).
// The candidate bit of column j is the sign of tau_lo - x, shifted in from
// the highest column down. Padding (-inf) adds +0 and sets no bit.
template <int JJ, bool BF16>
__device__ __forceinline__ void stats_row_approx(RowHead &H, RowCands &Cs, unsigned *cand_n,
                                                 const unsigned char *rb, const float2 (&x2)[JJ],
                                                 float c, float g, float tau_lo, float gmax,
                                                 int t, int lane, int w) {
  const float2 c2 = make_float2(c, c), g2 = make_float2(g, g);
  const float2 tl2 = make_float2(tau_lo, tau_lo), m1 = make_float2(-1.0f, -1.0f);
  float2 s2[2] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f)};  // even / odd columns
  uint32_t bx = 0u, by = 0u;
#pragma unroll
  for (int j = JJ - 1; j >= 0; --j) {
    const float2 u = __ffma2_rn(x2[j], c2, g2);
    s2[j & 1] = __fadd2_rn(s2[j & 1], make_float2(ex2_approx(u.x), ex2_approx(u.y)));
    const float2 d = __ffma2_rn(x2[j], m1, tl2);
    bx = __funnelshift_l(__float_as_uint(d.x), bx, 1);
    by = __funnelshift_l(__float_as_uint(d.y), by, 1);
  }
  stats_finish<BF16>(H, Cs, cand_n, rb, __fadd2_rn(s2[0], s2[1]), bx, by, gmax, 1, t, lane, w);
}

// Rows the approximate stats take: k <= 128 (the tail's scratch holds both
// term arrays), T in [2^-17, 2^20] and |xmax| <= 2^60 (x c + g cannot overflow
// near the max), |taux| >= 2^-60 (quotients near the threshold are normal, so
// the 2^-21 step below taux clears every tie).
constexpr int kApproxMaxK = 128;
__device__ __forceinline__ bool approx_row_ok(const RowP &rp, float xmax, float taux) {
  return rp.k <= kApproxMaxK && rp.T >= 0x1p-17f && rp.T <= 0x1p20f && fabsf(xmax) <= 0x1p60f &&
         fabsf(taux) >= 0x1p-60f;
}

// A lower bound of the r-th largest of the warp's 32 values (1 <= r <= 32): r
// rounds of removing every copy of the current maximum (a tie removed at once
// counts once, which can only lower the result). Every lane at or above the
// result holds a value at least that large, and at least r lanes do.
__device__ __forceinline__ float warp_rth_redux(float v, int r) {
  float m;
  for (int it = 0;; ++it) {
    m = warp_max(v);
    if (it + 1 >= r) break;
    v = v == m ? -f_inf() : v;
  }
  return m;
}

// The r-th largest of the warp's 32 lane maxima (r <= 32), by a bitonic sort.
__device__ __forceinline__ float warp_rth_of32(float v, int r, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const float o = __shfl_xor_sync(kFull, v, stride);
      const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0);
      v = keep_max ? fmaxf(v, o) : fminf(v, o);
    }
  return __shfl_sync(kFull, v, r - 1);
}

// Per row: x from the stage into registers, max / |x| range / per-warp
// candidate threshold, one barrier; then stats_row; the last warp to finish
// with a stage refills it with the row `stages` ahead.
// EXACT: JJ == ceil(V / 256), so only the last column can run past V.
// Declared here, defined with the select kernel.
template <int S>
__device__ __forceinline__ void sort_cands(const unsigned long long *cs, const RowCands &Cs,
                                           int C, int k, float T, unsigned long long *sk,
                                           int lane);
__device__ __forceinline__ void select_cands(const RowCands &Cs, int C, int k, float T,
                                             unsigned long long *sk, int lane);

// The select kernel's work on one row whose record is complete: the row's
// lse, its subkey, the top k of its candidates in rank order in sk, the tail.
__device__ __forceinline__ bool select_row(const KArgs &a, int row, int C,
                                           const unsigned long long *cs, const RowCands &Cs,
                                           uint2 key, const RowP &rp, float lse_lo, float lse_hi,
                                           unsigned long long *sk, float *scr, int lane);

// APPROX: rows that approx_row_ok accepts take stats_row_approx and are marked
// approximate in their header; the others (and every row when APPROX is off)
// take the exact stats_row. APPROX kernels need a.finite == nullptr (no row min).
template <int JJ, bool BF16, bool EXACT, bool SELECT, bool APPROX>
__global__ void __launch_bounds__(kFastThreads, kStatMinBlocks)
    sample_stats_kernel(const KArgs a, RowHead *heads, RowCands *cands, int stages, int span) {
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ StatSmem sm;
  constexpr int PP = kFastPP;
  constexpr int NT = kFastThreads;
  constexpr int ESZ = BF16 ? 2 : 4;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int V = a.V;
  const uint64_t pol = evict_first_policy();
  if (t == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&sm.mbar[s], 1);
      sm.stage_done[s] = 0;
      sm.cand_n[s] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();
  const bool direct = SELECT && a.direct;
  if (t == 0 && !direct)
    for (int s = 0; s < stages; ++s) {
      const int r = blockIdx.x + s * gridDim.x;
      if (r < a.N) issue_row<ESZ>(a, r, dsm + (size_t)s * span, &sm.mbar[s], pol);
    }
  if (direct && (int)blockIdx.x < a.N) {
    // the row lives in host memory mapped into the device: the CTA's threads
    // copy its 16-byte-aligned span into the stage, each 16-byte load fetched
    // anew from the host (ld.global.cv)
    const uintptr_t start =
        (uintptr_t)a.logits + (uintptr_t)phys_row(a, blockIdx.x) * (uintptr_t)a.ld * ESZ;
    const uintptr_t lo = start & ~(uintptr_t)15;
    const int chunks = (int)((((start + (uintptr_t)V * ESZ + 15) & ~(uintptr_t)15) - lo) / 16);
    for (int c = t; c < chunks; c += NT)
      reinterpret_cast<uint4 *>(dsm)[c] = __ldcv(reinterpret_cast<const uint4 *>(lo) + c);
    __syncthreads();
  }
  RawP nxt{};
  if (SELECT && (int)blockIdx.x < a.N) nxt = load_raw(a, blockIdx.x);
  // Persistent CTAs: each warp resolves the parameters of the CTA's next 32
  // rows at once, lane i those of the i-th, and shuffles them out per row.
  // (approximate kernels also take each row's RN(log2(e) / T) and RN(1 / T))
  float T32 = 1.0f, p32 = 1.0f, c32 = 1.0f, rT32 = 1.0f;
  int k32 = 1, st32 = D3S_ROW_BADPARAM;
  int it = 0;
  bool failed = false;
  for (;; ++it) {
    const int row = blockIdx.x + it * gridDim.x;
    if (row >= a.N) break;
    RowP rp;
    int pst;
    RawP cur{};
    if constexpr (SELECT) {
      cur = nxt;
      if (row + (int)gridDim.x < a.N) nxt = load_raw(a, row + gridDim.x);
      pst = resolve(a, cur, rp);
    } else {
      if ((it & 31) == 0) {
        const int r = row + lane * (int)gridDim.x;
        if (r < a.N) {
          RowP q{1.0f, 1.0f, 1};
          st32 = resolve(a, load_raw(a, r), q);
          T32 = q.T;
          p32 = q.p;
          k32 = q.k;
          if constexpr (APPROX) {
            c32 = __fdiv_rn(kL2E, q.T);
            rT32 = __frcp_rn(q.T);
          }
        }
      }
      const int src = it & 31;
      pst = __shfl_sync(kFull, st32, src);
      rp.T = __shfl_sync(kFull, T32, src);
      rp.p = __shfl_sync(kFull, p32, src);
      rp.k = __shfl_sync(kFull, k32, src);
    }
    const int s = it % stages, par = it & 1;
    const bool ok = direct || mbar_wait_bounded(&sm.mbar[s], (uint32_t)(it / stages) & 1u);
    const unsigned char *rb =
        dsm + (size_t)s * span +
        (((uintptr_t)a.logits + (uintptr_t)phys_row(a, row) * (uintptr_t)a.ld * ESZ) & 15);
    static_assert(PP == 2, "two partials per thread, one packed pair per column");
    float2 q2[JJ];
    float pm[PP] = {-f_inf(), -f_inf()};
    float pmn = f_inf();
#pragma unroll
    for (int j = 0; j < JJ; ++j) {
      const int i0 = t + kPartials * j, i1 = i0 + NT;
      const bool v0 = (EXACT && j < JJ - 1) || i0 < V;
      const bool v1 = (EXACT && j < JJ - 1) || i1 < V;
      const float x0 = v0 ? lds_x<BF16>(rb, i0) : -f_inf();  // padding: -inf
      const float x1 = v1 ? lds_x<BF16>(rb, i1) : -f_inf();
      q2[j] = make_float2(x0, x1);
      pm[0] = max_nan(pm[0], x0);
      pm[1] = max_nan(pm[1], x1);
      if (!APPROX) {
        if (v0) pmn = fminf(pmn, x0);
        if (v1) pmn = fminf(pmn, x1);
      }
    }
    {
      const float lm = max_nan(pm[0], pm[PP - 1]);
      const float wm = warp_max_nan(lm);
      const float wi = APPROX ? 0.0f : -warp_max(-pmn);
      // candidate threshold in x: the ceil(k/4)-th largest lane maximum of this
      // warp (each of those lanes holds an element at least that large); x / T
      // is monotone, so the threshold in q is RN(min over warps / T)
      float tw = -f_inf();
      if (pst == D3S_ROW_OK && rp.k <= kFastMaxK && wm == wm) {
        const int r = (rp.k + kFastW - 1) / kFastW;
        if (r <= 32) {
          tw = APPROX ? warp_rth_redux(lm, r) : warp_rth_of32(lm, r, lane);
        } else {
          float v2[PP];
#pragma unroll
          for (int m = 0; m < PP; ++m) v2[m] = pm[m];
          tw = warp_rth_largest<PP>(v2, r);
        }
      }
      if (lane == 0) {
        sm.red_max[par][w] = wm;
        sm.red_min[par][w] = wi;
        sm.red_tau[par][w] = tw;
      }
    }
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    if (!APPROX && a.finite && t == 0) {  // every logit finite: no NaN, and the max and min are finite
      float fx = sm.red_max[par][0], fn = sm.red_min[par][0];
#pragma unroll
      for (int i = 1; i < kFastW; ++i) {
        fx = max_nan(fx, sm.red_max[par][i]);
        fn = fminf(fn, sm.red_min[par][i]);
      }
      a.finite[row] = (fabsf(fx) < f_inf() && fabsf(fn) < f_inf()) ? 1 : 0;
    }
    RowHead &H = heads[row];
    if (pst == D3S_ROW_OK && rp.k <= kFastMaxK) {
      float xmax = sm.red_max[par][0], xmin = sm.red_min[par][0], taux = sm.red_tau[par][0];
#pragma unroll
      for (int i = 1; i < kFastW; ++i) {
        xmax = max_nan(xmax, sm.red_max[par][i]);
        xmin = fminf(xmin, sm.red_min[par][i]);
        taux = fminf(taux, sm.red_tau[par][i]);
      }
      float gmax, tau, q2nd, rT;
      if constexpr (APPROX && !SELECT) {
        // log2(e) / T and 1 / T from the 32-row batch; max / T (= max(x / T), RN
        // being monotone) by the per-row reciprocal where that is the IEEE
        // quotient; the threshold's quotient only for rows of the exact path
        const int src = it & 31;
        q2nd = __shfl_sync(kFull, c32, src);
        rT = __shfl_sync(kFull, rT32, src);
        const float ax = fabsf(xmax);
        gmax = (ax >= 0x1p-100f && ax <= 0x1p60f && rp.T >= 0x1p-17f && rp.T <= 0x1p20f)
                   ? div_rows(xmax, rT, -rp.T)
                   : __fdiv_rn(xmax, rp.T);
        tau = 0.0f;
      } else {
        // the row's four quotients in one divide across lanes: max (max(x / T) =
        // RN(max(x) / T), RN being monotone), threshold, min (APPROX: log2(e) /
        // T), and 1 / T (= RN(1 / T))
        const float num =
            lane == 0 ? xmax : (lane == 1 ? taux : (lane == 2 ? (APPROX ? kL2E : xmin) : 1.0f));
        const float quo = __fdiv_rn(num, rp.T);
        gmax = __shfl_sync(kFull, quo, 0);
        tau = __shfl_sync(kFull, quo, 1);
        q2nd = __shfl_sync(kFull, quo, 2);
        rT = __shfl_sync(kFull, quo, 3);
      }
      if (!(fabsf(gmax) < f_inf())) {
        if (t == 0) {  // NaN, +inf, or every value -inf
          flag_row(a, row, D3S_ROW_NONFINITE);
          H.done = 1;
        }
      } else if (APPROX && approx_row_ok(rp, xmax, taux)) {
        stats_row_approx<JJ, BF16>(H, cands[row], &sm.cand_n[s], rb, q2, q2nd,
                                   __fmul_rn(-xmax, q2nd),
                                   __fmaf_rn(-fabsf(taux), 0x1p-21f, taux), gmax, t, lane, w);
      } else if (APPROX) {  // no row min here: the IEEE divide per element and the term floor
        stats_row<JJ, BF16, EXACT>(a, H, cands[row], &sm.cand_n[s], rb, q2, rp.T, rT, gmax,
                                   __fdiv_rn(taux, rp.T), -f_inf(), false, t, lane, w);
      } else {
        stats_row<JJ, BF16, EXACT>(a, H, cands[row], &sm.cand_n[s], rb, q2, rp.T, rT, gmax, tau,
                                   q2nd, div_rows_ok(xmin, xmax, rp.T, gmax, tau), t, lane, w);
      }
    } else if (t == 0) {
      if (pst != D3S_ROW_OK)
        flag_row(a, row, pst);
      else
        defer_row(a, row);
      H.done = 1;
    }
    // this warp is done with the stage; the last of the four refills it
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      if (atomicAdd(&sm.stage_done[s], 1u) == kFastW - 1) {
        // every warp has added its candidates: the row's count is final
        H.cnt = (int)sm.cand_n[s];
        sm.cand_n[s] = 0;
        sm.stage_done[s] = 0;
        const int nrow = row + stages * (int)gridDim.x;
        if (nrow < a.N) {
          fence_proxy_async();
          issue_row<ESZ>(a, nrow, dsm + (size_t)s * span, &sm.mbar[s], pol);
        }
      }
    }
    if constexpr (SELECT) {
      // One row per CTA (small batches): once every warp has added its
      // candidates, warp 0 samples the row; the stage is free and holds the
      // sorted keys and the tail's scratch.
      __syncthreads();
      if (w == 0 && !H.done) {
        float lse_lo, lse_hi;
        row_lse(H, a.approx_c0, lse_lo, lse_hi);
        (void)select_row(a, row, H.cnt, cands[row].cand, cands[row], raw_key(a, cur, lane), rp,
                         lse_lo, lse_hi, reinterpret_cast<unsigned long long *>(dsm),
                         reinterpret_cast<float *>(dsm + kCandCap * 8), lane);
      }
    }
  }
  if (SELECT && a.done_flag) {
    // every result of the launch is written (thread 0 wrote the row's id and
    // status itself): publish it to the host polling mapped memory
    __syncthreads();
    if (t == 0) {
      __threadfence_system();
      *reinterpret_cast<volatile int32_t *>(a.done_flag) = 1;
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

// ---- select kernel (K2): one warp per row ----

constexpr int kSelWarps = 8;
constexpr int kSelThreads = 32 * kSelWarps;
constexpr int kSelExactRows = 16;  // rows per CTA that wait for the exact sum at the end
constexpr int kStageCands = 128;  // candidates staged in shared memory per row

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int m) {
  const unsigned lo = __shfl_xor_sync(kFull, (unsigned)v, m);
  const unsigned hi = __shfl_xor_sync(kFull, (unsigned)(v >> 32), m);
  return ((unsigned long long)hi << 32) | lo;
}

// Compare-exchange of elements e (in x) and e + stride (in y) of one lane.
__device__ __forceinline__ void inreg_exchange(unsigned long long &x, unsigned long long &y, int e,
                                               int size) {
  const bool desc = (e & size) == 0;
  const bool swap = desc ? (x < y) : (x > y);
  const unsigned long long a = x;
  x = swap ? y : x;
  y = swap ? a : y;
}

// Bitonic sort of 32 * S keys held as v[s] = element lane + 32 s, descending.
// Fully unrolled: every stage's direction and partner masks are constants.
template <int S>
__device__ __forceinline__ void warp_sort_desc(unsigned long long (&v)[S], int lane) {
  constexpr int n = 32 * S;
#pragma unroll
  for (int size = 2; size <= n; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < 32) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const unsigned long long o = shfl_xor_u64(v[s], stride);
          const bool desc = ((lane + 32 * s) & size) == 0;
          const bool keep_max = ((lane & stride) == 0) == desc;
          v[s] = (v[s] > o) == keep_max ? v[s] : o;
        }
      } else if constexpr (S >= 2) {
        // partners in the same lane: register s and s ^ (stride / 32)
        if (stride == 32) {
#pragma unroll
          for (int s = 0; s < S; s += 2) inreg_exchange(v[s], v[s + 1], lane + 32 * s, size);
        } else if constexpr (S >= 4) {
#pragma unroll
          for (int s = 0; s < S; ++s)
            if ((s & 2) == 0) inreg_exchange(v[s], v[s + 2], lane + 32 * s, size);
        }
      }
    }
  }
}

// The same network on 32-bit keys (one shuffle and a min / max a step).
__device__ __forceinline__ void inreg_exchange32(uint32_t &x, uint32_t &y, bool desc) {
  const uint32_t hi = max(x, y), lo = min(x, y);
  x = desc ? hi : lo;
  y = desc ? lo : hi;
}

template <int S>
__device__ __forceinline__ void warp_sort_desc32(uint32_t (&v)[S], int lane) {
  constexpr int n = 32 * S;
#pragma unroll
  for (int size = 2; size <= n; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      if (stride < 32) {
#pragma unroll
        for (int s = 0; s < S; ++s) {
          const uint32_t o = __shfl_xor_sync(kFull, v[s], stride);
          const bool desc = ((lane + 32 * s) & size) == 0;
          const bool keep_max = ((lane & stride) == 0) == desc;
          v[s] = keep_max ? max(v[s], o) : min(v[s], o);
        }
      } else if constexpr (S >= 2) {
        // partners in the same lane; above 32 the direction depends on s only
        if (stride == 32) {
#pragma unroll
          for (int s = 0; s < S; s += 2) inreg_exchange32(v[s], v[s + 1], ((32 * s) & size) == 0);
        } else if constexpr (S >= 4) {
#pragma unroll
          for (int s = 0; s < S; ++s)
            if ((s & 2) == 0) inreg_exchange32(v[s], v[s + 2], ((32 * s) & size) == 0);
        }
      }
    }
  }
}

// Bitonic merge of a bitonic sequence of 32 keys (one a lane) into descending
// order.
__device__ __forceinline__ uint32_t merge32_desc(uint32_t v, int lane) {
#pragma unroll
  for (int stride = 16; stride > 0; stride >>= 1) {
    const uint32_t o = __shfl_xor_sync(kFull, v, stride);
    v = (lane & stride) == 0 ? max(v, o) : min(v, o);
  }
  return v;
}

// Two descending 32-key lists (one key a lane) into one descending 64-key list:
// hi holds ranks 0-31, lo ranks 32-63 ([a | reversed b] is bitonic).
__device__ __forceinline__ void merge64_desc(uint32_t a, uint32_t b, uint32_t &hi, uint32_t &lo,
                                             int lane) {
  const uint32_t br = __shfl_sync(kFull, b, 31 - lane);
  hi = merge32_desc(max(a, br), lane);
  lo = merge32_desc(min(a, br), lane);
}

// The k largest of C <= 128 32-bit keys (keys[], shared memory, left as they
// are) into top[0..k) in rank order, for k <= 64 or C <= 64: each 32-key block
// sorted by the one-register network (a rolled loop, so one copy of its code),
// pairs of blocks merged into sorted 64-key lists, and for more than 64 keys
// the top 64 of two such lists (the elementwise max of one and the other
// reversed is a bitonic sequence holding them) merged once more. top needs 128
// entries.
__device__ __forceinline__ void rank_keys32(const uint32_t *keys, int C, int k, uint32_t *top,
                                            int lane) {
  const int nb = (C + 31) >> 5;
#pragma unroll 1
  for (int b = 0; b < nb; ++b) {
    uint32_t v[1] = {32 * b + lane < C ? keys[32 * b + lane] : 0u};
    warp_sort_desc32<1>(v, lane);
    top[32 * b + lane] = v[0];
  }
  __syncwarp();
  if (nb == 1) return;  // the sorted block is the ranking
  uint32_t p0, p1;
  merge64_desc(top[lane], top[32 + lane], p0, p1, lane);
  if (nb > 2) {
    uint32_t q0, q1;
    merge64_desc(top[64 + lane], nb > 3 ? top[96 + lane] : 0u, q0, q1, lane);
    const uint32_t m0 = max(p0, __shfl_sync(kFull, q1, 31 - lane));
    const uint32_t m1 = max(p1, __shfl_sync(kFull, q0, 31 - lane));
    p0 = merge32_desc(max(m0, m1), lane);
    p1 = merge32_desc(min(m0, m1), lane);
  }
  __syncwarp();
  top[lane] = p0;
  if (32 + lane < k) top[32 + lane] = p1;
}

// Sort the row's C <= 32 S candidates (the first kStageCands staged in cs, the
// rest in the slab) with the warp and store the first k keys, in rank order,
// into sk.
template <int S>
__device__ __forceinline__ void sort_cands(const unsigned long long *cs, const RowCands &Cs,
                                           int C, int k, float T, unsigned long long *sk,
                                           int lane) {
  unsigned long long v[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int e = lane + 32 * s;
    v[s] = e < C ? raw_to_key(e < kStageCands ? cs[e] : Cs.cand[e], T) : 0ull;
  }
  warp_sort_desc<S>(v, lane);
#pragma unroll
  for (int s = 0; s < S; ++s)
    if (lane + 32 * s < k) sk[lane + 32 * s] = v[s];
}

// More than 128 candidates: the k largest taken one at a time (two warp reduxes
// per rank), into sk in rank order.
__device__ __forceinline__ void select_cands(const RowCands &Cs, int C, int k, float T,
                                             unsigned long long *sk, int lane) {
  unsigned long long v[8], best = 0ull;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int e = lane + 32 * s;
    v[s] = e < C ? raw_to_key(Cs.cand[e], T) : 0ull;
    best = v[s] > best ? v[s] : best;
  }
  for (int r = 0; r < k; ++r) {
    const unsigned mh = __reduce_max_sync(kFull, (unsigned)(best >> 32));
    const unsigned ml =
        __reduce_max_sync(kFull, (unsigned)(best >> 32) == mh ? (unsigned)best : 0u);
    const unsigned long long wk = ((unsigned long long)mh << 32) | ml;
    if (best == wk) {
      unsigned long long nb = 0ull;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (v[s] == wk) v[s] = 0ull;
        nb = v[s] > nb ? v[s] : nb;
      }
      best = nb;
    }
    if (lane == 0) sk[r] = wk;
  }
}

// In place in shared memory: sort the C <= 32 S keys of list[] and leave the
// first k in rank order at list[0..k).
template <int S>
__device__ __forceinline__ void sort_list(unsigned long long *list, int C, int k, int lane) {
  unsigned long long v[S];
#pragma unroll
  for (int s = 0; s < S; ++s) {
    const int e = lane + 32 * s;
    v[s] = e < C ? list[e] : 0ull;
  }
  warp_sort_desc<S>(v, lane);
  __syncwarp();
#pragma unroll
  for (int s = 0; s < S; ++s)
    if (lane + 32 * s < k) list[lane + 32 * s] = v[s];
}

// In place: the k largest of C <= 256 keys, one per round, into list[0..k).
__device__ __forceinline__ void select_list(unsigned long long *list, int C, int k, int lane) {
  unsigned long long v[8], best = 0ull;
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    const int e = lane + 32 * s;
    v[s] = e < C ? list[e] : 0ull;
    best = v[s] > best ? v[s] : best;
  }
  __syncwarp();
  for (int r = 0; r < k; ++r) {
    const unsigned mh = __reduce_max_sync(kFull, (unsigned)(best >> 32));
    const unsigned ml =
        __reduce_max_sync(kFull, (unsigned)(best >> 32) == mh ? (unsigned)best : 0u);
    const unsigned long long wk = ((unsigned long long)mh << 32) | ml;
    if (best == wk) {
      unsigned long long nb = 0ull;
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        if (v[s] == wk) v[s] = 0ull;
        nb = v[s] > nb ? v[s] : nb;
      }
      best = nb;
    }
    if (lane == 0) list[r] = wk;
  }
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_prev() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// A row's header and its first candidates, staged by cp.async: as many as the
// row holds, up to kStageCands (the count is read one row earlier).
struct alignas(16) SelStage {
  RowHead head;
  unsigned long long cand[kStageCands];
};

constexpr int kHeadChunks = (int)(sizeof(RowHead) / 16);
static_assert(sizeof(RowHead) % 16 == 0 && kHeadChunks <= 32, "RowHead is copied in 16-byte chunks");

__device__ __forceinline__ int row_count(const RowHead *heads, int row) {
  return min(max(heads[row].cnt, 0), kStageCands);
}

__device__ __forceinline__ void stage_row(const RowHead *heads, const RowCands *cands, int row,
                                          int cnt, SelStage &st, int lane) {
  if (lane < kHeadChunks)
    cp_async16(reinterpret_cast<char *>(&st.head) + 16 * lane,
               reinterpret_cast<const char *>(heads + row) + 16 * lane);
  const int chunks = (cnt + 1) >> 1;  // two keys per 16-byte chunk
  for (int c = lane; c < chunks; c += 32)
    cp_async16(reinterpret_cast<char *>(st.cand) + 16 * c,
               reinterpret_cast<const char *>(cands + row) + 16 * c);
}

// The top k of a row's C <= 256 candidates (the first kStageCands in cs, all of
// them in Cs), keyed by their exact quotients in one pass into sk (>= C keys of
// shared memory) and ranked there in place: sk[0 .. k) in rank order.
__device__ __forceinline__ void rank_cands_smem(const unsigned long long *cs, const RowCands &Cs,
                                                int C, int k, float T, unsigned long long *sk,
                                                int lane) {
  for (int e = lane; e < C; e += 32) sk[e] = raw_to_key(e < kStageCands ? cs[e] : Cs.cand[e], T);
  __syncwarp();
  if (C <= 32)
    sort_list<1>(sk, C, k, lane);
  else if (C <= 64)
    sort_list<2>(sk, C, k, lane);
  else if (C <= 128)
    sort_list<4>(sk, C, k, lane);
  else
    select_list(sk, C, k, lane);
}

// The same ranking with the keys in registers (sk needs only k entries).
__device__ __forceinline__ void rank_cands(const unsigned long long *cs, const RowCands &Cs, int C,
                                           int k, float T, unsigned long long *sk, int lane) {
  if (C <= 32)
    sort_cands<1>(cs, Cs, C, k, T, sk, lane);
  else if (C <= 64)
    sort_cands<2>(cs, Cs, C, k, T, sk, lane);
  else if (C <= 128)
    sort_cands<4>(cs, Cs, C, k, T, sk, lane);
  else
    select_cands(Cs, C, k, T, sk, lane);
}

// key draws the row's uniforms; the row's lse lies in [lse_lo, lse_hi] (equal
// when exact). Returns false, having written nothing, when the row's top-p cut
// needs the exact full-row sum (an approximate-sum row whose cut is uncertain).
__device__ __forceinline__ bool select_row(const KArgs &a, int row, int C,
                                           const unsigned long long *cs, const RowCands &Cs,
                                           uint2 key, const RowP &rp, float lse_lo, float lse_hi,
                                           unsigned long long *sk, float *scr, int lane) {
  // more candidates than the list holds (ties), or fewer than k (the top k
  // reaches below every candidate: -inf entries): the wide kernel's exact path
  if (C > kCandCap || C < rp.k) {
    if (lane == 0) defer_row(a, row);
    return true;
  }
  if (C <= 128 && (rp.k <= 64 || C <= 64) && !a.topk_ids) {
    // rank the 32-bit value keys (okey(q)); the tail looks up the drawn rank's id
    uint32_t *top = reinterpret_cast<uint32_t *>(sk);  // [0, 128)
    uint32_t *keys = top + kFastMaxK;                   // [0, C)
    for (int e = lane; e < C; e += 32)
      keys[e] = okey(__fdiv_rn(
          __uint_as_float((uint32_t)((e < kStageCands ? cs[e] : Cs.cand[e]) >> 32)), rp.T));
    __syncwarp();
    rank_keys32(keys, C, rp.k, top, lane);
    __syncwarp();
    return sample_tail_r(a, row, key, Ranks32{top, keys, C, cs, Cs.cand, kStageCands}, scr, rp.k,
                         lse_lo, lse_hi, rp.p, lane);
  }
  rank_cands_smem(cs, Cs, C, rp.k, rp.T, sk, lane);
  __syncwarp();
  return sample_tail(a, row, key, sk, scr, rp.k, lse_lo, lse_hi, rp.p, lane);
}

// The rows whose cut needed the exact full-row sum, by the whole CTA once its
// warps are done: thread t < 256 computes partial t of the definition, then warp
// 0 ranks the row's stored candidates (sk: 256 keys of shared memory) and runs the
// tail with the exact lse. Few rows per launch come here (the cut must fall
// within about 1e-5 of top_p); doing them last keeps their reads of the row (long
// evicted from L2) off every warp's critical path but one. Called by every thread
// of the CTA (at least kPartials of them).
__device__ __forceinline__ void finish_exact_rows(const KArgs &a, const RowHead *heads,
                                                  const RowCands *cands, const int *rows, unsigned n,
                                                  unsigned long long *red, unsigned long long *sk,
                                                  float *scr) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  for (unsigned e = 0; e < n; ++e) {
    const int xrow = rows[e];
    RowP rp;
    row_params(a, xrow, rp);
    const RowHead &H = heads[xrow];
    const float gmax = H.gmax;
    if (t < kPartials) {
      const int64_t off = phys_row(a, xrow) * a.ld;
      const bool bf16 = a.dtype == D3S_BF16;
      const float rT = __frcp_rn(rp.T), mT = -rp.T;
      const bool recip = rp.T >= 0x1p-17f && rp.T <= 0x1p20f;  // div_rows' exact range of T
      float xv[kFastMaxV / kPartials];
#pragma unroll
      for (int j = 0; j < kFastMaxV / kPartials; ++j) {
        const int i = t + kPartials * j;
        xv[j] = i < a.V ? (bf16 ? load_x<true>(a.logits, off + i) : load_x<false>(a.logits, off + i))
                        : 0.0f;
      }
      float sp = 0.0f;
#pragma unroll
      for (int j = 0; j < kFastMaxV / kPartials; ++j) {
        if (t + kPartials * j < a.V) {
          const float ax = fabsf(xv[j]);
          const float q = (recip && ax >= 0x1p-100f && ax <= 0x1p60f) ? div_rows(xv[j], rT, mT)
                                                                       : __fdiv_rn(xv[j], rp.T);
          sp = __fadd_rn(sp, exp_term(__fsub_rn(q, gmax)));
        }
      }
      const unsigned long long ws = warp_sum_fixed(__float2ull_rz(__fmul_rn(sp, 0x1p46f)));
      if (lane == 0) red[w] = ws;
    }
    __syncthreads();
    if (w == 0) {
      unsigned long long Se = 0;
#pragma unroll
      for (int i = 0; i < kPartials / 32; ++i) Se += red[i];
      const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(Se), 0x1p-46f)));
      const RowCands &Cs = cands[xrow];
      rank_cands_smem(Cs.cand, Cs, H.cnt, rp.k, rp.T, sk, lane);
      __syncwarp();
      sample_tail(a, xrow, row_key(a, xrow), sk, scr, rp.k, lse, lse, rp.p, lane);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kSelThreads, 4) sample_select_kernel(const KArgs a,
                                                                        const RowHead *heads,
                                                                        const RowCands *cands) {
  __shared__ __align__(16) float scr_all[kSelWarps][kFastMaxK + 4];
  __shared__ unsigned long long sk_all[kSelWarps][kFastMaxK];
  __shared__ SelStage stg_all[kSelWarps][2];
  __shared__ int exact_rows[kSelExactRows];
  __shared__ unsigned exact_n;
  __shared__ unsigned long long exact_red[kSelWarps];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (threadIdx.x == 0) exact_n = 0u;
  __syncthreads();
  const int gw = blockIdx.x * kSelWarps + w, nw = gridDim.x * kSelWarps;
  unsigned long long *sk = sk_all[w];
  int row = gw, b = 0;
  int cnt_next = 0;  // candidate count of row + nw
  // The per-row scalars of the warp's next 32 rows, lane i holding those of
  // the i-th (its key, its lse bracket from the header, its parameters): one
  // key derivation and one pair of logs per lane instead of per row.
  uint2 key32 = make_uint2(0u, 0u);
  float lo32 = 0.0f, hi32 = 0.0f, T32 = 1.0f, p32 = 1.0f;
  int k32 = 1;
  if (row < a.N) {
    stage_row(heads, cands, row, row_count(heads, row), stg_all[w][0], lane);
    if (row + nw < a.N) cnt_next = row_count(heads, row + nw);
  }
  cp_async_commit();
  for (int iter = 0; row < a.N; row += nw, b ^= 1, ++iter) {
    if ((iter & 31) == 0) {
      const int r = row + lane * nw;
      if (r < a.N && !heads[r].done) {
        key32 = row_key(a, r);
        row_lse(heads[r], a.approx_c0, lo32, hi32);
        RowP rr;
        resolve(a, load_raw(a, r), rr);  // valid: the stats kernel flagged every other row
        T32 = rr.T;
        p32 = rr.p;
        k32 = rr.k;
      }
    }
    const int src = iter & 31;
    const uint2 key = make_uint2(__shfl_sync(kFull, key32.x, src), __shfl_sync(kFull, key32.y, src));
    const float lse_lo = __shfl_sync(kFull, lo32, src), lse_hi = __shfl_sync(kFull, hi32, src);
    RowP rp;
    rp.T = __shfl_sync(kFull, T32, src);
    rp.p = __shfl_sync(kFull, p32, src);
    rp.k = __shfl_sync(kFull, k32, src);
    // the next row's header and candidates are copied while this row is
    // sampled, and the count of the row after it is read
    const int nrow = row + nw;
    int cnt_nn = 0;
    __syncwarp();
    if (nrow < a.N) {
      stage_row(heads, cands, nrow, cnt_next, stg_all[w][b ^ 1], lane);
      if (nrow + nw < a.N) cnt_nn = row_count(heads, nrow + nw);
    }
    cp_async_commit();
    cp_async_wait_prev();
    __syncwarp();
    const SelStage &st = stg_all[w][b];
    if (!st.head.done) {
      if (!select_row(a, row, st.head.cnt, st.cand, cands[row], key, rp, lse_lo, lse_hi, sk,
                      scr_all[w], lane) &&
          lane == 0) {
        const unsigned pos = atomicAdd(&exact_n, 1u);
        if (pos < (unsigned)kSelExactRows)
          exact_rows[pos] = row;
        else
          defer_row_exact_sum(a, row);
      }
    }
    cnt_next = cnt_nn;
  }
  static_assert(kSelThreads >= kPartials, "one partial per thread");
  __syncthreads();
  finish_exact_rows(a, heads, cands, exact_rows, min(exact_n, (unsigned)kSelExactRows), exact_red,
                    sk_all[0], scr_all[0]);
}

// ---- row-warp kernel: one warp takes a row from its logits to its draw ----
//
// Each warp owns a shared-memory stage holding one row (one bulk copy of the
// 16-byte-aligned span around it; the row starts s elements into the stage)
// plus a candidate list and scratch. Lane l reads the stage's 16-byte chunks
// l, l + 32, ..., l + 32 (NC - 1). Chunk c, component e is element
// EPC c + e - s (EPC = 4 for f32, 8 for bf16), so a lane always meets the
// elements of the same eight partials (element i belongs to partial
// i mod 256), each in increasing order: f32 lane l holds partials
// 4l + e - s + 128 (i & 1), bf16 lane l holds 8l + e - s (mod 256).
//   pass 1: max, min, and four group maxima per lane (chunk i in group i % 4);
//   threshold: min over the groups of the ceil(k/4)-th largest of the 32 lanes'
//     group maxima (every group contributes >= ceil(k/4) elements at or above
//     it, so >= k elements reach it);
//   pass 2: q = x / T, the lane's eight partial sums of exp(max(q - max, -86))
//     as packed fp32x2 chains, and a bit per element with q >= threshold;
//   then the candidates go to the warp's list, the next row's copy starts into
//   the stage, and the warp sorts the candidates and runs the tail.
// Rows it cannot finish (k > 256, more than 256 candidates) go to the
// hand-off list for the wide kernel.

constexpr int kRwCandBytes = kCandCap * 8;
constexpr int kRwScrBytes = (kFastMaxK + 4) * 4;
constexpr int kRwTailBytes = kRwCandBytes + kRwScrBytes + 16;  // + the mbarrier
constexpr int kRowWarpMaxBatch = 2048;  // long rows: batches up to this take the row-warp kernel
constexpr int kSmallBatch = 512;        // batches up to this: one CTA per row, select in the same launch

// min over four 32-lane columns (v[c] of every lane) of each column's r-th
// largest value (1 <= r <= 32): four interleaved bitonic sorts.
__device__ __forceinline__ float warp_tau4(float (&v)[4], int r, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float o = __shfl_xor_sync(kFull, v[c], stride);
        v[c] = keep_max ? fmaxf(v[c], o) : fminf(v[c], o);
      }
    }
  float t = __shfl_sync(kFull, v[0], r - 1);
#pragma unroll
  for (int c = 1; c < 4; ++c) t = fminf(t, __shfl_sync(kFull, v[c], r - 1));
  return t;
}

// One 16-byte chunk of the stage as floats.
template <bool BF16>
__device__ __forceinline__ void rw_chunk(const unsigned char *stage, int c,
                                         float (&x)[BF16 ? 8 : 4]) {
  const uint4 u = *reinterpret_cast<const uint4 *>(stage + 16 * (size_t)c);
  if constexpr (BF16) {
    const unsigned w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      x[2 * j] = __uint_as_float(w[j] << 16);
      x[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    x[0] = __uint_as_float(u.x);
    x[1] = __uint_as_float(u.y);
    x[2] = __uint_as_float(u.z);
    x[3] = __uint_as_float(u.w);
  }
}

// Pass 2 over the lane's chunks. FAST: the per-row reciprocal division holds
// for every element; CLAMP: some term may fall below the -86 floor.
template <int NC, bool BF16, bool FAST, bool CLAMP>
__device__ __forceinline__ void rw_pass2(const unsigned char *stage, int lane, int s, int V,
                                         int cfull, float T, float rT, float gmax, float tau,
                                         float2 (&acc)[4],
                                         unsigned long long (&bits)[(NC * (BF16 ? 8 : 4) + 63) / 64]) {
  constexpr int EPC = BF16 ? 8 : 4;
  const float2 rT2 = make_float2(rT, rT), mT2 = make_float2(-T, -T);
  const float2 mg = make_float2(-gmax, -gmax);
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    const int c = lane + 32 * i;
    float x[EPC];
    rw_chunk<BF16>(stage, c, x);
    const bool partial = i == 0 || 32 * i + 31 >= cfull;  // warp-uniform
#pragma unroll
    for (int pp = 0; pp < EPC / 2; ++pp) {
      float2 q;
      if (FAST) {
        q = div_rows2(make_float2(x[2 * pp], x[2 * pp + 1]), rT2, mT2);
      } else {
        q = make_float2(__fdiv_rn(x[2 * pp], T), __fdiv_rn(x[2 * pp + 1], T));
      }
      float2 e = exp_term2<CLAMP>(__fadd2_rn(q, mg));
      bool v0 = true, v1 = true;
      if (partial) {
        const int p0 = EPC * c + 2 * pp;
        v0 = p0 >= s && p0 < V + s;
        v1 = p0 + 1 >= s && p0 + 1 < V + s;
        if (!v0) e.x = 0.0f;
        if (!v1) e.y = 0.0f;
      }
      const int ai = BF16 ? pp : 2 * (i & 1) + pp;
      acc[ai] = __fadd2_rn(acc[ai], e);
      const int b = i * EPC + 2 * pp;
      if (v0 && q.x >= tau) bits[b >> 6] |= 1ull << (b & 63);
      if (v1 && q.y >= tau) bits[(b + 1) >> 6] |= 1ull << ((b + 1) & 63);
    }
  }
}

// Warps that fit on an SM: the f32 rows of the largest chunk counts are held
// back by shared memory (about 20 KB a warp), so they may use more registers.
template <int NC>
struct RwBounds {
  static constexpr int kMinBlocks = NC >= 25 ? 10 : 16;
};

template <int NC, bool BF16>
__global__ void __launch_bounds__(32, RwBounds<NC>::kMinBlocks)
    sample_rowwarp_kernel(const KArgs a, int stage_bytes) {
  extern __shared__ __align__(128) unsigned char dsm[];
  constexpr int ESZ = BF16 ? 2 : 4;
  constexpr int EPC = 16 / ESZ;
  constexpr int NBW = (NC * EPC + 63) / 64;
  const int lane = threadIdx.x;
  unsigned char *stage = dsm;
  unsigned long long *cs = reinterpret_cast<unsigned long long *>(dsm + stage_bytes);
  float *scr = reinterpret_cast<float *>(dsm + stage_bytes + kRwCandBytes);
  uint64_t *bar = reinterpret_cast<uint64_t *>(dsm + stage_bytes + kRwCandBytes + kRwScrBytes);
  const int V = a.V;
  const uint64_t pol = evict_first_policy();
  if (lane == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  int row = blockIdx.x;
  const int nrows = gridDim.x;
  if (row < a.N && lane == 0) issue_row<ESZ>(a, row, stage, bar, pol);
  RawP nxt;
  if (row < a.N) nxt = load_raw(a, row);
  uint32_t phase = 0;
  for (; row < a.N; row += nrows, phase ^= 1u) {
    const RawP cur = nxt;
    const int nrow = row + nrows;
    if (nrow < a.N) nxt = load_raw(a, nrow);
    RowP rp;
    const int pst = resolve(a, cur, rp);
    if (!mbar_wait_bounded(bar, phase)) {
      if (lane == 0) {
        atomicOr(a.error, 1);
        mbar_wait_bounded(bar, phase);  // let the copy in flight land before exiting
      }
      return;
    }
    const int s = (int)((((uintptr_t)a.logits + (uintptr_t)phys_row(a, row) * (uintptr_t)a.ld * ESZ) &
                         15) / ESZ);
    const int cfull = (V + s) / EPC;  // chunks 1 .. cfull - 1 lie inside the row

    // pass 1: max, min, group maxima
    float pm[4] = {-f_inf(), -f_inf(), -f_inf(), -f_inf()};
    float mn0 = f_inf(), mn1 = f_inf();
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      float x[EPC];
      rw_chunk<BF16>(stage, c, x);
      if (i == 0 || 32 * i + 31 >= cfull) {
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          const int p = EPC * c + e;
          const bool valid = p >= s && p < V + s;
          pm[i & 3] = max_nan(pm[i & 3], valid ? x[e] : -f_inf());
          if (e & 1)
            mn1 = fminf(mn1, valid ? x[e] : f_inf());
          else
            mn0 = fminf(mn0, valid ? x[e] : f_inf());
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          pm[i & 3] = max_nan(pm[i & 3], x[e]);
          if (e & 1)
            mn1 = fminf(mn1, x[e]);
          else
            mn0 = fminf(mn0, x[e]);
        }
      }
    }
    const float xmax = warp_max_nan(max_nan(max_nan(pm[0], pm[1]), max_nan(pm[2], pm[3])));
    const float xmin = -warp_max(-fminf(mn0, mn1));
    if (a.finite && lane == 0) a.finite[row] = (fabsf(xmax) < f_inf() && fabsf(xmin) < f_inf()) ? 1 : 0;

    bool go = false;
    float lse = 0.0f;
    int C = 0;
    if (pst != D3S_ROW_OK) {
      if (lane == 0) flag_row(a, row, pst);
    } else if (rp.k > kFastMaxK) {
      if (lane == 0) defer_row(a, row);
    } else {
      const float T = rp.T;
      const float gmax = __fdiv_rn(xmax, T);  // max(x / T) = RN(max(x) / T): RN is monotone
      if (!(fabsf(gmax) < f_inf())) {         // NaN, +inf, or every value -inf
        if (lane == 0) flag_row(a, row, D3S_ROW_NONFINITE);
      } else {
        const int r = (rp.k + 3) >> 2;
        float v4[4] = {pm[0], pm[1], pm[2], pm[3]};
        const float taux = r <= 32 ? warp_tau4(v4, r, lane) : warp_rth_largest<4>(v4, rp.k);
        const float tau = __fdiv_rn(taux, T);
        const float rT = __frcp_rn(T);
        const bool fast = div_rows_ok(xmin, xmax, T, gmax, tau);
        const bool clamp = !(__fsub_rn(__fdiv_rn(xmin, T), gmax) >= kTermFloor);
        float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                         make_float2(0.0f, 0.0f)};
        unsigned long long bits[NBW];
#pragma unroll
        for (int j = 0; j < NBW; ++j) bits[j] = 0ull;
        if (fast && !clamp)
          rw_pass2<NC, BF16, true, false>(stage, lane, s, V, cfull, T, rT, gmax, tau, acc, bits);
        else if (fast)
          rw_pass2<NC, BF16, true, true>(stage, lane, s, V, cfull, T, rT, gmax, tau, acc, bits);
        else
          rw_pass2<NC, BF16, false, true>(stage, lane, s, V, cfull, T, rT, gmax, tau, acc, bits);
        // the lane's eight partials, each truncated to 2^-46 fixed point, added exactly
        unsigned long long fx = 0ull;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          fx += __float2ull_rz(__fmul_rn(acc[j].x, 0x1p46f)) + __float2ull_rz(__fmul_rn(acc[j].y, 0x1p46f));
        const unsigned long long S = warp_sum_u64(fx);
        lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(S), 0x1p-46f)));
        // candidates into the warp's list
        int mine = 0;
#pragma unroll
        for (int j = 0; j < NBW; ++j) mine += __popcll(bits[j]);
        int incl = mine;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const int o = __shfl_up_sync(kFull, incl, d);
          if (lane >= d) incl += o;
        }
        C = __shfl_sync(kFull, incl, 31);
        if (C > kCandCap || C < rp.k) {  // C < k: the top k reaches below every candidate (-inf)
          if (lane == 0) defer_row(a, row);
        } else {
          int pos = incl - mine;
#pragma unroll
          for (int j = 0; j < NBW; ++j) {
            unsigned long long m = bits[j];
            while (m) {
              const int b = 64 * j + __ffsll((long long)m) - 1;
              m &= m - 1;
              const int i = b / EPC, e = b - i * EPC;
              const int p = EPC * (lane + 32 * i) + e;
              float xv;
              if constexpr (BF16)
                xv = __uint_as_float((unsigned)reinterpret_cast<const unsigned short *>(stage)[p] << 16);
              else
                xv = reinterpret_cast<const float *>(stage)[p];
              cs[pos++] = cand_key(__fdiv_rn(xv, T), (uint32_t)(p - s));
            }
          }
          go = true;
        }
      }
    }
    // the stage has been read: start the next row's copy into it
    __syncwarp();
    if (lane == 0 && nrow < a.N) {
      fence_proxy_async();
      issue_row<ESZ>(a, nrow, stage, bar, pol);
    }
    if (go) {
      const int k = rp.k;
      if (C <= 32)
        sort_list<1>(cs, C, k, lane);
      else if (C <= 64)
        sort_list<2>(cs, C, k, lane);
      else if (C <= 128)
        sort_list<4>(cs, C, k, lane);
      else
        select_list(cs, C, k, lane);
      __syncwarp();
      sample_tail(a, row, raw_key(a, cur, lane), cs, scr, k, lse, lse, rp.p, lane);
    }
    __syncwarp();
  }
}

// ---- one-warp stats kernel: the streaming pass with one warp per row ----
//
// The approximate-sum stats of the pair, done by one warp per row instead of
// four, so the per-row work (parameters, reductions, threshold, sums,
// candidate positions) runs once per row. Warp gw of the grid (NW warps) takes
// rows gw, gw + NW, ...; it owns `depth` stages of NC * 512 bytes (every chunk a
// lane reads) and keeps the bulk copies of its next depth - 1 rows in flight.
// Per row:
//   the stage's elements outside the row (before it in the first chunk, after
//     it up to the end of the stage) are set to -inf, so no pass tests bounds;
//   pass 1: lane l reads 16-byte chunks l + 32 i; each chunk's max stays in a
//     register, chunk i also feeds group i % 4's max; the row max;
//   threshold: for each group the ceil(k/4)-th largest of its 32 lane maxima
//     (repeated warp max reduxes), then the largest of the four that at least
//     k of the 128 group maxima reach (each such maximum is a distinct element,
//     and the smallest of the four always qualifies); tau_lo just under it as
//     in the four-warp kernel;
//   pass 2: the terms 2^(x c + g) by the SFU into eight accumulators and one
//     candidate bit per chunk (chunk max > tau_lo);
//   the candidates (x > tau_lo) of the chunks whose bit is set into the row's
//     list at positions from a shared counter (their order does not matter:
//     the select kernel ranks them by key);
//   the header, then the bulk copy of row it + depth into the stage.
// Rows the approximate path does not take (k > 128, T or |x| at the extremes)
// go to the wide kernel; bad parameters and non-finite rows are flagged here.
// The exact stats of a row in the one-warp kernel's stage (rows with k <= 256
// that the approximate path does not take): the row min, the candidate
// threshold (min over eight groups, chunk i in group i % 8, of the
// ceil(k/8)-th largest of the 32 lanes' group maxima, so at least k elements
// reach it), then the definition's 256 partial sums as the row-warp kernel
// computes them (lane l holds partials 4l + e - s + 128 (i & 1) of f32 rows,
// 8l + e - s of bf16 rows, each a sequential float sum in element order; q by
// the per-row reciprocal where that is the IEEE quotient; exp with the -86
// floor; padding adds +0) and every element with q >= RN(taux / T) into the
// row's list. Returns the fixed-point full-row sum. Loops stay rolled: such
// rows are rare, and the code must not crowd the approximate path.
template <int NC, bool BF16>
__device__ __forceinline__ unsigned long long stats1_exact(const KArgs &a, const RowP &rp, RowCands &Cs,
                                                           const unsigned char *stage, unsigned *cand_n,
                                                           float xmax, float gmax, float rT, int s,
                                                           int lane) {
  constexpr int EPC = BF16 ? 8 : 4;
  const int V = a.V;
  float mn = f_inf(), v8[8], t8[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) v8[g] = -f_inf();
#pragma unroll 1
  for (int i8 = 0; i8 < NC; i8 += 8) {
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      const int ch = lane + 32 * (i8 + h);
      if (i8 + h < NC) {
        float x[EPC];
        rw_chunk<BF16>(stage, ch, x);
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          const int p = EPC * ch + e;
          mn = fminf(mn, (p >= s && p < V + s) ? x[e] : f_inf());
          v8[h] = fmaxf(v8[h], x[e]);  // outside the row the stage holds -inf
        }
      }
    }
  }
  const float xmin = -warp_max(-mn);
  const int r = (rp.k + 7) >> 3;  // <= 32: k <= 256
  for (int j = 0;; ++j) {
#pragma unroll
    for (int g = 0; g < 8; ++g) t8[g] = warp_max(v8[g]);
    if (j + 1 >= r) break;
#pragma unroll
    for (int g = 0; g < 8; ++g) v8[g] = v8[g] == t8[g] ? -f_inf() : v8[g];
  }
  float taux = t8[0];
#pragma unroll
  for (int g = 1; g < 8; ++g) taux = fminf(taux, t8[g]);
  const float T = rp.T;
  const float tau = __fdiv_rn(taux, T);
  const bool fast = div_rows_ok(xmin, xmax, T, gmax, tau);
  float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                   make_float2(0.0f, 0.0f)};
#pragma unroll 1
  for (int i2 = 0; i2 < NC; i2 += 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int ch = lane + 32 * (i2 + h);
      if (i2 + h < NC) {
        float x[EPC];
        rw_chunk<BF16>(stage, ch, x);
#pragma unroll
        for (int e = 0; e < EPC; ++e) {
          const int p = EPC * ch + e;
          const bool valid = p >= s && p < V + s;
          const float q = fast ? div_rows(x[e], rT, -T) : __fdiv_rn(x[e], T);
          const float t = valid ? exp_term(__fsub_rn(q, gmax)) : 0.0f;
          const int ai = BF16 ? e / 2 : 2 * h + e / 2;
          if (e & 1)
            acc[ai].y = __fadd_rn(acc[ai].y, t);
          else
            acc[ai].x = __fadd_rn(acc[ai].x, t);
          if (valid && q >= tau) {
            const unsigned pos = atomicAdd(cand_n, 1u);
            if (pos < (unsigned)kCandCap) Cs.cand[pos] = raw_cand(x[e], (uint32_t)(p - s));
          }
        }
      }
    }
  }
  unsigned long long fx = 0ull;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    fx += __float2ull_rz(__fmul_rn(acc[j].x, 0x1p46f)) + __float2ull_rz(__fmul_rn(acc[j].y, 0x1p46f));
  return warp_sum_u64(fx);
}

constexpr int kS1MaxWarps = 16;
constexpr int kS1MaxDepth = 4;
constexpr int kS1SmemBytes = 227 * 1024 - 1024;  // dynamic shared memory of the one-warp kernel's CTA

// One row of the one-warp stats (the stage holds the row's bulk copy): the
// bytes outside the row set to -inf, pass 1, the threshold, pass 2 (or the
// exact stats), the candidates into the row's list and the header. cand_n is the
// warp's candidate counter in shared memory (zero between rows).
template <int NC, bool BF16>
__device__ __forceinline__ void stats1_row(const KArgs &a, RowHead *heads, RowCands *cands,
                                           unsigned char *stage, unsigned *cand_n, int row, int pst,
                                           RowP rp, float c, float rT, int lane) {
  constexpr int ESZ = BF16 ? 2 : 4;
  constexpr int EPC = 16 / ESZ;
  const int V = a.V;
  const uintptr_t start =
      (uintptr_t)a.logits + (uintptr_t)phys_row(a, row) * (uintptr_t)a.ld * ESZ;
  const int s = (int)((start & 15) / ESZ);
  const int nch = (int)((((start + (uintptr_t)V * ESZ + 15) & ~(uintptr_t)15) - (start & ~(uintptr_t)15)) / 16);
  // -inf outside the row: the s elements before it, the rest of its last
  // chunk, and every chunk past the copy up to the end of the stage
  if constexpr (BF16) {
    unsigned short *e = reinterpret_cast<unsigned short *>(stage);
    if (lane < s) e[lane] = 0xFF80u;
    if (V + s + lane < nch * EPC && lane < EPC) e[V + s + lane] = 0xFF80u;
  } else {
    float *e = reinterpret_cast<float *>(stage);
    if (lane < s) e[lane] = -f_inf();
    if (V + s + lane < nch * EPC && lane < EPC) e[V + s + lane] = -f_inf();
  }
  {
    const uint4 ninf = BF16 ? make_uint4(0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u, 0xFF80FF80u)
                            : make_uint4(0xFF800000u, 0xFF800000u, 0xFF800000u, 0xFF800000u);
    for (int ch = nch + lane; ch < 32 * NC; ch += 32) reinterpret_cast<uint4 *>(stage)[ch] = ninf;
  }
  __syncwarp();

  // pass 1: chunk maxima, group maxima, the row max
  float cm[NC];
  float gm[4] = {-f_inf(), -f_inf(), -f_inf(), -f_inf()};
#pragma unroll
  for (int i = 0; i < NC; ++i) {
    float x[EPC];
    rw_chunk<BF16>(stage, lane + 32 * i, x);
    float m = max_nan(x[0], x[1]);
#pragma unroll
    for (int e = 2; e < EPC; e += 2) m = max_nan(m, max_nan(x[e], x[e + 1]));
    cm[i] = m;
    gm[i & 3] = max_nan(gm[i & 3], m);
  }
  const float xmax = warp_max_nan(max_nan(max_nan(gm[0], gm[1]), max_nan(gm[2], gm[3])));

  RowHead &H = heads[row];
  // 0: written here (flagged or handed on), 1: approximate stats, 2: exact stats
  int mode = 0;
  float gmax = 0.0f, taux = 0.0f;
  if (pst != D3S_ROW_OK) {
    if (lane == 0) flag_row(a, row, pst);
  } else if (rp.k > kFastMaxK) {
    if (lane == 0) defer_row(a, row);
  } else {
    const float ax = fabsf(xmax);
    gmax = (ax >= 0x1p-100f && ax <= 0x1p60f && rp.T >= 0x1p-17f && rp.T <= 0x1p20f)
               ? div_rows(xmax, rT, -rp.T)
               : __fdiv_rn(xmax, rp.T);  // max(x / T) = RN(max(x) / T): RN is monotone
    if (!(fabsf(gmax) < f_inf())) {     // NaN, +inf, or every value -inf
      if (lane == 0) flag_row(a, row, D3S_ROW_NONFINITE);
    } else if (rp.k <= kApproxMaxK) {
      const int r = (rp.k + 3) >> 2;  // <= 32
      float v[4] = {gm[0], gm[1], gm[2], gm[3]}, t[4];
      for (int j = 0;; ++j) {
#pragma unroll
        for (int g = 0; g < 4; ++g) t[g] = warp_max(v[g]);
        if (j + 1 >= r) break;
#pragma unroll
        for (int g = 0; g < 4; ++g) v[g] = v[g] == t[g] ? -f_inf() : v[g];
      }
      taux = fminf(fminf(t[0], t[1]), fminf(t[2], t[3]));
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        int n = 0;
#pragma unroll
        for (int h = 0; h < 4; ++h) n += gm[h] >= t[g] ? 1 : 0;
        if ((int)__reduce_add_sync(kFull, (unsigned)n) >= rp.k) taux = fmaxf(taux, t[g]);
      }
      mode = approx_row_ok(rp, xmax, taux) ? 1 : 2;
    } else {
      mode = 2;
    }
  }
  if (mode == 0) {
    if (lane == 0) H.done = 1;
  } else {
    RowCands &Cs = cands[row];
    unsigned long long S;
    if (mode == 1) {
      // pass 2: the approximate full-row sum and the candidate chunks
      const float tau_lo = __fmaf_rn(-fabsf(taux), 0x1p-21f, taux);
      const float2 c2 = make_float2(c, c);
      const float g = __fmul_rn(-xmax, c);
      const float2 g2 = make_float2(g, g);
      float2 acc[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                       make_float2(0.0f, 0.0f)};
      uint32_t b0 = 0u, b1 = 0u;  // bit i: chunk i (i < 32), chunk 32 + i
#pragma unroll
      for (int i = NC - 1; i >= 0; --i) {
        float x[EPC];
        rw_chunk<BF16>(stage, lane + 32 * i, x);
#pragma unroll
        for (int pp = 0; pp < EPC / 2; ++pp) {
          const float2 u = __ffma2_rn(make_float2(x[2 * pp], x[2 * pp + 1]), c2, g2);
          const int ai = (2 * i + pp) & 3;
          acc[ai] = __fadd2_rn(acc[ai], make_float2(ex2_approx(u.x), ex2_approx(u.y)));
        }
        // the sign of tau_lo - max: set when the chunk holds an element > tau_lo
        const uint32_t d = __float_as_uint(__fsub_rn(tau_lo, cm[i]));
        if (i >= 32)
          b1 = __funnelshift_l(d, b1, 1);
        else
          b0 = __funnelshift_l(d, b0, 1);
      }
      const float2 s4 = __fadd2_rn(__fadd2_rn(acc[0], acc[1]), __fadd2_rn(acc[2], acc[3]));
      S = warp_sum_u64(__float2ull_rz(__fmul_rn(__fadd_rn(s4.x, s4.y), 0x1p46f)));
      // the candidates of the marked chunks
      while (__any_sync(kFull, (b0 | b1) != 0u)) {
        if ((b0 | b1) != 0u) {
          int i;
          if (b0) {
            i = __ffs(b0) - 1;
            b0 &= b0 - 1;
          } else {
            i = 32 + __ffs(b1) - 1;
            b1 &= b1 - 1;
          }
          const int ch = lane + 32 * i;
          float x[EPC];
          rw_chunk<BF16>(stage, ch, x);
          int n = 0;
#pragma unroll
          for (int e = 0; e < EPC; ++e) n += x[e] > tau_lo ? 1 : 0;
          unsigned pos = atomicAdd(cand_n, (unsigned)n);
#pragma unroll
          for (int e = 0; e < EPC; ++e)
            if (x[e] > tau_lo) {
              if (pos < (unsigned)kCandCap) Cs.cand[pos] = raw_cand(x[e], (uint32_t)(EPC * ch + e - s));
              ++pos;
            }
        }
      }
    } else {
      S = stats1_exact<NC, BF16>(a, rp, Cs, stage, cand_n, xmax, gmax, rT, s, lane);
    }
    __syncwarp();
    if (lane == 0) {
      const int C = (int)atomicExch(cand_n, 0u);
      reinterpret_cast<int4 *>(&H)[0] = make_int4(__float_as_int(gmax), 0, C, mode == 1 ? 1 : 0);
      reinterpret_cast<ulonglong2 *>(&H)[1] = make_ulonglong2(S, 0ull);
      reinterpret_cast<ulonglong2 *>(&H)[2] = make_ulonglong2(0ull, 0ull);
    }
  }
}

template <int NC, bool BF16>
__global__ void __launch_bounds__(32 * kS1MaxWarps)
    sample_stats1_kernel(const KArgs a, RowHead *heads, RowCands *cands, int depth) {
  extern __shared__ __align__(128) unsigned char dsm[];
  __shared__ uint64_t bars[kS1MaxWarps][kS1MaxDepth];
  __shared__ unsigned cand_n[kS1MaxWarps];
  constexpr int ESZ = BF16 ? 2 : 4;
  constexpr int EPC = 16 / ESZ;
  constexpr int SB = NC * 512;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nwb = blockDim.x >> 5;
  const int V = a.V;
  unsigned char *stages = dsm + (size_t)w * depth * SB;
  uint64_t *bar = bars[w];
  const uint64_t pol = evict_first_policy();
  const long long gw = (long long)blockIdx.x * nwb + w, NW = (long long)gridDim.x * nwb;
  if (lane == 0) {
    for (int d = 0; d < depth; ++d) mbar_init(&bar[d], 1);
    cand_n[w] = 0u;
    fence_mbar_init();
    for (int d = 0; d < depth; ++d)
      if (gw + d * NW < a.N) issue_row<ESZ>(a, (int)(gw + d * NW), stages + (size_t)d * SB, &bar[d], pol);
  }
  __syncwarp();
  float T32 = 1.0f, c32 = 1.0f, rT32 = 1.0f;
  int k32 = 1, st32 = D3S_ROW_BADPARAM;
  int slot = 0;
  uint32_t phase = 0u;
  int it = 0;
  bool failed = false;
  for (;; ++it) {
    const long long row64 = gw + (long long)it * NW;
    if (row64 >= a.N) break;
    const int row = (int)row64;
    // the parameters of the warp's next 32 rows, lane i those of the i-th
    if ((it & 31) == 0) {
      const long long r = row64 + (long long)lane * NW;
      if (r < a.N) {
        RowP q{1.0f, 1.0f, 1};
        st32 = resolve(a, load_raw(a, (int)r), q);
        T32 = q.T;
        k32 = q.k;
        c32 = __fdiv_rn(kL2E, q.T);
        rT32 = __frcp_rn(q.T);
      }
    }
    const int src = it & 31;
    const int pst = __shfl_sync(kFull, st32, src);
    RowP rp;
    rp.T = __shfl_sync(kFull, T32, src);
    rp.k = __shfl_sync(kFull, k32, src);
    rp.p = 1.0f;
    const float c = __shfl_sync(kFull, c32, src), rT = __shfl_sync(kFull, rT32, src);
    unsigned char *stage = stages + (size_t)slot * SB;
    if (!__all_sync(kFull, mbar_wait_bounded(&bar[slot], phase))) {
      failed = true;
      break;
    }
    stats1_row<NC, BF16>(a, heads, cands, stage, &cand_n[w], row, pst, rp, c, rT, lane);
    // the stage has been read: the copy of row it + depth goes into it
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      const long long nrow = row64 + (long long)depth * NW;
      if (nrow < a.N) issue_row<ESZ>(a, (int)nrow, stage, &bar[slot], pol);
    }
    if (++slot == depth) {
      slot = 0;
      phase ^= 1u;
    }
  }
  if (failed && lane == 0) {
    // A bulk copy did not complete in time: record it, then wait (bounded) for
    // this warp's copies still in flight before the shared memory goes away.
    atomicOr(a.error, 1);
    for (int d = 0; d < depth; ++d) {
      if (gw + (long long)(it + d) * NW >= a.N) break;
      if (!mbar_wait_bounded(&bar[slot], phase)) break;
      if (++slot == depth) {
        slot = 0;
        phase ^= 1u;
      }
    }
  }
}

// ---- wide kernel ----

// Rows on the hand-off list are processed in full (exact max, exact full-row
// sum, exact k-th key by bisection, bitonic sort), except entries -(row + 1):
// rows of the approximate-sum kernels whose cut needed the exact sum, which is
// computed here (one partial per thread) before warp 0 ranks the row's stored
// candidates (heads / cands) and runs the tail with the exact lse.
template <bool BF16>
__global__ void __launch_bounds__(kWideThreads) sample_wide_kernel(const KArgs a, int use_list,
                                                                    int kcap, const RowHead *heads,
                                                                    const RowCands *cands) {
  extern __shared__ unsigned long long keys[];  // [pow2 >= kcap] keys, then float scr[kcap]
  __shared__ float red_max[kWideWarps];
  __shared__ unsigned long long red_sum[kWideWarps];
  __shared__ int red_cnt[2][kWideWarps];
  __shared__ unsigned gather_n;
  int kp_cap = 2;
  while (kp_cap < kcap) kp_cap <<= 1;
  float *scr = reinterpret_cast<float *>(keys + kp_cap);  // 16-byte aligned: kp_cap is even
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int V = a.V;
  const unsigned nrows =
      use_list ? (unsigned)min((long long)*((volatile uint32_t *)a.deferred_n), (long long)a.deferred_cap)
               : (unsigned)a.N;
  for (unsigned idx = blockIdx.x; idx < nrows; idx += gridDim.x) {
    const int entry = use_list ? a.deferred[idx] : (int)idx;
    const bool exact_sum_only = entry < 0;
    const int row = exact_sum_only ? -entry - 1 : entry;
    if (a.finite && !use_list) {  // (rows handed on by the stats kernel have theirs)
      const void *b0 = row_base<BF16>(a, row);
      bool fin = true;
      for (int i = t; i < V; i += kWideThreads) fin = fin && fabsf(load_x<BF16>(b0, i)) < f_inf();
      fin = __syncthreads_and(fin);
      if (t == 0) a.finite[row] = fin ? 1 : 0;
    }
    RowP rp;
    const int pst = row_params(a, row, rp);
    if (pst != D3S_ROW_OK || rp.k > kcap) {
      if (t == 0) flag_row(a, row, D3S_ROW_BADPARAM);
      continue;
    }
    const int k = rp.k;
    if (exact_sum_only) {
      // A row of the stats kernels (V <= 8192, finite, its exact max in the
      // header): thread t's partial, all of its <= 32 elements loaded at once
      // (the row left L2 long ago), the reciprocal quotient where it is exact.
      const void *b0 = row_base<BF16>(a, row);
      const float gmax = heads[row].gmax;
      float xv[kFastMaxV / kWideThreads];
#pragma unroll
      for (int j = 0; j < kFastMaxV / kWideThreads; ++j) {
        const int i = t + kWideThreads * j;
        xv[j] = i < V ? load_x<BF16>(b0, i) : 0.0f;
      }
      const float rT = __frcp_rn(rp.T), mT = -rp.T;
      const bool recip = rp.T >= 0x1p-17f && rp.T <= 0x1p20f;
      float sp = 0.0f;
#pragma unroll
      for (int j = 0; j < kFastMaxV / kWideThreads; ++j) {
        if (t + kWideThreads * j < V) {
          const float ax = fabsf(xv[j]);
          const float q = (recip && ax >= 0x1p-100f && ax <= 0x1p60f) ? div_rows(xv[j], rT, mT)
                                                                       : __fdiv_rn(xv[j], rp.T);
          sp = __fadd_rn(sp, exp_term(__fsub_rn(q, gmax)));
        }
      }
      const unsigned long long ws = warp_sum_fixed(__float2ull_rz(__fmul_rn(sp, 0x1p46f)));
      if (lane == 0) red_sum[w] = ws;
      __syncthreads();
      if (w == 0) {
        unsigned long long Se = 0;
#pragma unroll
        for (int i = 0; i < kWideWarps; ++i) Se += red_sum[i];
        const float lse = __fadd_rn(gmax, log_full(__fmul_rn(__ull2float_rn(Se), 0x1p-46f)));
        const RowCands &Cs = cands[row];
        rank_cands(Cs.cand, Cs, heads[row].cnt, k, rp.T, keys, lane);
        __syncwarp();
        sample_tail(a, row, row_key(a, row), keys, scr, k, lse, lse, rp.p, lane);
      }
      __syncthreads();
      continue;
    }
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
    if (w == 0) sample_tail(a, row, row_key(a, row), keys, scr, k, lse, lse, rp.p, lane);
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
      case 3: r = div_rows(v, __frcp_rn(T), -T); break;
      default: r = ex2_approx(v); break;
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
      if (!(ax >= 0x1p-100f && ax <= 0x1p60f)) continue;
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

using StatFn = void (*)(const KArgs, RowHead *, RowCands *, int, int);

template <bool BF16, bool EXACT, bool SELECT>
StatFn pick_stats_e(int J) {
  switch (J) {
    case 1: return sample_stats_kernel<1, BF16, EXACT, SELECT, false>;
    case 2: return sample_stats_kernel<2, BF16, EXACT, SELECT, false>;
    case 4: return sample_stats_kernel<4, BF16, EXACT, SELECT, false>;
    case 8: return sample_stats_kernel<8, BF16, EXACT, SELECT, false>;
    case 12: return sample_stats_kernel<12, BF16, EXACT, SELECT, false>;
    case 16: return sample_stats_kernel<16, BF16, EXACT, SELECT, false>;
    case 17: return sample_stats_kernel<17, BF16, EXACT, SELECT, false>;
    case 24: return sample_stats_kernel<24, BF16, EXACT, SELECT, false>;
    case 32: return sample_stats_kernel<32, BF16, EXACT, SELECT, false>;
    default: return nullptr;
  }
}

// The approximate-sum stats kernels (large batches; the long rows that reach
// the stats + select pair have J >= 8).
template <bool BF16, bool EXACT>
StatFn pick_stats_approx_e(int J) {
  switch (J) {
    case 8: return sample_stats_kernel<8, BF16, EXACT, false, true>;
    case 12: return sample_stats_kernel<12, BF16, EXACT, false, true>;
    case 16: return sample_stats_kernel<16, BF16, EXACT, false, true>;
    case 17: return sample_stats_kernel<17, BF16, EXACT, false, true>;
    case 24: return sample_stats_kernel<24, BF16, EXACT, false, true>;
    case 32: return sample_stats_kernel<32, BF16, EXACT, false, true>;
    default: return nullptr;
  }
}

template <bool BF16, bool SELECT>
StatFn pick_stats(int J, int V) {
  return J == (V + kPartials - 1) / kPartials ? pick_stats_e<BF16, true, SELECT>(J)
                                              : pick_stats_e<BF16, false, SELECT>(J);
}

template <bool BF16>
StatFn pick_stats_approx(int J, int V) {
  return J == (V + kPartials - 1) / kPartials ? pick_stats_approx_e<BF16, true>(J)
                                              : pick_stats_approx_e<BF16, false>(J);
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

// Per device and kernel: raise the dynamic shared-memory limit once (and, when
// asked, the largest shared-memory carveout), and remember the occupancy per (threads, smem).
// The attribute calls and the occupancy query cost microseconds each, more
// than a one-row launch takes on the GPU. Returns blocks per SM, or 0 when an
// attribute call failed.
int prepare(const void *fn, int threads, size_t smem, bool max_carveout = false) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, size_t> limit;
  static std::map<std::tuple<int, const void *, int, size_t>, int> occ;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(dev, fn);
  auto it = limit.find(key);
  if (it == limit.end() || it->second < smem) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return 0;
    if (max_carveout && it == limit.end() &&
        cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
      return 0;
    limit[key] = smem;
  }
  const auto ok = std::make_tuple(dev, fn, threads, smem);
  auto jt = occ.find(ok);
  if (jt != occ.end()) return jt->second;
  const int b = occupancy(fn, threads, smem);
  occ[ok] = b;
  return b;
}

size_t wide_smem(int kcap) {
  int kp = 2;
  while (kp < kcap) kp <<= 1;
  return (size_t)kp * sizeof(unsigned long long) + (size_t)(kcap + 4) * sizeof(float);
}

template <bool BF16>
int launch_wide(const KArgs &a, int use_list, int kcap, cudaStream_t st, int max_grid = 1 << 30,
                const RowHead *heads = nullptr, const RowCands *cands = nullptr) {
  const size_t smem = wide_smem(kcap);
  auto fn = sample_wide_kernel<BF16>;
  const int occ = prepare((const void *)fn, kWideThreads, smem);
  if (occ <= 0) return D3S_ERR_CUDA;
  const int sms = device_sms();
  int grid = sms * occ;
  if (!use_list) grid = std::min(grid, a.N);
  grid = std::min(grid, max_grid);
  if (grid < 1) grid = 1;
  fn<<<grid, kWideThreads, smem, st>>>(a, use_list, kcap, heads, cands);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

// The row-independent part of the approximate full-row sum's error bound (see
// row_lse) for rows of V with J columns per stats thread, rounded up:
// 2^-24 (1.01 (5 ln V + n_p + L + 1 + 6) + 1), where n_p = ceil(V / 256) and
// L = J terms per accumulator.
float approx_bound_c0(int V, int J) {
  const double n_p = (double)((V + kPartials - 1) / kPartials);
  const double units = 1.01 * (5.0 * std::log((double)V) + n_p + (double)J + 1.0 + 6.0) + 1.0;
  return (float)std::ldexp(units, -24);
}

// The fast path: stats (K1) -> select (K2) -> wide kernel for the rows handed on.
template <bool BF16>
int launch_fast(const KArgs &a0, const Scratch &sc, int J, int wide_kcap, cudaStream_t st) {
  KArgs a = a0;
  a.approx_c0 = approx_bound_c0(a.V, J);
  constexpr int esz = BF16 ? 2 : 4;
  const int span = ((a.V * esz + 15) / 16) * 16 + 16;
  int stages = BF16 ? 3 : 2;
  while (stages > 2 && (size_t)stages * span > 64 * 1024) --stages;
  const size_t smem = (size_t)stages * span;
  // the approximate full-row sum unless the caller wants per-row finite flags
  StatFn fn = a.finite ? nullptr : pick_stats_approx<BF16>(J, a.V);
  if (!fn) fn = pick_stats<BF16, false>(J, a.V);
  if (!fn) return D3S_ERR_ARG;
  const int occ = prepare((const void *)fn, kFastThreads, smem);
  const int sms = device_sms();
  if (occ <= 0 || sms <= 0) return D3S_ERR_CUDA;
  const int grid = std::max(1, std::min(a.N, sms * occ));
  fn<<<grid, kFastThreads, smem, st>>>(a, sc.heads, sc.cands, stages, span);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  const int sel_occ = prepare((const void *)sample_select_kernel, kSelThreads, 0);
  const int sel_grid = std::max(1, std::min((a.N + kSelWarps - 1) / kSelWarps, sms * sel_occ));
  sample_select_kernel<<<sel_grid, kSelThreads, 0, st>>>(a, sc.heads, sc.cands);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  return launch_wide<BF16>(a, 1, wide_kcap, st, 1 << 30, sc.heads, sc.cands);
}

// The pair with the one-warp stats kernel: stats1 -> select -> wide kernel.
template <bool BF16, int NC>
int launch_fast1_nc(const KArgs &a0, const Scratch &sc, int wide_kcap, cudaStream_t st) {
  KArgs a = a0;
  // longest sequential chain of the approximate sum: a float of an accumulator
  // takes one term per chunk of its parity (f32) or per chunk (bf16), then
  // three levels of the final adds
  a.approx_c0 = approx_bound_c0(a.V, (BF16 ? NC : (NC + 1) / 2) + 3);
  // one stage a warp (the copy of a warp's next row starts when it has read
  // its row), as many warps as one CTA's shared memory holds stages: the pass
  // is bound by rows in flight, and warps running rows are worth more than
  // rows copied ahead
  const int depth = 1;
  const int warps = std::min(kS1MaxWarps, std::max(1, (int)((kS1SmemBytes) / (NC * 512))));
  const size_t smem = (size_t)warps * depth * NC * 512;
  auto fn = sample_stats1_kernel<NC, BF16>;
  const int occ = prepare((const void *)fn, 32 * warps, smem, true);
  const int sms = device_sms();
  if (occ <= 0 || sms <= 0) return D3S_ERR_CUDA;
  const long long need = (a.N + warps - 1) / warps;
  const int grid = (int)std::max(1LL, std::min(need, (long long)sms * occ));
  fn<<<grid, 32 * warps, smem, st>>>(a, sc.heads, sc.cands, depth);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  const int sel_occ = prepare((const void *)sample_select_kernel, kSelThreads, 0);
  const int sel_grid = std::max(1, std::min((a.N + kSelWarps - 1) / kSelWarps, sms * sel_occ));
  sample_select_kernel<<<sel_grid, kSelThreads, 0, st>>>(a, sc.heads, sc.cands);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  return launch_wide<BF16>(a, 1, wide_kcap, st, 1 << 30, sc.heads, sc.cands);
}

template <bool BF16>
int launch_fast1(const KArgs &a, const Scratch &sc, int nc, int wide_kcap, cudaStream_t st) {
  switch (nc) {
    case 17: return launch_fast1_nc<BF16, 17>(a, sc, wide_kcap, st);
    case 25: return launch_fast1_nc<BF16, 25>(a, sc, wide_kcap, st);
    case 33: return launch_fast1_nc<BF16, 33>(a, sc, wide_kcap, st);
    default: return D3S_ERR_ARG;
  }
}

// Small batches: one CTA per row runs the stats kernel's four warps and then,
// in the same launch, the select work on warp 0; the wide kernel after it
// (on at most N CTAs) takes any row handed on.
template <bool BF16>
int launch_small(const KArgs &a, const Scratch &sc, int J, int wide_kcap, cudaStream_t st) {
  constexpr int esz = BF16 ? 2 : 4;
  const int span = ((a.V * esz + 15) / 16) * 16 + 16;
  const size_t smem = std::max<size_t>((size_t)span, (size_t)kCandCap * 8 + (kFastMaxK + 4) * 4);
  StatFn fn = pick_stats<BF16, true>(J, a.V);
  if (!fn) return D3S_ERR_ARG;
  if (prepare((const void *)fn, kFastThreads, smem) <= 0) return D3S_ERR_CUDA;
  fn<<<a.N, kFastThreads, smem, st>>>(a, sc.heads, sc.cands, 1, span);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  if (a.skip_handoff) return D3S_OK;
  return launch_wide<BF16>(a, 1, wide_kcap, st, a.N);
}

template <bool BF16, int NC>
int launch_rowwarp_nc(const KArgs &a, cudaStream_t st) {
  const int stage_bytes = NC * 512;  // every chunk a lane may read
  const size_t smem = (size_t)stage_bytes + kRwTailBytes;
  auto fn = sample_rowwarp_kernel<NC, BF16>;
  const int occ = prepare((const void *)fn, 32, smem, true);
  const int sms = device_sms();
  if (occ <= 0 || sms <= 0) return D3S_ERR_CUDA;
  const int grid = std::max(1, std::min(a.N, sms * occ));
  fn<<<grid, 32, smem, st>>>(a, stage_bytes);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

// Chunks of 16 bytes a lane reads for rows of V elements (the stage starts up to
// one chunk before the row); 0 when the row-warp kernel does not take V.
template <bool BF16>
int rowwarp_nc(int V) {
  constexpr int EPC = BF16 ? 8 : 4;
  const int chunks = (V + 2 * EPC - 2) / EPC;
  const int nc = (chunks + 31) / 32;
  const int opts[] = {1, 2, 3, 5, 9, 17, 25, 33};
  for (int o : opts)
    if (nc <= o) return o;
  return 0;
}

template <bool BF16>
int launch_rowwarp(const KArgs &a, int nc, cudaStream_t st) {
  switch (nc) {
    case 1: return launch_rowwarp_nc<BF16, 1>(a, st);
    case 2: return launch_rowwarp_nc<BF16, 2>(a, st);
    case 3: return launch_rowwarp_nc<BF16, 3>(a, st);
    case 5: return launch_rowwarp_nc<BF16, 5>(a, st);
    case 9: return launch_rowwarp_nc<BF16, 9>(a, st);
    case 17: return launch_rowwarp_nc<BF16, 17>(a, st);
    case 25: return launch_rowwarp_nc<BF16, 25>(a, st);
    case 33: return launch_rowwarp_nc<BF16, 33>(a, st);
    default: return D3S_ERR_ARG;
  }
}

// Test hook: 0 = the usual choice, 1 = the four-warp stats kernel + select,
// 3 = the row-warp kernel, 4 = the one-warp stats kernel + select, for
// batches that reach the choice between them (above the small-batch path).
std::atomic<int> g_force_path{0};

template <bool BF16>
int launch_typed(const KArgs &a, const Scratch &s, cudaStream_t st) {
  const bool scalar_k = a.k_rows == nullptr;
  const int J = a.V <= kFastMaxV ? pick_J(a.V) : 0;
  const int kscalar = std::min(a.top_k, a.V);
  if (J == 0 || (scalar_k && kscalar > kFastMaxK))
    return launch_wide<BF16>(a, 0, scalar_k ? kscalar : D3S_MAX_K, st);
  if (!s.deferred || !s.counters || s.capacity < a.N) return D3S_ERR_ARG;
  // One warp per row (then the wide kernel for the rows it handed on) for short
  // rows, where the kernel is compact and many warps fit on an SM, and for
  // batches of at most one wave, where fewer launches matter more than issue
  // efficiency; long rows in large batches go to the stats + select kernels
  // (four warps share a row: more warps resident per row in flight).
  const int kcap = scalar_k ? kscalar : D3S_MAX_K;
  if (a.N <= kSmallBatch && s.heads && s.rec_capacity >= a.N)
    return launch_small<BF16>(a, s, J, kcap, st);
  const int nc = rowwarp_nc<BF16>(a.V);
  const int force = g_force_path.load(std::memory_order_relaxed);
  if (nc > 0 && (force == 3 || (force == 0 && (nc <= 9 || a.N <= kRowWarpMaxBatch)))) {
    const int rc = launch_rowwarp<BF16>(a, nc, st);
    if (rc != D3S_OK) return rc;
    return launch_wide<BF16>(a, 1, scalar_k ? kscalar : D3S_MAX_K, st);
  }
  if (!s.heads || s.rec_capacity < a.N) return D3S_ERR_ARG;
  // the stats pass by one warp per row for rows it holds (up to 33 chunks a
  // lane); the four-warp stats kernel for longer rows, for per-row finite
  // flags, and when path 1 is forced
  if (force != 1 && !a.finite && nc >= 17)
    return launch_fast1<BF16>(a, s, nc, scalar_k ? kscalar : D3S_MAX_K, st);
  return launch_fast<BF16>(a, s, J, scalar_k ? kscalar : D3S_MAX_K, st);
}

}  // namespace

int prepare_launch(const void *fn, int threads, size_t smem) { return prepare(fn, threads, smem); }

void set_force_path(int path) { g_force_path.store(path, std::memory_order_relaxed); }

int launch_sample(const KArgs &a, const Scratch &s, cudaStream_t st) {
  if (a.N == 0) return D3S_OK;
  return a.dtype == D3S_BF16 ? launch_typed<true>(a, s, st) : launch_typed<false>(a, s, st);
}

int launch_handoff(const KArgs &a, cudaStream_t st) {
  if (a.N == 0) return D3S_OK;
  const int kcap = a.k_rows ? D3S_MAX_K : std::min(a.top_k, a.V);
  return a.dtype == D3S_BF16 ? launch_wide<true>(a, 1, kcap, st, a.N)
                             : launch_wide<false>(a, 1, kcap, st, a.N);
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

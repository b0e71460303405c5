// d3s_device.cuh - device arithmetic of the sampler: exp / log, threefry and
// MLX's uniform layout, float <-> ordered-key helpers.
//
// Every float operation is an explicit round-to-nearest intrinsic (__fmaf_rn,
// __fadd_rn, __fmul_rn, __fdiv_rn), so the compiler cannot contract or reorder
// it: the results equal the CPU oracle's (oracle/d3s_oracle.c) bit for bit.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace d3s {

// Float roundings of log2(e), ln(2) (high part and the remainder), the
// coefficients of exp's polynomial on [-ln2/2, ln2/2] (p(r) = 1 + r + r^2 q(r)
// with q of degree 4, minimax for the relative error of p, derived by a
// linear program over a dense grid and rounded to float) and the atanh-series
// coefficients 1/(2j+1).
constexpr float kL2E = 0x1.715476p+0f;
constexpr float kLn2Hi = 0x1.62e430p-1f;
constexpr float kLn2Lo = -0x1.05c610p-29f;
constexpr float kShifter = 0x1.8p23f;  // adding it rounds to an integer in the low bits
constexpr uint32_t kShifterBits = 0x4B400000u;
constexpr float kE6 = 0x1.69d528p-10f;
constexpr float kE5 = 0x1.126946p-7f;
constexpr float kE4 = 0x1.55596cp-5f;
constexpr float kE3 = 0x1.55544p-3f;
constexpr float kE2 = 0x1.fffffcp-2f;
constexpr float kInv13 = 0x1.3b13b2p-4f;
constexpr float kInv11 = 0x1.745d18p-4f;
constexpr float kInv9 = 0x1.c71c72p-4f;
constexpr float kInv7 = 0x1.24924ap-3f;
constexpr float kInv5 = 0x1.99999ap-3f;
constexpr float kInv3 = 0x1.555556p-2f;
constexpr float kMinTemperature = 1e-5f;     // MIN_TEMPERATURE, src/sampling.c:16
constexpr float kUniformUpper = 0x1.fffffep-1f;  // the float below 1

__device__ __forceinline__ float f_inf() { return __int_as_float(0x7f800000); }
__device__ __forceinline__ float f_nan() { return __int_as_float(0x7fffffff); }

// max that returns NaN when either input is NaN (PTX max.NaN, sm_80+)
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
// warp-wide float max (redux.sync .f32, sm_100a); NaN-propagating
__device__ __forceinline__ float warp_max_nan(float a) {
  float d;
  asm volatile("redux.sync.max.NaN.f32 %0, %1, 0xffffffff;" : "=f"(d) : "f"(a));
  return d;
}
__device__ __forceinline__ float warp_max(float a) {
  float d;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(d) : "f"(a));
  return d;
}

// exp over the whole float range: Cody-Waite reduction against a two-float
// ln 2, the degree-6 polynomial in Horner form, exact scaling by 2^n (two
// steps outside the normal range so a subnormal result rounds once).
__device__ __forceinline__ float exp_full(float x) {
  if (x < -104.0f) return 0.0f;
  if (x > 89.0f) return f_inf();
  float t = __fmaf_rn(x, kL2E, kShifter);
  float nf = __fsub_rn(t, kShifter);
  int n = (int)(__float_as_uint(t) - kShifterBits);
  float r = __fmaf_rn(nf, -kLn2Hi, x);
  r = __fmaf_rn(nf, -kLn2Lo, r);
  float p = kE6;
  p = __fmaf_rn(p, r, kE5);
  p = __fmaf_rn(p, r, kE4);
  p = __fmaf_rn(p, r, kE3);
  p = __fmaf_rn(p, r, kE2);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int n2 = n < -126 ? -64 : (n > 127 ? 1 : 0);
  float s1 = __uint_as_float((unsigned)(n - n2 + 127) << 23);
  float s2 = __uint_as_float((unsigned)(n2 + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

// exp_full for x <= 0 (the tail's terms: quotients never exceed the row max,
// and lse is at least the max): the same arithmetic without the overflow test
// and the upward scaling step, which cannot apply there.
__device__ __forceinline__ float exp_nonpos(float x) {
  if (x < -104.0f) return 0.0f;
  float t = __fmaf_rn(x, kL2E, kShifter);
  float nf = __fsub_rn(t, kShifter);
  int n = (int)(__float_as_uint(t) - kShifterBits);
  float r = __fmaf_rn(nf, -kLn2Hi, x);
  r = __fmaf_rn(nf, -kLn2Lo, r);
  float p = kE6;
  p = __fmaf_rn(p, r, kE5);
  p = __fmaf_rn(p, r, kE4);
  p = __fmaf_rn(p, r, kE3);
  p = __fmaf_rn(p, r, kE2);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int n2 = n < -126 ? -64 : 0;
  float s1 = __uint_as_float((unsigned)(n - n2 + 127) << 23);
  float s2 = __uint_as_float((unsigned)(n2 + 127) << 23);
  return __fmul_rn(__fmul_rn(p, s1), s2);
}

// p * 2^n for p in [0.7, 1.42] and n >= -124, as integers: t = 1.5 * 2^23 + n has
// bits 0x4B400000 + n, and (0x4B400000 << 23) wraps to 0, so bits(p) + (t's bits
// << 23) adds n to p's exponent. The result is normal, so this is exactly the
// rounded product p * 2^n.
__device__ __forceinline__ float scale_pow2(float p, float t) {
  unsigned r;
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(r) : "r"(__float_as_uint(t)), "r"(__float_as_uint(p)));
  return __uint_as_float(r);
}

// 2^x by the special-function unit (ex2.approx.ftz.f32): relative error below
// 2^-22.7 wherever the result is normal (the tests measure it over every input
// in [-127, 2^-8]), subnormal results flushed to zero. It only feeds the
// approximate full-row sum, whose error bound the sampler carries into the
// top-p cut (a cut it cannot certify is recomputed with the exact sum).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One term of the full-row sum for d = q - max in [-inf, 0] (never NaN):
// exp(max(d, -86)). Below -86 a term (< 2^-124) is far under the 2^-46
// resolution of the fixed-point sum; the floor keeps n >= -124, so the result
// is normal and equals exp_full's.
constexpr float kTermFloor = -86.0f;
__device__ __forceinline__ float exp_term(float d) {
  d = fmaxf(d, kTermFloor);
  float t = __fmaf_rn(d, kL2E, kShifter);
  float nf = __fsub_rn(t, kShifter);
  float r = __fmaf_rn(nf, -kLn2Hi, d);
  r = __fmaf_rn(nf, -kLn2Lo, r);
  float p = kE6;
  p = __fmaf_rn(p, r, kE5);
  p = __fmaf_rn(p, r, kE4);
  p = __fmaf_rn(p, r, kE3);
  p = __fmaf_rn(p, r, kE2);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  return scale_pow2(p, t);
}

// Two terms at once on the packed fp32x2 pipe (sm_100a); same roundings as
// exp_term, element by element. CLAMP = false when the caller knows d >= -86.
template <bool CLAMP>
__device__ __forceinline__ float2 exp_term2(float2 d) {
  if (CLAMP) {
    d.x = fmaxf(d.x, kTermFloor);
    d.y = fmaxf(d.y, kTermFloor);
  }
  float2 t = __ffma2_rn(d, make_float2(kL2E, kL2E), make_float2(kShifter, kShifter));
  float2 nf = __fadd2_rn(t, make_float2(-kShifter, -kShifter));
  float2 r = __ffma2_rn(nf, make_float2(-kLn2Hi, -kLn2Hi), d);
  r = __ffma2_rn(nf, make_float2(-kLn2Lo, -kLn2Lo), r);
  float2 p = make_float2(kE6, kE6);
  p = __ffma2_rn(p, r, make_float2(kE5, kE5));
  p = __ffma2_rn(p, r, make_float2(kE4, kE4));
  p = __ffma2_rn(p, r, make_float2(kE3, kE3));
  p = __ffma2_rn(p, r, make_float2(kE2, kE2));
  p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
  p = __ffma2_rn(p, r, make_float2(1.0f, 1.0f));
  return make_float2(scale_pow2(p.x, t.x), scale_pow2(p.y, t.y));
}

// log: x = 2^e m, m in (sqrt2/2, sqrt2], s = (m-1)/(m+1), log m = 2 atanh(s)
// by its series to s^13, plus e ln 2 through the two-float ln 2.
__device__ __forceinline__ float log_full(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? -f_inf() : f_nan();
  if (x == f_inf()) return x;
  unsigned b = __float_as_uint(x);
  int e = 0;
  if (b < 0x00800000u) {
    x = __fmul_rn(x, 0x1p23f);
    b = __float_as_uint(x);
    e = -23;
  }
  e += (int)(b >> 23) - 127;
  b = (b & 0x007fffffu) | 0x3f800000u;
  if (b > 0x3fb504f3u) {
    b -= 0x00800000u;
    e += 1;
  }
  float m = __uint_as_float(b);
  float f = __fsub_rn(m, 1.0f);
  float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
  float z = __fmul_rn(s, s);
  float P = kInv13;
  P = __fmaf_rn(P, z, kInv11);
  P = __fmaf_rn(P, z, kInv9);
  P = __fmaf_rn(P, z, kInv7);
  P = __fmaf_rn(P, z, kInv5);
  P = __fmaf_rn(P, z, kInv3);
  float t = __fadd_rn(s, s);
  float L = __fmaf_rn(__fmul_rn(t, z), P, t);
  float ef = __int2float_rn(e);
  return __fmaf_rn(ef, kLn2Hi, __fmaf_rn(ef, kLn2Lo, L));
}

// ---- threefry-2x32-20 (Salmon et al., SC'11) and MLX's key / bits layout ----

__host__ __device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) {
#ifdef __CUDA_ARCH__
  return __funnelshift_l(x, x, r);
#else
  return (x << r) | (x >> (32 - r));
#endif
}

__host__ __device__ __forceinline__ uint2 threefry2x32(uint2 key, uint2 ctr) {
  const uint32_t k0 = key.x, k1 = key.y, k2 = key.x ^ key.y ^ 0x1BD11BDAu;
  uint32_t x0 = ctr.x + k0, x1 = ctr.y + k1;
#define D3S_TF_ROUND(r) \
  x0 += x1;             \
  x1 = rotl32(x1, r);   \
  x1 ^= x0;
#define D3S_TF_EVEN D3S_TF_ROUND(13) D3S_TF_ROUND(15) D3S_TF_ROUND(26) D3S_TF_ROUND(6)
#define D3S_TF_ODD D3S_TF_ROUND(17) D3S_TF_ROUND(29) D3S_TF_ROUND(16) D3S_TF_ROUND(24)
  D3S_TF_EVEN x0 += k1;
  x1 += k2 + 1u;
  D3S_TF_ODD x0 += k2;
  x1 += k0 + 2u;
  D3S_TF_EVEN x0 += k0;
  x1 += k1 + 3u;
  D3S_TF_ODD x0 += k1;
  x1 += k2 + 4u;
  D3S_TF_EVEN x0 += k2;
  x1 += k0 + 5u;
#undef D3S_TF_ROUND
#undef D3S_TF_EVEN
#undef D3S_TF_ODD
  return make_uint2(x0, x1);
}

// Word f of MLX's bits(key, n words): counter (i, h + o + i) gives words i and
// h + o + i for i < h = n / 2; an odd n fills word h from counter (h, 0).
__host__ __device__ __forceinline__ uint32_t bits_word(uint2 key, uint64_t n, uint64_t f) {
  const uint64_t h = n >> 1, o = n & 1;
  if (f < h) return threefry2x32(key, make_uint2((uint32_t)f, (uint32_t)(h + o + f))).x;
  if (o && f == h) return threefry2x32(key, make_uint2((uint32_t)h, 0u)).x;
  const uint64_t g = f - h - o;
  return threefry2x32(key, make_uint2((uint32_t)g, (uint32_t)(h + o + g))).y;
}

// bits_word with one threefry evaluation: the counter pair and the output
// half are selected first, so the hash is inlined once.
__device__ __forceinline__ uint32_t bits_word1(uint2 key, uint64_t n, uint64_t f) {
  const uint64_t h = n >> 1, o = n & 1;
  const bool odd_mid = o && f == h;
  const bool first = f < h || odd_mid;
  const uint64_t g = first ? f : f - h - o;
  const uint32_t c1 = odd_mid ? 0u : (uint32_t)(h + o + g);
  const uint2 r = threefry2x32(key, make_uint2((uint32_t)g, c1));
  return first ? r.x : r.y;
}

// random::key(seed)
__host__ __device__ __forceinline__ uint2 key_from_seed(uint64_t seed) {
  return make_uint2((uint32_t)(seed >> 32), (uint32_t)seed);
}
// random::split(key): bits(key, 4) read as (k0, k1)
__host__ __device__ __forceinline__ void key_split(uint2 key, uint2 &k0, uint2 &k1) {
  const uint2 a = threefry2x32(key, make_uint2(0u, 2u));
  const uint2 b = threefry2x32(key, make_uint2(1u, 3u));
  k0 = make_uint2(a.x, b.x);
  k1 = make_uint2(a.y, b.y);
}
// the subkey that d3_sample's first uniform draws from, after m_seed(seed)
__host__ __device__ __forceinline__ uint2 seed_subkey(uint64_t seed) {
  uint2 k0, k1;
  key_split(key_from_seed(seed), k0, k1);
  return k1;
}

// seed_subkey computed by a whole warp: lanes 0 and 1 evaluate the two
// threefry blocks of the split side by side (every lane must call it).
__device__ __forceinline__ uint2 seed_subkey_warp(uint64_t seed, int lane) {
  const uint32_t c = (uint32_t)(lane & 1);
  const uint2 r = threefry2x32(key_from_seed(seed), make_uint2(c, c + 2u));
  return make_uint2(__shfl_sync(0xffffffffu, r.y, 0), __shfl_sync(0xffffffffu, r.y, 1));
}

// random::uniform(0, 1, float32): float(bits) / 2^32, clamped below 1.
__device__ __forceinline__ float bits_to_uniform(uint32_t b) {
  return fminf(__fmul_rn(__uint2float_rn(b), 0x1p-32f), kUniformUpper);
}

// ---- ordered keys ----

// Order-preserving map float -> uint32 (for finite values and +-inf); -0 and +0
// map to the same key, so key order equals float comparison order.
__device__ __forceinline__ uint32_t okey(float f) {
  uint32_t b = __float_as_uint(__fadd_rn(f, 0.0f));  // -0 + 0 = +0
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float okey_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// Candidate key: value first, then the lower id (ties go to the lower id).
__device__ __forceinline__ unsigned long long cand_key(float q, uint32_t id) {
  return ((unsigned long long)okey(q) << 32) | (unsigned long long)(0xFFFFFFFFu - id);
}
__device__ __forceinline__ float cand_value(unsigned long long key) {
  return okey_to_float((uint32_t)(key >> 32));
}
__device__ __forceinline__ int32_t cand_id(unsigned long long key) {
  return (int32_t)(0xFFFFFFFFu - (uint32_t)key);
}

}  // namespace d3s

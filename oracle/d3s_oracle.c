/* d3s_oracle.c - CPU restatement of drama3-mlx's token sampler.
 *
 * TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline); see
 * d3s_oracle.h for what is restated, the parity status and the floating-point
 * conventions. Build with -ffp-contract=off and without -ffast-math: every
 * float operation below must round exactly once, as written.
 */
#include "d3s_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float u2f(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------------------ */
/* Threefry-2x32 with 20 rounds: Salmon, Moraes, Dror, Shaw, "Parallel random
 * numbers: as easy as 1, 2, 3", SC'11. Rotation schedule R_2x32 and the key
 * schedule (third word = k0 ^ k1 ^ 0x1BD11BDA, injection every 4 rounds with
 * the round-group counter) as published there. MLX's random::threefry2x32_hash
 * is this function (MLX 0.32.3, mlx/random.cpp). */
static inline uint32_t rotl32(uint32_t x, int r) { return (x << r) | (x >> (32 - r)); }

void d3o_threefry2x32(const uint32_t key[2], const uint32_t ctr[2], uint32_t out[2]) {
  static const int R[2][4] = {{13, 15, 26, 6}, {17, 29, 16, 24}};
  uint32_t ks[3] = {key[0], key[1], key[0] ^ key[1] ^ 0x1BD11BDAu};
  uint32_t x0 = ctr[0] + ks[0], x1 = ctr[1] + ks[1];
  for (int g = 0; g < 5; g++) {
    for (int j = 0; j < 4; j++) {
      x0 += x1;
      x1 = rotl32(x1, R[g & 1][j]);
      x1 ^= x0;
    }
    x0 += ks[(g + 1) % 3];
    x1 += ks[(g + 2) % 3] + (uint32_t)(g + 1);
  }
  out[0] = x0;
  out[1] = x1;
}

/* MLX random::key(seed): the high word first. */
void d3o_key_from_seed(uint64_t seed, uint32_t key[2]) {
  key[0] = (uint32_t)(seed >> 32);
  key[1] = (uint32_t)seed;
}

/* Word f of bits(key, n) for n 32-bit words under one key (MLX RandomBits):
 * with h = n / 2 and o = n % 2, counter pair (i, h + o + i) gives word i (first
 * output) and word h + o + i (second output) for i < h; an odd count fills word
 * h from counter (h, 0), first output. */
uint32_t d3o_bits_word(const uint32_t key[2], uint64_t n, uint64_t f) {
  uint64_t h = n / 2, o = n & 1;
  uint32_t c[2], r[2];
  if (f < h) {
    c[0] = (uint32_t)f;
    c[1] = (uint32_t)(h + o + f);
    d3o_threefry2x32(key, c, r);
    return r[0];
  }
  if (o && f == h) {
    c[0] = (uint32_t)h;
    c[1] = 0;
    d3o_threefry2x32(key, c, r);
    return r[0];
  }
  uint64_t g = f - h - o;
  c[0] = (uint32_t)g;
  c[1] = (uint32_t)(h + o + g);
  d3o_threefry2x32(key, c, r);
  return r[1];
}

void d3o_bits(const uint32_t key[2], uint64_t n, uint32_t *out) {
  for (uint64_t f = 0; f < n; f++) out[f] = d3o_bits_word(key, n, f);
}

/* random::split(key) = bits(key, [2, 2]) read as two keys. */
void d3o_split(const uint32_t key[2], uint32_t k0[2], uint32_t k1[2]) {
  uint32_t w[4];
  d3o_bits(key, 4, w);
  k0[0] = w[0];
  k0[1] = w[1];
  k1[0] = w[2];
  k1[1] = w[3];
}

/* KeySequence::next: the state keeps the first half of the split. */
void d3o_next_key(uint32_t state[2], uint32_t sub[2]) {
  uint32_t k0[2];
  d3o_split(state, k0, sub);
  state[0] = k0[0];
  state[1] = k0[1];
}

/* random::uniform(0, 1, float32): float(bits) / float(UINT32_MAX) (which is
 * 2^32 in float, so the divide is exact), clamped to the float below 1. */
float d3o_bits_to_uniform(uint32_t b) {
  float u = (float)b / 4294967296.0f;
  const float upper = 0x1.fffffep-1f;
  return u < upper ? u : upper;
}

void d3o_uniform(const uint32_t key[2], uint64_t n, float *out) {
  for (uint64_t f = 0; f < n; f++) out[f] = d3o_bits_to_uniform(d3o_bits_word(key, n, f));
}

/* ------------------------------------------------------------------------ */
/* exp: Cody & Waite range reduction x = n ln2 + r (n = nearest integer to
 * x log2 e, r by two fused steps against a two-float ln2), exp(r) by a
 * degree-6 polynomial p(r) = 1 + r + r^2 q(r) in Horner form, then an exact
 * scaling by 2^n (two steps when 2^n is outside the normal range, so subnormal
 * results round once). Constants: the float roundings of log2 e and ln 2 (high
 * part and low remainder); q's coefficients minimise the relative error of p on
 * [-ln2/2, ln2/2] (a linear program over a dense grid, rounded to float).
 * Error below 1 ulp over the float range. */
#define D3_L2E 0x1.715476p+0f
#define D3_LN2_HI 0x1.62e430p-1f
#define D3_LN2_LO -0x1.05c610p-29f
#define D3_SHIFTER 0x1.8p23f

float d3o_exp(float x) {
  if (x < -104.0f) return 0.0f;
  if (x > 89.0f) return INFINITY;
  float t = fmaf(x, D3_L2E, D3_SHIFTER);
  float nf = t - D3_SHIFTER;
  int32_t n = (int32_t)(f2u(t) - f2u(D3_SHIFTER));
  float r = fmaf(nf, -D3_LN2_HI, x);
  r = fmaf(nf, -D3_LN2_LO, r);
  float p = 0x1.69d528p-10f;
  p = fmaf(p, r, 0x1.126946p-7f);
  p = fmaf(p, r, 0x1.55596cp-5f);
  p = fmaf(p, r, 0x1.55544p-3f);
  p = fmaf(p, r, 0x1.fffffcp-2f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int32_t n2 = n < -126 ? -64 : (n > 127 ? 1 : 0);
  float s1 = u2f((uint32_t)(n - n2 + 127) << 23);
  float s2 = u2f((uint32_t)(n2 + 127) << 23);
  return (p * s1) * s2;
}

/* log: x = 2^e m with m in (sqrt(2)/2, sqrt(2)], f = m - 1 (exact),
 * s = f / (2 + f), log m = 2 atanh(s) = 2s (1 + s^2/3 + s^4/5 + ... + s^12/13),
 * then e ln2 added through the two-float ln2. Error below 2 ulp. */
float d3o_log(float x) {
  if (!(x > 0.0f)) return x == 0.0f ? -INFINITY : NAN;
  if (x == INFINITY) return x;
  uint32_t b = f2u(x);
  int32_t e = 0;
  if (b < 0x00800000u) { /* subnormal: normalise first */
    x = x * 0x1p23f;
    b = f2u(x);
    e = -23;
  }
  e += (int32_t)(b >> 23) - 127;
  b = (b & 0x007fffffu) | 0x3f800000u;
  if (b > 0x3fb504f3u) { /* m > sqrt(2): halve it */
    b -= 0x00800000u;
    e += 1;
  }
  float m = u2f(b);
  float f = m - 1.0f;
  float s = f / (2.0f + f);
  float z = s * s;
  float P = 0x1.3b13b2p-4f;          /* 1/13 */
  P = fmaf(P, z, 0x1.745d18p-4f);    /* 1/11 */
  P = fmaf(P, z, 0x1.c71c72p-4f);    /* 1/9 */
  P = fmaf(P, z, 0x1.24924ap-3f);    /* 1/7 */
  P = fmaf(P, z, 0x1.99999ap-3f);    /* 1/5 */
  P = fmaf(P, z, 0x1.555556p-2f);    /* 1/3 */
  float t = s + s;
  float L = fmaf(t * z, P, t);
  float ef = (float)e;
  return fmaf(ef, D3_LN2_HI, fmaf(ef, D3_LN2_LO, L));
}

/* A term of the full-row sum, d = q - max <= 0: exp(max(d, -86)). Below -86
 * the term (< 2^-124) is far under the 2^-46 resolution of the fixed-point
 * sum; the floor keeps exp's result in the normal range. NaN stays NaN (it
 * marks a non-finite row); -inf gives exp(-86). */
static float d3o_exp_term(float d) {
  if (d != d) return d;
  if (d < -86.0f) d = -86.0f;
  return d3o_exp(d);
}

void d3o_exp_array(const float *x, float *y, int64_t n) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (n > 65536)
#endif
  for (int64_t i = 0; i < n; i++) y[i] = d3o_exp(x[i]);
}
void d3o_log_array(const float *x, float *y, int64_t n) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (n > 65536)
#endif
  for (int64_t i = 0; i < n; i++) y[i] = d3o_log(x[i]);
}
void d3o_term_array(const float *x, float *y, int64_t n) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) if (n > 65536)
#endif
  for (int64_t i = 0; i < n; i++) y[i] = d3o_exp_term(x[i]);
}

/* ------------------------------------------------------------------------ */
/* top k */

typedef struct {
  float v;
  int32_t i;
} vi_t;

static int cmp_vi_desc(const void *a, const void *b) {
  const vi_t *x = a, *y = b;
  if (x->v > y->v) return -1;
  if (x->v < y->v) return 1;
  return (x->i > y->i) - (x->i < y->i);
}

/* (value desc, id asc): the order a stable descending sort gives, which is the
 * order src/sampling.c:27-36 produces (ties go to the lower id). */
void d3o_topk_stable(const float *q, int V, int k, float *vals, int32_t *ids) {
  if (k > 128) {
    vi_t *a = malloc(sizeof(vi_t) * (size_t)V);
    for (int i = 0; i < V; i++) {
      a[i].v = q[i];
      a[i].i = i;
    }
    qsort(a, (size_t)V, sizeof(vi_t), cmp_vi_desc);
    for (int r = 0; r < k; r++) {
      vals[r] = a[r].v;
      ids[r] = a[r].i;
    }
    free(a);
    return;
  }
  int n = 0;
  for (int i = 0; i < V; i++) {
    float v = q[i];
    if (n == k && !(v > vals[k - 1])) continue; /* an equal value has a higher id: it loses */
    int pos = n < k ? n : k - 1;
    while (pos > 0 && v > vals[pos - 1]) {
      vals[pos] = vals[pos - 1];
      ids[pos] = ids[pos - 1];
      pos--;
    }
    vals[pos] = v;
    ids[pos] = i;
    if (n < k) n++;
  }
}

/* The Metal kernel's selection (src/sampling.c:93-121): 32 simdgroups of 32
 * lanes, thread tid = 32 sg + lane holding q[tid + 1024 i]; each simdgroup takes
 * KS rounds of (lane best untaken, simd max, lowest id among lanes at the max),
 * then simdgroup 0 merges the 32 ranked lists in K rounds the same way. */
void d3o_topk_metal_order(const float *q, int V, int K, float *vals, int32_t *ids) {
  const int TG = 1024;
  int PER = (V + TG - 1) / TG;
  int KS = K < 32 * PER ? K : 32 * PER;
  float *lv = malloc(sizeof(float) * 32 * (size_t)KS);
  uint32_t *li = malloc(sizeof(uint32_t) * 32 * (size_t)KS);
  unsigned char *taken = calloc((size_t)TG * PER, 1);
  for (int sg = 0; sg < 32; sg++) {
    for (int r = 0; r < KS; r++) {
      float bv_l[32];
      uint32_t bi_l[32];
      int bj_l[32];
      for (int lane = 0; lane < 32; lane++) {
        int tid = sg * 32 + lane;
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        int bj = -1;
        for (int i = 0; i < PER; i++) {
          uint32_t idx = (uint32_t)(tid + i * TG);
          float v = idx < (uint32_t)V ? q[idx] : -INFINITY;
          if (idx < (uint32_t)V && !taken[tid * PER + i] && (bj < 0 || v > bv)) {
            bv = v;
            bi = idx;
            bj = i;
          }
        }
        bv_l[lane] = bv;
        bi_l[lane] = bi;
        bj_l[lane] = bj;
      }
      float best = -INFINITY;
      for (int lane = 0; lane < 32; lane++) best = bv_l[lane] > best ? bv_l[lane] : best;
      uint32_t win = 0xFFFFFFFFu;
      for (int lane = 0; lane < 32; lane++) {
        uint32_t c = (bj_l[lane] >= 0 && bv_l[lane] == best) ? bi_l[lane] : 0xFFFFFFFFu;
        win = c < win ? c : win;
      }
      for (int lane = 0; lane < 32; lane++)
        if (bj_l[lane] >= 0 && bi_l[lane] == win) taken[(sg * 32 + lane) * PER + bj_l[lane]] = 1;
      lv[sg * KS + r] = best;
      li[sg * KS + r] = win;
    }
  }
  int head[32] = {0};
  for (int r = 0; r < K; r++) {
    float best = -INFINITY;
    for (int lane = 0; lane < 32; lane++) {
      float hv = head[lane] < KS ? lv[lane * KS + head[lane]] : -INFINITY;
      best = hv > best ? hv : best;
    }
    uint32_t win = 0xFFFFFFFFu;
    for (int lane = 0; lane < 32; lane++) {
      int has = head[lane] < KS;
      float hv = has ? lv[lane * KS + head[lane]] : -INFINITY;
      uint32_t hi = has ? li[lane * KS + head[lane]] : 0xFFFFFFFFu;
      uint32_t c = hv == best ? hi : 0xFFFFFFFFu;
      win = c < win ? c : win;
    }
    for (int lane = 0; lane < 32; lane++) {
      int has = head[lane] < KS;
      uint32_t hi = has ? li[lane * KS + head[lane]] : 0xFFFFFFFFu;
      if (has && hi == win) head[lane]++;
    }
    vals[r] = best;
    ids[r] = (int32_t)win;
  }
  free(lv);
  free(li);
  free(taken);
}

/* ------------------------------------------------------------------------ */
/* the sampler */

static inline float bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

/* sample_fn (src/sampling.c:22-49) with the reduction conventions of the
 * header. x [V] logits, u [k] uniforms. */
int d3o_sample_row(const float *x, int V, float temperature, float top_p, int k,
                   const float *u, int32_t *topk_ids, float *probs, d3o_diag *diag) {
  d3o_diag dg;
  memset(&dg, 0, sizeof(dg));
  if (temperature < D3O_MIN_TEMPERATURE) temperature = D3O_MIN_TEMPERATURE; /* src/sampling.c:195 */
  float *q = malloc(sizeof(float) * (size_t)V);
  float *vals = malloc(sizeof(float) * (size_t)k);
  int32_t *ids = malloc(sizeof(int32_t) * (size_t)k);
  float gmax = -INFINITY;
  for (int i = 0; i < V; i++) {
    q[i] = x[i] / temperature; /* src/sampling.c:25 */
    if (q[i] > gmax) gmax = q[i];
  }
  /* full-row log-sum-exp (src/sampling.c:37-38) */
  uint64_t S = 0;
  int bad = 0;
  for (int p = 0; p < D3O_PARTIALS && p < V; p++) {
    float s = 0.0f;
    for (int i = p; i < V; i += D3O_PARTIALS) s = s + d3o_exp_term(q[i] - gmax);
    if (s != s)
      bad = 1;
    else
      S += (uint64_t)(s * 0x1p46f);
  }
  dg.gmax = gmax;
  dg.sum_fixed = S;
  int result = -1;
  if (bad) {
    dg.bad = 1;
    dg.lse = NAN;
    if (topk_ids)
      for (int r = 0; r < k; r++) topk_ids[r] = -1;
    if (probs)
      for (int r = 0; r < k; r++) probs[r] = 0.0f;
    goto done;
  }
  float lse = gmax + d3o_log((float)S * 0x1p-46f);
  dg.lse = lse;
  d3o_topk_stable(q, V, k, vals, ids);
  /* inclusive cumsum over the ranked top k; drop when cum > top_p and rank > 0
   * (src/sampling.c:39-43). cum never decreases, so the survivors are a prefix. */
  float cum = 0.0f;
  int kept = k;
  float margin = INFINITY;
  for (int r = 0; r < k; r++) {
    cum = cum + d3o_exp(vals[r] - lse);
    if (r > 0) {
      float m = fabsf(cum - top_p);
      if (m < margin) margin = m;
      if (cum > top_p) {
        kept = r;
        break;
      }
    }
  }
  /* softmax over the survivors (src/sampling.c:44, src/sampling.c:124-131) */
  float top = vals[0], sum = 0.0f;
  for (int r = 0; r < kept; r++) sum = sum + d3o_exp(vals[r] - top);
  float inv = 1.0f / sum;
  /* exponential race, first strictly greater score wins
   * (src/sampling.c:45-47, src/sampling.c:132-139) */
  float best = -1.0f, second = -1.0f;
  int choice = 0;
  for (int r = 0; r < k; r++) {
    float p = r < kept ? d3o_exp(vals[r] - top) * inv : 0.0f;
    float noise = -d3o_log(1.0f - u[r]);
    float score = p / noise;
    if (probs) probs[r] = p;
    if (score > best) {
      second = best;
      best = score;
      choice = r;
    } else if (score > second) {
      second = score;
    }
  }
  if (topk_ids)
    for (int r = 0; r < k; r++) topk_ids[r] = ids[r];
  dg.kept = kept;
  dg.choice = choice;
  dg.cum_margin = margin;
  dg.race_gap = best - second;
  result = ids[choice];
done:
  if (diag) *diag = dg;
  free(q);
  free(vals);
  free(ids);
  return result;
}

int d3o_row_cums(const float *x, int V, float temperature, int k, float *cums) {
  if (temperature < D3O_MIN_TEMPERATURE) temperature = D3O_MIN_TEMPERATURE;
  float *q = malloc(sizeof(float) * (size_t)V);
  float *vals = malloc(sizeof(float) * (size_t)k);
  int32_t *ids = malloc(sizeof(int32_t) * (size_t)k);
  float gmax = -INFINITY;
  for (int i = 0; i < V; i++) {
    q[i] = x[i] / temperature;
    if (q[i] > gmax) gmax = q[i];
  }
  uint64_t S = 0;
  int bad = 0;
  for (int p = 0; p < D3O_PARTIALS && p < V; p++) {
    float s = 0.0f;
    for (int i = p; i < V; i += D3O_PARTIALS) s = s + d3o_exp_term(q[i] - gmax);
    if (s != s)
      bad = 1;
    else
      S += (uint64_t)(s * 0x1p46f);
  }
  if (!bad) {
    float lse = gmax + d3o_log((float)S * 0x1p-46f);
    d3o_topk_stable(q, V, k, vals, ids);
    float cum = 0.0f;
    for (int r = 0; r < k; r++) {
      cum = cum + d3o_exp(vals[r] - lse);
      cums[r] = cum;
    }
  }
  free(q);
  free(vals);
  free(ids);
  return bad ? -1 : 0;
}

double d3o_exp_max_relerr(float lo, float hi) {
  double worst = 0.0;
  const uint32_t b_lo = f2u(hi) | 0x80000000u, b_hi = f2u(lo); /* -|hi| .. -|lo|, bits ascending */
#ifdef _OPENMP
#pragma omp parallel for reduction(max : worst) schedule(static)
#endif
  for (int64_t b = (int64_t)b_lo; b <= (int64_t)b_hi; b++) {
    const float d = u2f((uint32_t)b);
    const double r = exp((double)d);
    const double e = fabs((double)d3o_exp(d) - r) / r;
    if (e > worst) worst = e;
  }
  return worst;
}

int64_t d3o_log_nonmonotone(float lo, float hi) {
  int64_t bad = 0;
  const uint32_t b_lo = f2u(lo), b_hi = f2u(hi);
#ifdef _OPENMP
#pragma omp parallel for reduction(+ : bad) schedule(static)
#endif
  for (int64_t b = (int64_t)b_lo; b < (int64_t)b_hi; b++)
    if (d3o_log(u2f((uint32_t)b + 1u)) < d3o_log(u2f((uint32_t)b))) bad++;
  return bad;
}

static void row_to_f32(const void *logits, int dtype, int64_t ld, int row, int V, float *dst) {
  if (dtype == D3O_BF16) {
    const uint16_t *src = (const uint16_t *)logits + (int64_t)row * ld;
    for (int i = 0; i < V; i++) dst[i] = bf16_to_f32(src[i]);
  } else {
    memcpy(dst, (const float *)logits + (int64_t)row * ld, sizeof(float) * (size_t)V);
  }
}

int d3o_sample_with_noise(const void *logits, int dtype, int N, int V, int64_t ld,
                          const float *u, int k, float temperature, float top_p,
                          int32_t *ids, int nthreads) {
  int nbad = 0;
#ifdef _OPENMP
  if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(+ : nbad)
#endif
  {
    float *x = malloc(sizeof(float) * (size_t)V);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
    for (int r = 0; r < N; r++) {
      row_to_f32(logits, dtype, ld, r, V, x);
      ids[r] = d3o_sample_row(x, V, temperature, top_p, k, u + (int64_t)r * k, NULL, NULL, NULL);
      if (ids[r] < 0) nbad++;
    }
    free(x);
  }
  (void)nthreads;
  return nbad;
}

int d3o_sample_top_k_top_p(uint32_t state[2], const void *logits, int dtype, int N, int V,
                           int64_t ld, float temperature, int top_k, float top_p,
                           int32_t *ids, int nthreads) {
  int k = top_k < V ? top_k : V; /* src/sampling.c:207 */
  uint32_t sub[2];
  d3o_next_key(state, sub);
  float *u = malloc(sizeof(float) * (size_t)N * (size_t)k);
  d3o_uniform(sub, (uint64_t)N * (uint64_t)k, u);
  int nbad = d3o_sample_with_noise(logits, dtype, N, V, ld, u, k, temperature, top_p, ids, nthreads);
  free(u);
  return nbad;
}

void d3o_d3_sample(const float *logits, int N, int V, float temperature, int top_k,
                   float top_p, uint64_t seed, int32_t *out) {
  uint32_t state[2];
  d3o_key_from_seed(seed, state); /* m_seed(seed), src/testapi.c:159 */
  d3o_sample_top_k_top_p(state, logits, D3O_F32, N, V, V, temperature, top_k, top_p, out, 1);
}

int d3o_sample_rows(const void *logits, int dtype, int N, int V, int64_t ld,
                    const float *temperature, const float *top_p, const int32_t *top_k,
                    const uint64_t *seeds, float temperature_all, float top_p_all,
                    int top_k_all, uint64_t seed_all, int32_t *ids, int nthreads) {
  int nbad = 0;
#ifdef _OPENMP
  if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(+ : nbad)
#endif
  {
    float *x = malloc(sizeof(float) * (size_t)V);
    float *u = malloc(sizeof(float) * (size_t)V);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
    for (int r = 0; r < N; r++) {
      float T = temperature ? temperature[r] : temperature_all;
      float p = top_p ? top_p[r] : top_p_all;
      int tk = top_k ? top_k[r] : top_k_all;
      uint64_t seed = seeds ? seeds[r] : seed_all;
      if (tk < 1 || T != T) {
        ids[r] = -1;
        nbad++;
        continue;
      }
      int k = tk < V ? tk : V;
      uint32_t state[2], sub[2];
      d3o_key_from_seed(seed, state);
      d3o_next_key(state, sub);
      d3o_uniform(sub, (uint64_t)k, u);
      row_to_f32(logits, dtype, ld, r, V, x);
      ids[r] = d3o_sample_row(x, V, T, p, k, u, NULL, NULL, NULL);
      if (ids[r] < 0) nbad++;
    }
    free(x);
    free(u);
  }
  (void)nthreads;
  return nbad;
}

void d3o_frame_noise(uint32_t state[2], int n_draws, const int *ks, float *u) {
  for (int d = 0; d < n_draws; d++) {
    uint32_t sub[2];
    d3o_next_key(state, sub);
    d3o_uniform(sub, (uint64_t)ks[d], u);
    u += ks[d];
  }
}

int d3o_sample_rows_keys(const void *logits, int dtype, int N, int V, int64_t ld,
                         const float *temperature, const float *top_p, const int32_t *top_k,
                         float temperature_all, float top_p_all, int top_k_all,
                         const uint32_t *keys, int64_t ld_keys, int32_t *ids, int nthreads) {
  int nbad = 0;
  if (ld_keys < 1) ld_keys = 1;
#ifdef _OPENMP
  if (nthreads < 1) nthreads = omp_get_max_threads();
#pragma omp parallel num_threads(nthreads) reduction(+ : nbad)
#endif
  {
    float *x = malloc(sizeof(float) * (size_t)V);
    float *u = malloc(sizeof(float) * (size_t)V);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
    for (int r = 0; r < N; r++) {
      float T = temperature ? temperature[r] : temperature_all;
      float p = top_p ? top_p[r] : top_p_all;
      int tk = top_k ? top_k[r] : top_k_all;
      if (tk < 1 || T != T) {
        ids[r] = -1;
        nbad++;
        continue;
      }
      int k = tk < V ? tk : V;
      d3o_uniform(keys + 2 * (size_t)r * (size_t)ld_keys, (uint64_t)k, u);
      row_to_f32(logits, dtype, ld, r, V, x);
      ids[r] = d3o_sample_row(x, V, T, p, k, u, NULL, NULL, NULL);
      if (ids[r] < 0) nbad++;
    }
    free(x);
    free(u);
  }
  (void)nthreads;
  return nbad;
}

static int32_t candidate_token(int32_t idx, int semantic_start, int eos_id) {
  return idx == 0 ? eos_id : idx + semantic_start - 1; /* src/tower.c:405-409 */
}

static int is_semantic(int32_t tok, int semantic_start, int code_vocab) {
  return tok >= semantic_start && tok <= semantic_start + code_vocab - 1; /* src/tower.c:357-360 */
}

void d3o_frame_main(const void *logits, int dtype, int V, float temperature, float top_p,
                    int top_k, const uint32_t key_main[2], const uint32_t key_retry[2],
                    const int32_t *history, int hist_len, int semantic_start, int code_vocab,
                    int eos_id, int32_t *main_tok, int32_t *c0, int32_t *flags) {
  float *x = malloc(sizeof(float) * (size_t)V);
  float *u = malloc(sizeof(float) * (size_t)V);
  row_to_f32(logits, dtype, V, 0, V, x);
  int finite = 1;
  for (int i = 0; i < V; i++)
    if (!(x[i] == x[i]) || x[i] == INFINITY || x[i] == -INFINITY) finite = 0;
  int f = finite ? 0 : D3O_FRAME_NONFINITE;
  /* noise[0] and noise[1] of the frame (src/tower.c:420-421), k = min(top_k, V) */
  const int km = top_k < V ? top_k : V;
  const int kr = D3O_RAS_TOP_K < V ? D3O_RAS_TOP_K : V;
  int32_t first = -1, retry = -1;
  if (top_k >= 1 && temperature == temperature) {
    d3o_uniform(key_main, (uint64_t)km, u);
    first = d3o_sample_row(x, V, temperature, top_p, km, u, NULL, NULL, NULL);
  }
  d3o_uniform(key_retry, (uint64_t)kr, u);
  retry = d3o_sample_row(x, V, D3O_RAS_TEMPERATURE, D3O_RAS_TOP_P, kr, u, NULL, NULL, NULL);
  int32_t tok = -1;
  if (first >= 0 && retry >= 0) {
    const int32_t t1 = candidate_token(first, semantic_start, eos_id);
    const int32_t t2 = candidate_token(retry, semantic_start, eos_id);
    int seen = 0;
    for (int i = 0; i < hist_len; i++) seen |= history[i] == t1;
    /* only audio tokens are resampled; a stop is never redrawn (src/tower.c:429-433) */
    const int repeated = seen && is_semantic(t1, semantic_start, code_vocab);
    tok = repeated ? t2 : t1;
    if (repeated) f |= D3O_FRAME_RETRY;
    if (tok == eos_id) f |= D3O_FRAME_EOS;
  } else {
    f |= D3O_FRAME_NONFINITE;
  }
  int32_t c = tok - semantic_start;
  if (tok < 0) c = 0;
  c = c < 0 ? 0 : (c > code_vocab - 1 ? code_vocab - 1 : c);
  *main_tok = tok;
  *c0 = c;
  *flags = f;
  free(x);
  free(u);
}

void d3o_history_push(int32_t *history, int *hist_len, int32_t tok) {
  if (*hist_len == D3O_RAS_WINDOW) {
    for (int i = 1; i < D3O_RAS_WINDOW; i++) history[i - 1] = history[i];
    history[D3O_RAS_WINDOW - 1] = tok;
  } else {
    history[(*hist_len)++] = tok;
  }
}

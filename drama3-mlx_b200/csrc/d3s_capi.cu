// d3s_capi.cu - the C ABI declared in include/d3s.h: keys, contexts, argument
// checks, and the entry points that mirror drama3-mlx's sampling interface
// (src/model.h:169-176, src/testapi.c:155-166). No entry point exits the
// process; errors come back as D3S_ERR_* codes with a message.
#include <algorithm>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <chrono>
#include <cstring>
#include <mutex>
#include <string>

#include "d3s.h"
#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

struct d3s_ctx {
  int device = 0;
  d3s::Scratch scratch;
  // d3_sample's device staging: the logits, then at a 16-byte boundary the
  // call's error word (+ 12 bytes of padding), its N ids and its N statuses
  unsigned char *stage_dev = nullptr;
  size_t stage_cap = 0;  // bytes
  cudaStream_t stream = nullptr;
  d3s::FrameScratch frame;  // d3s_frame_main's per-draw arrays
  void *pinned = nullptr;   // d3_sample's host staging (stage_cap bytes), laid out as stage_dev
  // d3_sample of one row: the logits and the result in pinned host memory
  // mapped into the device, read and written by the kernel in place
  unsigned char *row_host = nullptr;  // [logits | id, status]
  unsigned char *row_dev = nullptr;   // the same bytes, device address
  size_t row_cap = 0;                 // bytes
};

namespace {

thread_local std::string g_err;
thread_local int g_last_status = D3S_OK;
std::mutex g_key_mu;
d3s_key g_key = {{0u, 0u}};  // the library's global key (MLX seeds its own from time)

int fail(int code, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char *what) {
  return fail(D3S_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceGuard {
  int prev = -1;
  bool ok = true;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

int reserve_records(d3s_ctx *ctx, int64_t rows) {
  if (ctx->scratch.rec_capacity >= rows) return D3S_OK;
  const int64_t cap = std::max<int64_t>(rows, 1024);
  d3s::RowHead *h = nullptr;
  d3s::RowCands *c = nullptr;
  cudaError_t e = cudaMalloc(&h, (size_t)cap * sizeof(d3s::RowHead));
  if (e == cudaSuccess) e = cudaMalloc(&c, (size_t)cap * sizeof(d3s::RowCands));
  if (e != cudaSuccess) {
    if (h) cudaFree(h);
    return fail(D3S_ERR_NOMEM, "row records: %s", cudaGetErrorString(e));
  }
  if (ctx->scratch.heads) {
    cudaDeviceSynchronize();  // the old records may be in use by queued work
    cudaFree(ctx->scratch.heads);
    cudaFree(ctx->scratch.cands);
  }
  ctx->scratch.heads = h;
  ctx->scratch.cands = c;
  ctx->scratch.rec_capacity = cap;
  return D3S_OK;
}

int reserve_scratch(d3s_ctx *ctx, int64_t rows) {
  const int rc = reserve_records(ctx, rows);
  if (rc != D3S_OK) return rc;
  if (ctx->scratch.capacity >= rows) return D3S_OK;
  int64_t cap = std::max<int64_t>(rows, 1024);
  int32_t *d = nullptr;
  uint32_t *c = nullptr;
  cudaError_t e = cudaMalloc(&d, (size_t)cap * sizeof(int32_t));
  if (e != cudaSuccess) return fail(D3S_ERR_NOMEM, "scratch: %s", cudaGetErrorString(e));
  if (!ctx->scratch.counters) {
    e = cudaMalloc(&c, 3 * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(c, 0, 3 * sizeof(uint32_t));
    if (e != cudaSuccess) {
      cudaFree(d);
      if (c) cudaFree(c);
      return fail(D3S_ERR_NOMEM, "scratch counters: %s", cudaGetErrorString(e));
    }
    ctx->scratch.counters = c;
  }
  if (ctx->scratch.deferred) {
    cudaDeviceSynchronize();  // the old list may be in use by queued work
    cudaFree(ctx->scratch.deferred);
  }
  ctx->scratch.deferred = d;
  ctx->scratch.capacity = cap;
  return D3S_OK;
}

int check_request(const d3s_request *r) {
  if (!r) return fail(D3S_ERR_ARG, "null request");
  if (r->N < 0 || r->V < 1) return fail(D3S_ERR_ARG, "bad shape N=%d V=%d", r->N, r->V);
  if (r->V > D3S_MAX_V) return fail(D3S_ERR_UNSUPPORTED, "V=%d exceeds %d", r->V, D3S_MAX_V);
  if (r->dtype != D3S_F32 && r->dtype != D3S_BF16) return fail(D3S_ERR_ARG, "bad dtype %d", r->dtype);
  if (r->ld < r->V) return fail(D3S_ERR_ARG, "ld=%lld < V=%d", (long long)r->ld, r->V);
  if (r->N > 0 && (!r->logits || !r->ids)) return fail(D3S_ERR_ARG, "null logits or ids");
  if (!r->top_k_rows) {
    if (r->top_k < 1) return fail(D3S_ERR_ARG, "top_k=%d < 1", r->top_k);
    if (std::min(r->top_k, r->V) > D3S_MAX_K)
      return fail(D3S_ERR_UNSUPPORTED, "k=%d exceeds %d", std::min(r->top_k, r->V), D3S_MAX_K);
  }
  if (!r->temperature_rows && r->temperature != r->temperature)
    return fail(D3S_ERR_ARG, "temperature is NaN");
  switch (r->noise) {
    case D3S_NOISE_KEY: {
      if (r->top_k_rows) return fail(D3S_ERR_ARG, "one-key noise needs one top_k for the batch");
      const uint64_t words = (uint64_t)r->N * (uint64_t)std::min(r->top_k, r->V);
      if (words >= (1ull << 32)) return fail(D3S_ERR_UNSUPPORTED, "N*k >= 2^32 uniform words");
      break;
    }
    case D3S_NOISE_SEEDS:
      if (r->N > 0 && !r->seeds) return fail(D3S_ERR_ARG, "null seeds");
      break;
    case D3S_NOISE_KEYS:
      if (r->N > 0 && !r->keys) return fail(D3S_ERR_ARG, "null keys");
      if (((uintptr_t)r->keys & 7) != 0) return fail(D3S_ERR_ARG, "keys must be 8-byte aligned");
      if (r->ld_keys < 0) return fail(D3S_ERR_ARG, "ld_keys < 0");
      break;
    case D3S_NOISE_GIVEN:
      if (r->N > 0 && !r->u) return fail(D3S_ERR_ARG, "null u");
      if (r->top_k_rows) return fail(D3S_ERR_ARG, "given noise needs one top_k for the batch");
      if (r->ld_u < std::min(r->top_k, r->V)) return fail(D3S_ERR_ARG, "ld_u < k");
      break;
    default:
      return fail(D3S_ERR_ARG, "bad noise mode %d", r->noise);
  }
  if ((r->probs || r->topk_ids)) {
    const int kmax = r->top_k_rows ? D3S_MAX_K : std::min(r->top_k, r->V);
    if (r->ld_out < std::min(kmax, r->V)) return fail(D3S_ERR_ARG, "ld_out too small");
  }
  return D3S_OK;
}

d3s::KArgs to_kargs(const d3s_request *r, const d3s_ctx *ctx) {
  d3s::KArgs a{};
  a.logits = r->logits;
  a.ld = r->ld;
  a.dtype = r->dtype;
  a.N = r->N;
  a.V = r->V;
  a.T = r->temperature;
  a.top_p = r->top_p;
  a.top_k = r->top_k;
  a.T_rows = r->temperature_rows;
  a.p_rows = r->top_p_rows;
  a.k_rows = r->top_k_rows;
  a.noise = r->noise;
  a.key = make_uint2(r->key.k[0], r->key.k[1]);
  a.seeds = r->seeds;
  a.u = r->u;
  a.ld_u = r->ld_u;
  a.ids = r->ids;
  a.status = r->status;
  a.kept = r->kept;
  a.probs = r->probs;
  a.topk_ids = r->topk_ids;
  a.ld_out = r->ld_out;
  a.keys = reinterpret_cast<const uint2 *>(r->keys);
  a.ld_keys = r->ld_keys > 0 ? r->ld_keys : 1;
  a.finite = r->finite;
  a.row_period = 0;
  a.deferred = ctx->scratch.deferred;
  a.deferred_n = ctx->scratch.counters;
  a.wide_done = ctx->scratch.counters ? ctx->scratch.counters + 1 : nullptr;
  a.deferred_cap = ctx->scratch.capacity;
  a.error = ctx->scratch.counters ? reinterpret_cast<int32_t *>(ctx->scratch.counters + 2) : nullptr;
  return a;
}

int next_key_locked(d3s_key *state, d3s_key *sub) {
  uint2 k0, k1;
  d3s::key_split(make_uint2(state->k[0], state->k[1]), k0, k1);
  state->k[0] = k0.x;
  state->k[1] = k0.y;
  sub->k[0] = k1.x;
  sub->k[1] = k1.y;
  return D3S_OK;
}

int take_subkey(d3s_key *state, d3s_key *sub) {
  if (state) return next_key_locked(state, sub);
  std::lock_guard<std::mutex> lk(g_key_mu);
  return next_key_locked(&g_key, sub);
}

}  // namespace

int d3s::set_error(int code, const char *msg) { return fail(code, "%s", msg); }

namespace {

// One allocation holds the 2S-entry arrays of d3s_frame_main.
int reserve_frame(d3s_ctx *ctx, int64_t streams) {
  d3s::FrameScratch &f = ctx->frame;
  if (f.capacity >= streams) return D3S_OK;
  const int64_t cap = std::max<int64_t>(streams, 256), n = 2 * cap;
  const size_t bytes = (size_t)n * (sizeof(uint2) + 2 * sizeof(float) + 3 * sizeof(int32_t));
  unsigned char *base = nullptr;
  const cudaError_t e = cudaMalloc(&base, bytes);
  if (e != cudaSuccess) return fail(D3S_ERR_NOMEM, "frame scratch: %s", cudaGetErrorString(e));
  if (f.keys) {
    cudaDeviceSynchronize();  // queued frames may still use the old arrays
    cudaFree(f.keys);         // the allocation's base
  }
  // keys first: the one 8-byte type keeps its alignment
  f.keys = reinterpret_cast<uint2 *>(base);
  f.T = reinterpret_cast<float *>(f.keys + n);
  f.p = f.T + n;
  f.k = reinterpret_cast<int32_t *>(f.p + n);
  f.ids = f.k + n;
  f.finite = f.ids + n;
  f.capacity = cap;
  return D3S_OK;
}

}  // namespace

extern "C" {

int d3s_version(void) { return D3S_VERSION; }

const char *d3s_last_error(void) { return g_err.c_str(); }

int d3s_key_from_seed(uint64_t seed, d3s_key *out) {
  if (!out) return fail(D3S_ERR_ARG, "null key");
  const uint2 k = d3s::key_from_seed(seed);
  out->k[0] = k.x;
  out->k[1] = k.y;
  return D3S_OK;
}

int d3s_key_split(const d3s_key *key, d3s_key *k0, d3s_key *k1) {
  if (!key || !k0 || !k1) return fail(D3S_ERR_ARG, "null key");
  uint2 a, b;
  d3s::key_split(make_uint2(key->k[0], key->k[1]), a, b);
  k0->k[0] = a.x;
  k0->k[1] = a.y;
  k1->k[0] = b.x;
  k1->k[1] = b.y;
  return D3S_OK;
}

int d3s_seed(d3s_key *state, uint64_t seed) {
  const uint2 k = d3s::key_from_seed(seed);
  if (state) {
    state->k[0] = k.x;
    state->k[1] = k.y;
    return D3S_OK;
  }
  std::lock_guard<std::mutex> lk(g_key_mu);
  g_key.k[0] = k.x;
  g_key.k[1] = k.y;
  return D3S_OK;
}

int d3s_next_key(d3s_key *state, d3s_key *sub) {
  if (!sub) return fail(D3S_ERR_ARG, "null subkey");
  return take_subkey(state, sub);
}

int d3s_ctx_create(int device, d3s_ctx **out) {
  if (!out) return fail(D3S_ERR_ARG, "null out");
  *out = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(D3S_ERR_ARG, "device %d of %d", device, n);
  DeviceGuard g(device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  d3s_ctx *c = new d3s_ctx();
  c->device = device;
  int rc = reserve_scratch(c, 1024);
  if (rc != D3S_OK) {
    delete c;
    return rc;
  }
  *out = c;
  return D3S_OK;
}

int d3s_ctx_reserve(d3s_ctx *ctx, int64_t max_rows) {
  if (!ctx || max_rows < 0) return fail(D3S_ERR_ARG, "bad ctx / rows");
  DeviceGuard g(ctx->device);
  return reserve_scratch(ctx, max_rows);
}

void d3s_ctx_destroy(d3s_ctx *ctx) {
  if (!ctx) return;
  DeviceGuard g(ctx->device);
  cudaDeviceSynchronize();
  cudaFree(ctx->scratch.deferred);
  cudaFree(ctx->scratch.counters);
  cudaFree(ctx->scratch.heads);
  cudaFree(ctx->scratch.cands);
  cudaFreeHost(ctx->row_host);
  cudaFree(ctx->stage_dev);
  cudaFreeHost(ctx->pinned);
  cudaFree(ctx->frame.keys);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

int d3s_sample(d3s_ctx *ctx, const d3s_request *req, void *stream) {
  if (!ctx) return fail(D3S_ERR_ARG, "null ctx");
  int rc = check_request(req);
  if (rc != D3S_OK) return rc;
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  rc = reserve_scratch(ctx, req->N);
  if (rc != D3S_OK) return rc;
  const d3s::KArgs a = to_kargs(req, ctx);
  rc = d3s::launch_sample(a, ctx->scratch, (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "sampler launch");
  return D3S_OK;
}

int d3s_sample_noise(d3s_ctx *ctx, d3s_key *state, int rows, int V, int top_k, float *u_dev,
                     void *stream) {
  if (!ctx) return fail(D3S_ERR_ARG, "null ctx");
  if (rows < 0 || V < 1 || top_k < 1) return fail(D3S_ERR_ARG, "bad rows/V/top_k");
  if (rows > 0 && !u_dev) return fail(D3S_ERR_ARG, "null u");
  const int k = std::min(top_k, V);
  if ((uint64_t)rows * (uint64_t)k >= (1ull << 32))
    return fail(D3S_ERR_UNSUPPORTED, "rows*k >= 2^32 uniform words");
  d3s_key sub;
  take_subkey(state, &sub);
  DeviceGuard g(ctx->device);
  const int rc = d3s::launch_uniform(make_uint2(sub.k[0], sub.k[1]), rows, k, u_dev,
                                     (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "uniform launch");
  return D3S_OK;
}

int d3s_sample_with_noise(d3s_ctx *ctx, const void *logits_dev, int dtype, int N, int V,
                          int64_t ld, const float *u_dev, int k, int64_t ld_u, float temperature,
                          float top_p, int32_t *ids_dev, void *stream) {
  if (k < 1 || k > V) return fail(D3S_ERR_ARG, "k=%d must be in [1, V=%d]", k, V);
  d3s_request r{};
  r.logits = logits_dev;
  r.dtype = dtype;
  r.N = N;
  r.V = V;
  r.ld = ld;
  r.temperature = temperature;
  r.top_p = top_p;
  r.top_k = k;
  r.noise = D3S_NOISE_GIVEN;
  r.u = u_dev;
  r.ld_u = ld_u;
  r.ids = ids_dev;
  return d3s_sample(ctx, &r, stream);
}

int d3s_sample_top_k_top_p(d3s_ctx *ctx, const void *logits_dev, int dtype, int N, int V,
                           int64_t ld, float temperature, int top_k, float top_p, d3s_key *state,
                           int32_t *ids_dev, void *stream) {
  d3s_request r{};
  r.logits = logits_dev;
  r.dtype = dtype;
  r.N = N;
  r.V = V;
  r.ld = ld;
  r.temperature = temperature;
  r.top_p = top_p;
  r.top_k = top_k;
  r.noise = D3S_NOISE_KEY;
  r.ids = ids_dev;
  int rc = check_request(&r);
  if (rc != D3S_OK) return rc;
  d3s_key sub;
  take_subkey(state, &sub);  // the key advances only for a valid call
  r.key = sub;
  return d3s_sample(ctx, &r, stream);
}

int d3s_debug_math(d3s_ctx *ctx, int op, const float *x_dev, float *y_dev, int64_t n,
                   float param, void *stream) {
  if (!ctx || op < 0 || op > 4 || n < 0) return fail(D3S_ERR_ARG, "bad math args");
  DeviceGuard g(ctx->device);
  const int rc = d3s::launch_math(op, x_dev, y_dev, n, param, (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "math launch");
  return D3S_OK;
}

int d3s_debug_div_check(d3s_ctx *ctx, const float *T_dev, int nT, uint64_t lo, uint64_t hi,
                        uint64_t step, unsigned long long *bad_dev, float *example_dev,
                        void *stream) {
  if (!ctx || !T_dev || nT < 0 || step == 0 || hi < lo || hi > (1ull << 32) || !bad_dev ||
      !example_dev)
    return fail(D3S_ERR_ARG, "bad division-check args");
  DeviceGuard g(ctx->device);
  const int rc = d3s::launch_div_check(T_dev, nT, lo, hi, step, bad_dev, example_dev,
                                       (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "division check launch");
  return D3S_OK;
}

int d3s_debug_force_path(int path) {
  if (path != 0 && path != 1 && path != 3 && path != 4)
    return fail(D3S_ERR_ARG, "path %d not 0, 1, 3 or 4", path);
  d3s::set_force_path(path);
  return D3S_OK;
}

int d3s_ctx_check(d3s_ctx *ctx) {
  if (!ctx) return fail(D3S_ERR_ARG, "null ctx");
  DeviceGuard g(ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "device");
  if (!ctx->scratch.counters) return D3S_OK;
  uint32_t err = 0;
  e = cudaMemcpy(&err, ctx->scratch.counters + 2, sizeof(err), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "error word");
  if (err) {
    cudaMemset(ctx->scratch.counters + 2, 0, sizeof(uint32_t));
    return fail(D3S_ERR_CUDA, "a sampler kernel gave up waiting for a row copy (rows left unsampled)");
  }
  return D3S_OK;
}

// ---- one decode frame ----

int d3s_keys_next(d3s_ctx *ctx, d3s_key *state_dev, int S, int n, d3s_key *sub_dev,
                  int64_t ld_sub, void *stream) {
  if (!ctx) return fail(D3S_ERR_ARG, "null ctx");
  if (S < 0 || n < 0) return fail(D3S_ERR_ARG, "bad S=%d / n=%d", S, n);
  if (S > 0 && n > 0 && (!state_dev || !sub_dev)) return fail(D3S_ERR_ARG, "null state or sub");
  if (ld_sub < n) return fail(D3S_ERR_ARG, "ld_sub=%lld < n=%d", (long long)ld_sub, n);
  if ((((uintptr_t)state_dev | (uintptr_t)sub_dev) & 7) != 0)
    return fail(D3S_ERR_ARG, "key arrays must be 8-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  const int rc = d3s::launch_keys_next(reinterpret_cast<uint2 *>(state_dev), S, n,
                                       reinterpret_cast<uint2 *>(sub_dev), ld_sub,
                                       (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "key launch");
  return D3S_OK;
}

int d3s_frame_main(d3s_ctx *ctx, const d3s_frame_request *f, void *stream) {
  if (!ctx || !f) return fail(D3S_ERR_ARG, "null ctx or request");
  if (f->S < 0 || f->V < 1) return fail(D3S_ERR_ARG, "bad shape S=%d V=%d", f->S, f->V);
  if (f->V > D3S_MAX_V) return fail(D3S_ERR_UNSUPPORTED, "V=%d exceeds %d", f->V, D3S_MAX_V);
  if (f->dtype != D3S_F32 && f->dtype != D3S_BF16) return fail(D3S_ERR_ARG, "bad dtype %d", f->dtype);
  if (f->ld < f->V) return fail(D3S_ERR_ARG, "ld < V");
  if (f->top_k < 1) return fail(D3S_ERR_ARG, "top_k=%d < 1", f->top_k);
  if (std::min(f->top_k, f->V) > D3S_MAX_K)
    return fail(D3S_ERR_UNSUPPORTED, "k=%d exceeds %d", std::min(f->top_k, f->V), D3S_MAX_K);
  if (f->temperature != f->temperature) return fail(D3S_ERR_ARG, "temperature is NaN");
  if (f->code_vocab < 1) return fail(D3S_ERR_ARG, "code_vocab=%d < 1", f->code_vocab);
  if (f->ld_keys < 2) return fail(D3S_ERR_ARG, "ld_keys=%lld < 2", (long long)f->ld_keys);
  if (f->S > 0 && (!f->logits || !f->keys || !f->history || !f->hist_len || !f->main_tok || !f->c0))
    return fail(D3S_ERR_ARG, "null logits / keys / history / hist_len / main_tok / c0");
  if (((uintptr_t)f->keys & 7) != 0) return fail(D3S_ERR_ARG, "keys must be 8-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  int rc = reserve_scratch(ctx, 2 * (int64_t)f->S);
  if (rc == D3S_OK) rc = reserve_frame(ctx, f->S);
  if (rc != D3S_OK) return rc;
  d3s_request r{};
  r.logits = f->logits;
  r.dtype = f->dtype;
  r.N = 2 * f->S;
  r.V = f->V;
  r.ld = f->ld;
  r.noise = D3S_NOISE_KEYS;
  const d3s::KArgs a = to_kargs(&r, ctx);
  d3s::FrameArgs fa;
  fa.S = f->S;
  fa.temperature = f->temperature;
  fa.top_p = f->top_p;
  fa.top_k = f->top_k;
  fa.keys = reinterpret_cast<const uint2 *>(f->keys);
  fa.ld_keys = f->ld_keys;
  fa.history = f->history;
  fa.hist_len = f->hist_len;
  fa.semantic_start = f->semantic_start;
  fa.code_vocab = f->code_vocab;
  fa.eos_id = f->eos_id;
  fa.update_history = f->update_history;
  fa.main_tok = f->main_tok;
  fa.c0 = f->c0;
  fa.flags = f->flags;
  rc = d3s::launch_frame(fa, ctx->frame, a, ctx->scratch, (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "frame launch");
  return D3S_OK;
}

// ---- the lm_head projection ----

static int check_lmhead(const void *h, int64_t ld_h, const void *W, int64_t ld_w, int B, int V,
                        int D, const void *out, int64_t ld_out) {
  if (B < 0 || V < 1 || D < 8) return fail(D3S_ERR_ARG, "bad shape B=%d V=%d D=%d", B, V, D);
  if (V > D3S_MAX_V) return fail(D3S_ERR_UNSUPPORTED, "V=%d exceeds %d", V, D3S_MAX_V);
  if (B > 0 && (!h || !W || !out)) return fail(D3S_ERR_ARG, "null h / W / logits");
  if (D % 8 || ld_h < D || ld_w < D || ld_h % 8 || ld_w % 8 || ld_out < V)
    return fail(D3S_ERR_ARG, "D, ld_h, ld_w must be multiples of 8 (16-byte rows), ld >= D, ld_logits >= V");
  if ((((uintptr_t)h | (uintptr_t)W) & 15) != 0) return fail(D3S_ERR_ARG, "h and W must be 16-byte aligned");
  if (((uintptr_t)out & 1) != 0) return fail(D3S_ERR_ARG, "logits must be 2-byte aligned");
  return D3S_OK;
}

int d3s_lmhead(d3s_ctx *ctx, const void *h_dev, int64_t ld_h, const void *W_dev, int64_t ld_w,
               int B, int V, int D, void *logits_dev, int64_t ld_logits, void *stream) {
  if (!ctx) return fail(D3S_ERR_ARG, "null ctx");
  int rc = check_lmhead(h_dev, ld_h, W_dev, ld_w, B, V, D, logits_dev, ld_logits);
  if (rc != D3S_OK) return rc;
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  d3s::LmArgs a;
  a.h = h_dev;
  a.ld_h = ld_h;
  a.W = W_dev;
  a.ld_w = ld_w;
  a.B = B;
  a.V = V;
  a.D = D;
  a.out = logits_dev;
  a.ld_out = ld_logits;
  a.error = reinterpret_cast<int32_t *>(ctx->scratch.counters + 2);
  rc = d3s::launch_lmhead(a, (cudaStream_t)stream);
  if (rc != D3S_OK) return cuda_fail(cudaGetLastError(), "lm_head launch");
  return D3S_OK;
}

int d3s_lmhead_sample(d3s_ctx *ctx, const void *h_dev, int64_t ld_h, const void *W_dev,
                      int64_t ld_w, int D, const d3s_request *req, void *stream) {
  if (!ctx || !req) return fail(D3S_ERR_ARG, "null ctx or request");
  if (req->dtype != D3S_BF16) return fail(D3S_ERR_ARG, "the projection writes bf16 logits");
  int rc = d3s_lmhead(ctx, h_dev, ld_h, W_dev, ld_w, req->N, req->V, D,
                      const_cast<void *>(req->logits), req->ld, stream);
  if (rc != D3S_OK) return rc;
  return d3s_sample(ctx, req, stream);
}

// ---- the test ABI of the reference ----

static std::mutex g_default_mu;
static d3s_ctx *g_default_ctx = nullptr;

static int default_ctx(d3s_ctx **out) {
  std::lock_guard<std::mutex> lk(g_default_mu);
  if (!g_default_ctx) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    int rc = d3s_ctx_create(dev, &g_default_ctx);
    if (rc != D3S_OK) return rc;
  }
  *out = g_default_ctx;
  return D3S_OK;
}

// d3_sample of one row with the kernel reading the logits from, and writing
// the id and status to, pinned host memory mapped into the device: no upload
// or download, one launch and one synchronisation. Returns kHandedOn when the
// kernel left the row on the hand-off list (k > 256 is excluded by the caller;
// ties beyond the candidate list, fewer finite logits than k): the ordinary
// path then samples it with the same subkey.
constexpr int kHandedOn = 1;
static int d3_sample_row(d3s_ctx *ctx, const float *logits, int V, float temperature, int top_k,
                         float top_p, d3s_key sub, int *out) {
  const size_t lbytes = ((size_t)V * sizeof(float) + 15) & ~(size_t)15;
  const size_t need = lbytes + 16;  // the row, then id, status and the done word
  cudaError_t e;
  if (need > ctx->row_cap) {
    cudaStreamSynchronize(ctx->stream);  // the old buffer may be in use by queued work
    cudaFreeHost(ctx->row_host);
    ctx->row_host = ctx->row_dev = nullptr;
    ctx->row_cap = 0;
    e = cudaHostAlloc(reinterpret_cast<void **>(&ctx->row_host), need, cudaHostAllocMapped);
    if (e != cudaSuccess) return fail(D3S_ERR_NOMEM, "mapped host staging: %s", cudaGetErrorString(e));
    e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&ctx->row_dev), ctx->row_host, 0);
    if (e != cudaSuccess) {
      cudaFreeHost(ctx->row_host);
      ctx->row_host = nullptr;
      return cuda_fail(e, "cudaHostGetDevicePointer");
    }
    ctx->row_cap = need;
  }
  std::memcpy(ctx->row_host, logits, (size_t)V * sizeof(float));
  volatile int32_t *res = reinterpret_cast<volatile int32_t *>(ctx->row_host + lbytes);
  res[0] = INT32_MIN;  // stays when the row is handed on
  res[1] = D3S_ROW_OK;
  res[2] = 0;          // the kernel sets it once the results are written
  d3s_request r{};
  r.logits = ctx->row_dev;
  r.dtype = D3S_F32;
  r.N = 1;
  r.V = V;
  r.ld = V;
  r.temperature = temperature;
  r.top_p = top_p;
  r.top_k = top_k;
  r.noise = D3S_NOISE_KEY;
  r.key = sub;
  r.ids = reinterpret_cast<int32_t *>(ctx->row_dev + lbytes);
  r.status = r.ids + 1;
  d3s::KArgs a = to_kargs(&r, ctx);
  a.direct = 1;        // the kernel loads the mapped row itself (no waits, no error word)
  a.skip_handoff = 1;  // a handed-on row is caught below
  a.done_flag = r.ids + 2;
  if (d3s::launch_sample(a, ctx->scratch, ctx->stream) != D3S_OK)
    return cuda_fail(cudaGetLastError(), "sampler launch");
  // Poll the done word the kernel writes last (the row was read long before, so
  // the next call may refill the staging at once); after 1 s, or when the word
  // never comes, the stream's own synchronisation decides (and reports errors).
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned spin = 0; res[2] == 0; ++spin)
    if ((spin & 1023u) == 1023u && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(1))
      break;
  if (res[2] == 0) {
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(e, "d3_sample");
  }
  const int32_t id = res[0], st = res[1];
  if (id == INT32_MIN) return kHandedOn;
  out[0] = id;
  if (st != D3S_ROW_OK) return fail(D3S_ERR_NONFINITE, "1 row(s) had non-finite logits");
  return D3S_OK;
}

static int d3_sample_impl(const float *logits, int N, int V, float temperature, int top_k,
                          float top_p, unsigned long long seed, int *out) {
  if (N < 0 || V < 1 || (N > 0 && (!logits || !out))) return fail(D3S_ERR_ARG, "bad d3_sample args");
  d3s_ctx *ctx = nullptr;
  int rc = default_ctx(&ctx);
  if (rc != D3S_OK) return rc;
  std::lock_guard<std::mutex> lk(g_default_mu);
  DeviceGuard g(ctx->device);
  if (!g.ok) return fail(D3S_ERR_CUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaError_t e;
  if (!ctx->stream) {
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
  }
  d3s_request r{};
  r.dtype = D3S_F32;
  r.N = N;
  r.V = V;
  r.ld = V;
  r.temperature = temperature;
  r.top_p = top_p;
  r.top_k = top_k;
  r.noise = D3S_NOISE_KEY;
  r.logits = logits;  // placeholders for the argument check; replaced below
  r.ids = out;
  rc = check_request(&r);
  if (rc != D3S_OK) return rc;
  if (N == 0) return D3S_OK;
  rc = reserve_scratch(ctx, N);
  if (rc != D3S_OK) return rc;
  d3s_seed(nullptr, seed);  // m_seed(seed), src/testapi.c:159
  d3s_key sub;
  take_subkey(nullptr, &sub);
  // one row on the one-CTA kernel (V <= 8192, k <= 256): zero-copy
  if (N == 1 && V <= 8192 && std::min(top_k, V) <= 256) {
    rc = d3_sample_row(ctx, logits, V, temperature, top_k, top_p, sub, out);
    if (rc != kHandedOn) return rc;
  }
  // One staging layout on both sides: [logits | error word, pad | ids | status].
  // One copy uploads the logits with a zeroed error word, one brings the error
  // word, the ids and the statuses back.
  const size_t nl = (size_t)N * (size_t)V;
  const size_t tail = (nl * sizeof(float) + 15) & ~(size_t)15;
  const size_t down = 16 + 2 * (size_t)N * sizeof(int32_t);
  const size_t need = tail + down;
  if (need > ctx->stage_cap) {
    cudaStreamSynchronize(ctx->stream);  // the old buffers may be in use by queued work
    cudaFree(ctx->stage_dev);
    cudaFreeHost(ctx->pinned);
    ctx->stage_dev = nullptr;
    ctx->pinned = nullptr;
    ctx->stage_cap = 0;
    e = cudaMalloc(&ctx->stage_dev, need);
    if (e != cudaSuccess) return fail(D3S_ERR_NOMEM, "d3_sample staging: %s", cudaGetErrorString(e));
    e = cudaMallocHost(&ctx->pinned, need);
    if (e != cudaSuccess) {
      cudaFree(ctx->stage_dev);
      ctx->stage_dev = nullptr;
      return fail(D3S_ERR_NOMEM, "host staging: %s", cudaGetErrorString(e));
    }
    ctx->stage_cap = need;
  }
  unsigned char *hp = static_cast<unsigned char *>(ctx->pinned);
  std::memcpy(hp, logits, nl * sizeof(float));
  std::memset(hp + nl * sizeof(float), 0, tail + 16 - nl * sizeof(float));
  int32_t *ids_dev = reinterpret_cast<int32_t *>(ctx->stage_dev + tail + 16);
  r.logits = ctx->stage_dev;
  r.ids = ids_dev;
  r.status = ids_dev + N;
  r.key = sub;
  d3s::KArgs a = to_kargs(&r, ctx);
  a.error = reinterpret_cast<int32_t *>(ctx->stage_dev + tail);  // this call's own error word
  e = cudaMemcpyAsync(ctx->stage_dev, hp, tail + 16, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "logits upload");
  if (d3s::launch_sample(a, ctx->scratch, ctx->stream) != D3S_OK)
    return cuda_fail(cudaGetLastError(), "sampler launch");
  e = cudaMemcpyAsync(hp + tail, ctx->stage_dev + tail, down, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return cuda_fail(e, "d3_sample");
  const int32_t *h_err = reinterpret_cast<const int32_t *>(hp + tail);
  const int32_t *h_ids = h_err + 4;
  std::memcpy(out, h_ids, (size_t)N * sizeof(int32_t));
  int bad = 0;
  for (int i = 0; i < N; i++) bad += h_ids[N + i] != D3S_ROW_OK;
  if (*h_err)
    return fail(D3S_ERR_CUDA, "a sampler kernel gave up waiting for a row copy (rows left unsampled)");
  if (bad) return fail(D3S_ERR_NONFINITE, "%d row(s) had non-finite logits", bad);
  return D3S_OK;
}

void d3_sample(const float *logits, int N, int V, float temperature, int top_k, float top_p,
               unsigned long long seed, int *out) {
  const int rc = d3_sample_impl(logits, N, V, temperature, top_k, top_p, seed, out);
  g_last_status = rc;
  if (rc != D3S_OK && rc != D3S_ERR_NONFINITE && out)
    for (int i = 0; i < N; i++) out[i] = -1;
}

int d3s_last_status(void) { return g_last_status; }

}  // extern "C"

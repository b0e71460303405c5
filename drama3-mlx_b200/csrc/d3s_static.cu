// d3s_static.cu - the batched sampler with its scratch in a fixed device array,
// for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at sampling time: a serving engine that
// plans every device byte up front and forbids allocation while it serves, or
// a real-time audio thread that cannot afford cudaMalloc's implicit device
// synchronisation. d3s_sample_rows_static runs the same kernels as d3s_sample
// with per-row parameters and seeds, but its scratch (row records and the
// hand-off list for the wide path) is the file-scope array below: every GPU
// that loads the library holds those bytes until the process exits, and no
// call allocates. The array's error word is sticky: a call clears only the
// hand-off and completion counters, and d3s_static_check reads and clears the
// error word, so a failure of any call since the last check is reported.
#include <cstdio>
#include <mutex>

#include "d3s.h"
#include "d3s_kernels.cuh"

namespace {

constexpr int kStaticRows = D3S_STATIC_MAX_ROWS;
constexpr size_t kHeadsOff = 0;
constexpr size_t kCandsOff = kHeadsOff + sizeof(d3s::RowHead) * kStaticRows;
constexpr size_t kListOff = kCandsOff + sizeof(d3s::RowCands) * kStaticRows;
constexpr size_t kCountersOff = kListOff + sizeof(int32_t) * kStaticRows;
constexpr size_t kStaticBytes = kCountersOff + 256;
static_assert(kCandsOff % 256 == 0 && kListOff % 256 == 0 && kCountersOff % 256 == 0,
              "scratch regions stay 256-byte aligned");

// The scratch every call shares: row headers, candidate slab, hand-off list,
// then the three counters: the hand-off count and the wide-kernel completion
// count, which each call clears before its kernels run, and the error word,
// which only d3s_static_check clears (zero when the module loads).
static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char *g_base[kMaxDevices];  // device address of g_static_scratch, per device

// The device address of g_static_scratch on the current device. Set-up, once
// per device, with that device current: the host-side name of the array is
// not a device address, so the runtime is asked for it.
int static_base(unsigned char **out) {
  char msg[160];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return d3s::set_error(D3S_ERR_CUDA, "static scratch: no current device");
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_base[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) {
      snprintf(msg, sizeof msg, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return d3s::set_error(D3S_ERR_CUDA, msg);
    }
    g_base[dev] = static_cast<unsigned char *>(p);
  }
  *out = g_base[dev];
  return D3S_OK;
}

int32_t *error_word(unsigned char *base) {
  return reinterpret_cast<int32_t *>(base + kCountersOff) + 2;
}

}  // namespace

extern "C" int d3s_sample_rows_static(const void *logits_dev, int dtype, int N, int V, int64_t ld,
                                      const float *temperature_dev, const float *top_p_dev,
                                      const int32_t *top_k_dev, const uint64_t *seeds_dev,
                                      int32_t *ids_dev, void *stream) {
  char msg[160];
  if (N < 0 || N > kStaticRows) {
    snprintf(msg, sizeof msg, "d3s_sample_rows_static: N=%d outside [0, %d]", N, kStaticRows);
    return d3s::set_error(N < 0 ? D3S_ERR_ARG : D3S_ERR_UNSUPPORTED, msg);
  }
  if (V < 1 || V > D3S_MAX_V || ld < V || (dtype != D3S_F32 && dtype != D3S_BF16))
    return d3s::set_error(D3S_ERR_ARG, "d3s_sample_rows_static: bad V, ld or dtype");
  if (N == 0) return D3S_OK;
  if (!logits_dev || !temperature_dev || !top_p_dev || !top_k_dev || !seeds_dev || !ids_dev)
    return d3s::set_error(D3S_ERR_ARG, "d3s_sample_rows_static: null pointer");
  unsigned char *base = nullptr;
  const int rc = static_base(&base);
  if (rc != D3S_OK) return rc;
  cudaError_t e;
  d3s::Scratch s;
  s.heads = reinterpret_cast<d3s::RowHead *>(base + kHeadsOff);
  s.cands = reinterpret_cast<d3s::RowCands *>(base + kCandsOff);
  s.deferred = reinterpret_cast<int32_t *>(base + kListOff);
  s.counters = reinterpret_cast<uint32_t *>(base + kCountersOff);
  s.capacity = kStaticRows;
  s.rec_capacity = kStaticRows;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(s.counters, 0, 2 * sizeof(uint32_t), st);  // not the error word
  if (e != cudaSuccess) {
    snprintf(msg, sizeof msg, "clearing the static scratch counters: %s", cudaGetErrorString(e));
    return d3s::set_error(D3S_ERR_CUDA, msg);
  }
  d3s::KArgs a{};
  a.logits = logits_dev;
  a.ld = ld;
  a.dtype = dtype;
  a.N = N;
  a.V = V;
  a.T_rows = temperature_dev;
  a.p_rows = top_p_dev;
  a.k_rows = top_k_dev;
  a.top_k = 1;
  a.noise = D3S_NOISE_SEEDS;
  a.seeds = seeds_dev;
  a.ids = ids_dev;
  a.deferred = s.deferred;
  a.deferred_n = s.counters;
  a.wide_done = s.counters + 1;
  a.error = reinterpret_cast<int32_t *>(s.counters + 2);
  a.deferred_cap = s.capacity;
  if (d3s::launch_sample(a, s, st) != D3S_OK) {
    snprintf(msg, sizeof msg, "d3s_sample_rows_static launch: %s",
             cudaGetErrorString(cudaGetLastError()));
    return d3s::set_error(D3S_ERR_CUDA, msg);
  }
  return D3S_OK;
}

extern "C" int d3s_static_check(void *stream) {
  unsigned char *base = nullptr;
  int rc = static_base(&base);
  if (rc != D3S_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t word = 0;
  char msg[160];
  cudaError_t e = cudaMemcpyAsync(&word, error_word(base), sizeof word, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && word != 0) e = cudaMemsetAsync(error_word(base), 0, sizeof word, st);
  if (e != cudaSuccess) {
    snprintf(msg, sizeof msg, "d3s_static_check: %s", cudaGetErrorString(e));
    return d3s::set_error(D3S_ERR_CUDA, msg);
  }
  if (word != 0)
    return d3s::set_error(D3S_ERR_CUDA,
                          "d3s_sample_rows_static: a kernel gave up waiting for a row copy "
                          "(ids of the calls since the last check are undefined)");
  return D3S_OK;
}

extern "C" int d3s_static_debug_set_error(int32_t value, void *stream) {
  unsigned char *base = nullptr;
  const int rc = static_base(&base);
  if (rc != D3S_OK) return rc;
  // a copy from pageable host memory is staged by the runtime before the call
  // returns, so `value` may live on this stack
  const cudaError_t e = cudaMemcpyAsync(error_word(base), &value, sizeof value,
                                        cudaMemcpyHostToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return d3s::set_error(D3S_ERR_CUDA, "d3s_static_debug_set_error: copy failed");
  return D3S_OK;
}

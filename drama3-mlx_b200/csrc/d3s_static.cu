// d3s_static.cu - the batched sampler with its scratch in a fixed device array,
// for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc at sampling time: a serving engine that
// plans every device byte up front and forbids allocation while it serves, a
// real-time audio thread that cannot afford cudaMalloc's implicit device
// synchronisation, or code running while someone else's stream capture is in
// progress. d3s_sample_rows_static runs the same kernels as d3s_sample with
// per-row parameters and seeds, but its scratch (row records and the hand-off
// list for the wide path) is the file-scope array below: every GPU that loads
// the library holds those bytes until the process exits, and no call allocates.
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
// then the three counters (hand-off count, wide-kernel completion count, error
// word), which each call clears before its kernels run.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char *g_base[kMaxDevices];  // device address of g_static_scratch, per device

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
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return d3s::set_error(D3S_ERR_CUDA, "d3s_sample_rows_static: no current device");
  unsigned char *base;
  {
    // Set-up, once per device, with that device current: the host-side name of
    // g_static_scratch is not a device address, so ask the runtime for it.
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
    base = g_base[dev];
  }
  d3s::Scratch s;
  s.heads = reinterpret_cast<d3s::RowHead *>(base + kHeadsOff);
  s.cands = reinterpret_cast<d3s::RowCands *>(base + kCandsOff);
  s.deferred = reinterpret_cast<int32_t *>(base + kListOff);
  s.counters = reinterpret_cast<uint32_t *>(base + kCountersOff);
  s.capacity = kStaticRows;
  s.rec_capacity = kStaticRows;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(s.counters, 0, 3 * sizeof(uint32_t), st);
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

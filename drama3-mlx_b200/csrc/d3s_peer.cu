// d3s_peer.cu - the gather of sampled ids to rank 0 over NVLink peer memory.
//
// Rows shard across the GPUs of one node, one process per GPU, and the only
// exchange is the gather of the int32 ids to rank 0. Instead of a collective
// after the sampler, the sampler of rank r writes its ids straight into rank
// 0's result buffer (a CUDA IPC mapping of it, plain stores over NVLink), at
// the rank's global row offset, so the transfer happens inside the sampler's
// own kernels. Completion is a counter in rank 0's memory: each rank adds 1
// (a release at system scope) after its sampler, and rank 0 waits (an acquire
// spin with a time limit) until every rank's addition for the step has
// landed. The result has `slots` slots (step s in slot s mod slots): a rank
// may write step s only after rank 0 released step s - slots, so rank 0 can
// still read the last slots - 1 steps while the ranks write step s, and the
// ranks may run up to slots - 1 steps ahead of rank 0's gather. Issued on a
// side stream (after an event of the sampler's stream), the signal and the
// wait overlap the next step's sampling.
//
// Layout of the allocation rank 0 owns (exported by cudaIpcGetMemHandle):
//   [0, 256)                      control words: arrived, released, lined_up
//   [256, 256 + 4 N slots)        `slots` slots of N int32 ids
#include <cstdio>
#include <cstring>
#include <new>

#include "d3s.h"
#include "d3s_kernels.cuh"

struct d3s_gather {
  int device = 0;
  int world = 1, rank = 0;
  int64_t rows = 0;            // N, the ids of every rank together
  int slots = 2;
  int64_t start = 0, stop = 0;  // this rank's rows
  unsigned char *base = nullptr;  // rank 0: its allocation; others: the IPC mapping
  bool opened = false;            // base is an IPC mapping (ranks > 0)
  int32_t *error_local = nullptr; // this rank's own wait-failure word (device)
};

namespace {

constexpr size_t kCtrlBytes = 256;
constexpr unsigned long long kWaitNs = 5000000000ull;  // 5 s

struct Ctrl {
  unsigned arrived;   // ranks' additions, cumulative over steps
  unsigned released;  // steps rank 0 has released (the next step it will gather)
  unsigned lined_up;  // ranks' additions at start lines, cumulative
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait (one thread, bounded by kWaitNs) until *word reaches target (modulo
// 2^32, acquire at system scope); on time-out set *err and return.
__global__ void gather_wait_kernel(const unsigned *word, unsigned target, int32_t *err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if ((int)(ld_acquire_sys(word) - target) >= 0) return;
  const unsigned long long t0 = now_ns();
  for (;;) {
    __nanosleep(64);
    if ((int)(ld_acquire_sys(word) - target) >= 0) return;
    if (now_ns() - t0 > kWaitNs) {
      atomicOr(err, 1);
      return;
    }
  }
}

// *word = value with release semantics at system scope. The reads of the
// released slot are earlier work of this stream, complete before this kernel
// starts; the peers only write the slot after they observe the new value.
__global__ void gather_publish_kernel(unsigned *word, unsigned value) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(word), "r"(value) : "memory");
}

// Add 1 to *word with release semantics at system scope, after every earlier
// write of this stream (the sampler's ids, stores to peer memory included).
__global__ void gather_signal_kernel(unsigned *word) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(word) : "memory");
}

// A start line: add 1 to *word (release, system scope, after every earlier
// write of this stream), then wait (bounded by kWaitNs) until every rank's
// addition for this line has landed (*word reaches target, acquire).
__global__ void gather_line_kernel(unsigned *word, unsigned target, int32_t *err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(word) : "memory");
  if ((int)(ld_acquire_sys(word) - target) >= 0) return;
  const unsigned long long t0 = now_ns();
  for (;;) {
    __nanosleep(64);
    if ((int)(ld_acquire_sys(word) - target) >= 0) return;
    if (now_ns() - t0 > kWaitNs) {
      atomicOr(err, 1);
      return;
    }
  }
}

int gfail(int code, const char *msg) { return d3s::set_error(code, msg); }

int gcuda(cudaError_t e, const char *what) {
  char msg[200];
  snprintf(msg, sizeof msg, "%s: %s", what, cudaGetErrorString(e));
  return d3s::set_error(D3S_ERR_CUDA, msg);
}

struct DevScope {
  int prev = -1;
  bool ok = true;
  explicit DevScope(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DevScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

Ctrl *ctrl(const d3s_gather *g) { return reinterpret_cast<Ctrl *>(g->base); }
int32_t *slot(const d3s_gather *g, int64_t step) {
  return reinterpret_cast<int32_t *>(g->base + kCtrlBytes) + (step % g->slots) * g->rows;
}

}  // namespace

extern "C" {

int d3s_gather_create(int device, int world, int rank, int64_t rows, int slots,
                      d3s_gather **out) {
  if (!out) return gfail(D3S_ERR_ARG, "d3s_gather_create: null out");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world || rows < 0 || rows > (int64_t)1 << 36 || slots < 2 ||
      slots > 64)
    return gfail(D3S_ERR_ARG, "d3s_gather_create: bad world / rank / rows / slots");
  DevScope d(device);
  if (!d.ok) return gfail(D3S_ERR_CUDA, "d3s_gather_create: cudaSetDevice failed");
  d3s_gather *g = new (std::nothrow) d3s_gather();
  if (!g) return gfail(D3S_ERR_NOMEM, "d3s_gather_create: host allocation");
  g->device = device;
  g->world = world;
  g->rank = rank;
  g->rows = rows;
  g->slots = slots;
  g->start = rows * rank / world;
  g->stop = rows * (rank + 1) / world;
  cudaError_t e = cudaMalloc(&g->error_local, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(g->error_local, 0, sizeof(int32_t));
  if (e == cudaSuccess && rank == 0) {
    const size_t bytes = kCtrlBytes + (size_t)slots * (size_t)rows * sizeof(int32_t);
    e = cudaMalloc(&g->base, bytes);
    if (e == cudaSuccess) e = cudaMemset(g->base, 0, bytes);
  }
  if (e != cudaSuccess) {
    cudaFree(g->error_local);
    cudaFree(g->base);
    delete g;
    return gcuda(e, "d3s_gather_create");
  }
  *out = g;
  return D3S_OK;
}

int d3s_gather_export(d3s_gather *g, void *handle) {
  if (!g || !handle || g->rank != 0) return gfail(D3S_ERR_ARG, "d3s_gather_export: rank 0 only");
  DevScope d(g->device);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, g->base);
  if (e != cudaSuccess) return gcuda(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == D3S_GATHER_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof h);
  return D3S_OK;
}

int d3s_gather_attach(d3s_gather *g, const void *handle) {
  if (!g || !handle) return gfail(D3S_ERR_ARG, "d3s_gather_attach: null argument");
  if (g->rank == 0) return D3S_OK;
  if (g->base) return gfail(D3S_ERR_ARG, "d3s_gather_attach: already attached");
  DevScope d(g->device);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof h);
  void *p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return gcuda(e, "cudaIpcOpenMemHandle");
  g->base = static_cast<unsigned char *>(p);
  g->opened = true;
  return D3S_OK;
}

int d3s_gather_begin(d3s_gather *g, int64_t step, int32_t **ids_dev, void *stream) {
  if (!g || !ids_dev || step < 0) return gfail(D3S_ERR_ARG, "d3s_gather_begin: bad argument");
  if (!g->base) return gfail(D3S_ERR_ARG, "d3s_gather_begin: not attached");
  DevScope d(g->device);
  // the slot of `step` is free once rank 0 released step - slots (rank 0
  // releases in the order of its own stream, so it never waits here)
  if (step >= g->slots && g->rank != 0) {
    gather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        &ctrl(g)->released, (unsigned)(step - g->slots + 1), g->error_local);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return gcuda(e, "gather slot wait launch");
  }
  *ids_dev = slot(g, step) + g->start;
  return D3S_OK;
}

int d3s_gather_end(d3s_gather *g, int64_t step, int32_t **result_dev, void *stream) {
  if (!g || step < 0) return gfail(D3S_ERR_ARG, "d3s_gather_end: bad argument");
  if (!g->base) return gfail(D3S_ERR_ARG, "d3s_gather_end: not attached");
  DevScope d(g->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (g->rank != 0) {
    gather_signal_kernel<<<1, 32, 0, st>>>(&ctrl(g)->arrived);
  } else if (g->world > 1) {
    // every other rank adds 1 per step: step s is complete at (world - 1)(s + 1)
    const unsigned target = (unsigned)((uint64_t)(g->world - 1) * (uint64_t)(step + 1));
    gather_wait_kernel<<<1, 32, 0, st>>>(&ctrl(g)->arrived, target, g->error_local);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gcuda(e, "gather end launch");
  if (result_dev) *result_dev = g->rank == 0 ? slot(g, step) : nullptr;
  return D3S_OK;
}

int d3s_gather_release(d3s_gather *g, int64_t step, void *stream) {
  if (!g || step < 0) return gfail(D3S_ERR_ARG, "d3s_gather_release: bad argument");
  if (g->rank != 0) return D3S_OK;
  DevScope d(g->device);
  gather_publish_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(&ctrl(g)->released,
                                                                        (unsigned)(step + 1));
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gcuda(e, "gather release launch");
  return D3S_OK;
}

int d3s_gather_line_up(d3s_gather *g, int64_t line, void *stream) {
  if (!g || line < 1) return gfail(D3S_ERR_ARG, "d3s_gather_line_up: bad argument");
  if (!g->base) return gfail(D3S_ERR_ARG, "d3s_gather_line_up: not attached");
  DevScope d(g->device);
  const unsigned target = (unsigned)((uint64_t)g->world * (uint64_t)line);
  gather_line_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(&ctrl(g)->lined_up, target,
                                                                     g->error_local);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return gcuda(e, "gather start line launch");
  return D3S_OK;
}

int d3s_gather_copy_result(d3s_gather *g, int64_t step, int32_t *dst_dev, void *stream) {
  if (!g || step < 0 || (!dst_dev && g->rows > 0) || g->rank != 0)
    return gfail(D3S_ERR_ARG, "d3s_gather_copy_result: rank 0 only, non-null destination");
  DevScope d(g->device);
  const cudaError_t e = cudaMemcpyAsync(dst_dev, slot(g, step), (size_t)g->rows * sizeof(int32_t),
                                        cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return gcuda(e, "d3s_gather_copy_result");
  return D3S_OK;
}

int d3s_gather_check(d3s_gather *g, void *stream) {
  if (!g) return gfail(D3S_ERR_ARG, "d3s_gather_check: null gather");
  DevScope d(g->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t word = 0;
  cudaError_t e = cudaMemcpyAsync(&word, g->error_local, sizeof word, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && word) e = cudaMemsetAsync(g->error_local, 0, sizeof word, st);
  if (e != cudaSuccess) return gcuda(e, "d3s_gather_check");
  if (word) return gfail(D3S_ERR_CUDA, "id gather: a wait for another rank timed out");
  return D3S_OK;
}

void d3s_gather_destroy(d3s_gather *g) {
  if (!g) return;
  DevScope d(g->device);
  cudaDeviceSynchronize();
  if (g->opened)
    cudaIpcCloseMemHandle(g->base);
  else
    cudaFree(g->base);
  cudaFree(g->error_local);
  delete g;
}

}  // extern "C"

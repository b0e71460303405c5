// d3s_frame.cu - the sampling part of one decode frame (tower_decode_step,
// src/tower.c:405-452) for many streams at once, and the per-stream key
// sequences that feed it.
//
// A frame of stream s draws, in this order, from the stream's key sequence:
// the main token (user parameters) and the retry token (RAS: T 1.0, top_p
// 0.95, top_k 30, src/tower.c:14-16), both from the same backbone logits row,
// then one token per codebook head. The main and retry draws of all streams
// run as ONE sampler request of 2S rows whose rows s and S + s read logits row
// s (KArgs::row_period), so the logits are streamed once per draw pair from
// HBM/L2 and the kernels launch once. A small kernel then applies
// candidate_token (index 0 -> eos, i >= 1 -> semantic_start + i - 1), the
// repetition check against the last RAS_WINDOW main tokens (only semantic
// tokens are redrawn, src/tower.c:429-433), c0 and the flags, and appends the
// main token to the history window (src/generate.c:97-100).
#include <cstdint>

#include "d3s.h"
#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

namespace d3s {
namespace {

constexpr float kRasTemperature = 1.0f;  // src/tower.c:14
constexpr int kRasTopK = 30;             // src/tower.c:15
constexpr float kRasTopP = 0.95f;        // src/tower.c:16

__global__ void keys_next_kernel(uint2 *state, int S, int n, uint2 *sub, int64_t ld_sub) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= S) return;
  uint2 st = state[s];
  for (int i = 0; i < n; ++i) {
    uint2 k0, k1;
    key_split(st, k0, k1);  // KeySequence::next: keep k0, hand out k1
    st = k0;
    sub[(int64_t)s * ld_sub + i] = k1;
  }
  state[s] = st;
}

// Parameters and keys of the 2S draws: rows [0, S) main, [S, 2S) retry.
__global__ void frame_prep_kernel(FrameArgs f, FrameScratch fs) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= 2 * f.S) return;
  const bool retry = r >= f.S;
  const int s = retry ? r - f.S : r;
  fs.T[r] = retry ? kRasTemperature : f.temperature;
  fs.p[r] = retry ? kRasTopP : f.top_p;
  fs.k[r] = retry ? kRasTopK : f.top_k;
  fs.keys[r] = f.keys[(int64_t)s * f.ld_keys + (retry ? 1 : 0)];
}

__device__ __forceinline__ int candidate_token(int idx, int semantic_start, int eos_id) {
  return idx == 0 ? eos_id : idx + semantic_start - 1;
}

__global__ void frame_finish_kernel(FrameArgs f, FrameScratch fs) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= f.S) return;
  const int id1 = fs.ids[s], id2 = fs.ids[f.S + s];
  int flags = fs.finite[s] ? 0 : D3S_FRAME_NONFINITE;
  int32_t *hist = f.history + (int64_t)s * D3S_RAS_WINDOW;
  int hl = f.hist_len[s];
  hl = hl < 0 ? 0 : (hl > D3S_RAS_WINDOW ? D3S_RAS_WINDOW : hl);
  int tok = -1;
  if (id1 >= 0 && id2 >= 0) {
    const int t1 = candidate_token(id1, f.semantic_start, f.eos_id);
    const int t2 = candidate_token(id2, f.semantic_start, f.eos_id);
    bool seen = false;
    for (int i = 0; i < hl; ++i) seen = seen || hist[i] == t1;
    const bool semantic = t1 >= f.semantic_start && t1 <= f.semantic_start + f.code_vocab - 1;
    const bool repeated = seen && semantic;
    tok = repeated ? t2 : t1;
    if (repeated) flags |= D3S_FRAME_RETRY;
    if (tok == f.eos_id) flags |= D3S_FRAME_EOS;
  } else {
    flags |= D3S_FRAME_NONFINITE;  // a draw was flagged (non-finite scaled logits)
  }
  int c = tok < 0 ? 0 : tok - f.semantic_start;
  c = c < 0 ? 0 : (c > f.code_vocab - 1 ? f.code_vocab - 1 : c);
  f.main_tok[s] = tok;
  f.c0[s] = c;
  if (f.flags) f.flags[s] = flags;
  if (f.update_history) {
    if (hl == D3S_RAS_WINDOW) {
      for (int i = 1; i < D3S_RAS_WINDOW; ++i) hist[i - 1] = hist[i];
      hist[D3S_RAS_WINDOW - 1] = tok;
    } else {
      hist[hl] = tok;
      f.hist_len[s] = hl + 1;
    }
  }
}

}  // namespace

int launch_keys_next(uint2 *state, int S, int n, uint2 *sub, int64_t ld_sub, cudaStream_t st) {
  if (S == 0 || n == 0) return D3S_OK;
  keys_next_kernel<<<(S + 127) / 128, 128, 0, st>>>(state, S, n, sub, ld_sub);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

int launch_frame(const FrameArgs &f, const FrameScratch &fs, KArgs a, const Scratch &sc,
                 cudaStream_t st) {
  if (f.S == 0) return D3S_OK;
  const int threads = 128;
  frame_prep_kernel<<<(2 * f.S + threads - 1) / threads, threads, 0, st>>>(f, fs);
  if (cudaGetLastError() != cudaSuccess) return D3S_ERR_CUDA;
  a.N = 2 * f.S;
  a.row_period = f.S;
  a.T_rows = fs.T;
  a.p_rows = fs.p;
  a.k_rows = fs.k;
  a.noise = D3S_NOISE_KEYS;
  a.keys = fs.keys;
  a.ld_keys = 1;
  a.ids = fs.ids;
  a.finite = fs.finite;
  const int rc = launch_sample(a, sc, st);
  if (rc != D3S_OK) return rc;
  frame_finish_kernel<<<(f.S + threads - 1) / threads, threads, 0, st>>>(f, fs);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

}  // namespace d3s

// d3s_lmhead.cu - the restricted lm_head projection in front of the sampler:
// logits[b, v] = bf16(sum_d h[b, d] * W[v, d]) with fp32 accumulation, the
// bf16 output of backbone_audio_logits -> m_linear -> gemv_row
// (src/backbone.c:1213, src/mlxu.c:397, src/mlxu.c:442-496).
//
// Two kernels:
//   * B <= kGemvMaxB: a CUDA-core GEMV. One warp per W row, 16-byte loads of
//     the row, h staged once per CTA in shared memory; it streams W once
//     (16.8 MB for the backbone's [4097, 2048]) and is HBM-bound.
//   * larger B: a tcgen05 GEMM with the operands swapped so that the long
//     side (V logit ids) is the UMMA M dimension: D[v, b] = W[v, :] . h[b, :].
//     Tiles of 128 W rows x BN batch rows, K staged 64 at a time by TMA
//     (128-byte swizzle) through a ring of shared-memory stages; one thread
//     issues tcgen05.mma (kind::f16, bf16 x bf16 -> fp32 in TMEM) and commits
//     each stage back to the producer; four epilogue warps read the
//     accumulator with tcgen05.ld, round to bf16 and store logits[b, v].
//     When the tiles alone leave most SMs idle (small B) the K loop is split
//     over the CTAs of a cluster, whose fp32 partials are added on chip
//     through distributed shared memory. Every CTA loads its own tiles from
//     this GPU's memory; no load is shared across the cluster.
// Every wait on an mbarrier is bounded (kLmWaitLimitNs); a wait that gives up
// sets the error word and the kernel drains its copies, frees its tensor
// memory and returns.
#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "d3s.h"
#include "d3s_device.cuh"
#include "d3s_kernels.cuh"

namespace d3s {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kBM = 128;           // W rows per tile (UMMA M)
constexpr int kBK = 64;            // K per stage: one 128-byte swizzle row of bf16
constexpr int kUK = 16;            // K per tcgen05.mma of kind::f16
constexpr int kGemmThreads = 192;  // warp 0: TMA, warp 1: TMEM + MMA, warps 2-5: epilogue
constexpr uint64_t kLmWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint32_t saddr(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false when it gave up or another role already gave up.
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity, volatile int *abort_flag) {
  if (bar_try(b, parity)) return true;
  const unsigned long long t0 = now_ns();
  while (!bar_try(b, parity)) {
    if (*abort_flag) return false;
    if (now_ns() - t0 > kLmWaitLimitNs) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void bar_expect_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(b)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(saddr(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Shared-memory matrix descriptor of a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO),
// leading offset 1 (unused for swizzled K-major), descriptor version 1,
// layout type 2 (SWIZZLE_128B). The tile base is 1024-byte aligned, so the
// base offset is 0; a K step inside the swizzle row adds its byte offset to
// the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B
// bf16 (bits 7-9 = 1, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at
// bits 17-22, M >> 4 at bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          saddr(bar))
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int BN>
struct GemmCfg {
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes > 8 ? 8 : (200 * 1024) / kStageBytes;
  static constexpr uint32_t kTmemCols = BN <= 32 ? 32 : BN;  // a power of two >= 32
  // stages, then 2 * stages + 1 mbarriers, the TMEM address and the abort flag,
  // plus slack to align the base to 1024
  static constexpr size_t kSmem = (size_t)kStages * kStageBytes + (2 * kStages + 1) * 8 + 16 + 1024;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M = 128");
  static_assert(kStageBytes % 1024 == 0, "stages keep the 1024-byte alignment of the swizzle");
  static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM columns: a power of two");
};

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Float offset of (row, 16-byte chunk kc) in a [128][BN] fp32 partial whose
// chunks are XOR-swizzled by row, so eight consecutive rows' same chunk fall
// in eight different bank groups.
template <int BN>
__device__ __forceinline__ int part_off(int row, int kc) {
  return row * BN + 4 * (kc ^ (row & 7));
}

// ks > 1: the ks CTAs of a cluster (along z) split the K loop of one output
// tile; once every CTA's MMAs are complete (a cluster barrier), the CTAs of
// rank > 0 store their fp32 partials into the rank-0 CTA's shared memory (its
// stages, free by then) through distributed shared memory, and after a second
// cluster barrier rank 0 adds them in rank order and writes bf16 logits.
template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    lmhead_gemm_kernel(const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmH, __nv_bfloat16 *out,
                       int64_t ld_out, int V, int B, int KT, int kps, int ks, int32_t *error) {
  using Cfg = GemmCfg<BN>;
  constexpr int S = Cfg::kStages;
  extern __shared__ unsigned char dsmem[];
  unsigned char *base =
      (unsigned char *)(((uintptr_t)dsmem + 1023) & ~(uintptr_t)1023);  // swizzle atoms: 1024-aligned
  uint64_t *full = reinterpret_cast<uint64_t *>(base + (size_t)S * Cfg::kStageBytes);
  uint64_t *empty = full + S;
  uint64_t *accum = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM;  // first W row (logit id) of the tile
  const int n0 = blockIdx.y * BN;   // first batch row of the tile
  // split K: this CTA's k-tiles [kt0, kt0 + nk)
  const int kt0 = blockIdx.z * kps;
  const int nk = min(KT - kt0, kps);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    bar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(Cfg::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
    // producer: W tile [128 x 64] and h tile [BN x 64] per stage
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (i >= S && !bar_wait(&empty[s], ((i / S) & 1) ^ 1, abort_flag)) break;
      unsigned char *st = base + (size_t)s * Cfg::kStageBytes;
      bar_expect_tx(&full[s], Cfg::kStageBytes);
      tma_load_2d(st, &tmW, (kt0 + i) * kBK, m0, &full[s]);
      tma_load_2d(st + Cfg::kABytes, &tmH, (kt0 + i) * kBK, n0, &full[s]);
      ++issued;
    }
    if (*abort_flag) {  // let the copies still in flight land before the CTA exits
      for (int kt = issued - S > 0 ? issued - S : 0; kt < issued; ++kt) {
        const unsigned long long t0 = now_ns();
        while (!bar_try(&full[kt % S], (kt / S) & 1) && now_ns() - t0 < kLmWaitLimitNs) {
        }
      }
    }
    }
    __syncwarp();  // the warp reconverges before the CTA barrier
  } else if (warp == 1) {
    if (lane == 0) {
    // MMA issuer
    constexpr uint32_t idesc = umma_idesc(kBM, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!bar_wait(&full[s], (i / S) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t a0 = saddr(base + (size_t)s * Cfg::kStageBytes);
      const uint32_t b0 = a0 + Cfg::kABytes;
#pragma unroll
      for (int kk = 0; kk < kBK / kUK; ++kk)
        umma_bf16(tmem, sw128_desc(a0 + kk * kUK * 2), sw128_desc(b0 + kk * kUK * 2), idesc,
                  (i | kk) != 0 ? 1u : 0u);
      umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
    }
    umma_commit(accum);  // arrives when every MMA issued above is complete
    }
    __syncwarp();
  } else if (warp >= 2) {
    // epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 = W rows of the tile
    const int q = warp & 3;
    const bool ok = bar_wait(accum, 0, abort_flag);
    tc_fence_after();
    const int v = m0 + q * 32 + lane;
    if (ks == 1) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
        if (ok && !*abort_flag && v < V) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int b = n0 + c + j;
            if (b < B) out[(int64_t)b * ld_out + v] = __float2bfloat16_rn(__uint_as_float(r[j]));
          }
        }
      }
    }
  }
  if (ks > 1) {
    // every CTA of the cluster has its partial in TMEM and its stages free
    cluster_sync_all();
    const uint32_t rank = cluster_rank();
    float *part = reinterpret_cast<float *>(base);  // [ks - 1][128][BN] in rank 0's stages
    if (warp >= 2 && rank > 0) {
      const int q = warp & 3, row = q * 32 + lane;
      float *mine = part + (size_t)(rank - 1) * kBM * BN;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const uint32_t local = saddr(mine + part_off<BN>(row, (c + j) >> 2));
          uint32_t remote;
          asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(remote) : "r"(local));
          asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(remote),
                       "r"(r[j]), "r"(r[j + 1]), "r"(r[j + 2]), "r"(r[j + 3])
                       : "memory");
        }
      }
    }
    cluster_sync_all();  // the partials are in rank 0's shared memory
    if (warp >= 2 && rank == 0) {
      const int q = warp & 3, row = q * 32 + lane, v = m0 + row;
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, r);
        float acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(r[j]);
        for (int z = 1; z < ks; ++z) {  // rank order: the sum of the k-tiles in split order
          const float *pz = part + (size_t)(z - 1) * kBM * BN;
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 f = *reinterpret_cast<const float4 *>(pz + part_off<BN>(row, (c + j) >> 2));
            acc[j] = __fadd_rn(acc[j], f.x);
            acc[j + 1] = __fadd_rn(acc[j + 1], f.y);
            acc[j + 2] = __fadd_rn(acc[j + 2], f.z);
            acc[j + 3] = __fadd_rn(acc[j + 3], f.w);
          }
        }
        if (!*abort_flag && v < V) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int b = n0 + c + j;
            if (b < B) out[(int64_t)b * ld_out + v] = __float2bfloat16_rn(acc[j]);
          }
        }
      }
    }
  }
  if (warp >= 2) tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(Cfg::kTmemCols)
                 : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(error, 2);
}

// ---- 2-SM GEMM (B >= 256): a CTA pair shares one 256 x 256 UMMA tile ----
//
// tcgen05.mma.cta_group::2 with M = 256 (W rows), N = 256 (batch rows): each
// CTA of the pair stages its 128 W rows and its 128 batch rows per K step
// (32 KB; the pair's MMA reads both CTAs' stages) and holds its 128 output rows
// x 256 columns in its own TMEM. Per K step a CTA moves 32 KB for the work a
// single-CTA 128 x 256 tile moves 48 KB for, so six stages hide the L2
// latency. The leader (rank 0) issues the MMAs; both CTAs' loads complete on
// the leader's full barrier (mapa address); the leader commits each stage to
// its own and to its peer's empty barrier, and the result to both accumulator
// barriers (two plain commits, one per CTA).

constexpr int kStages2 = 6;
constexpr int kPairMinB = 512;  // from here the pair tiles alone fill the GPU (V = 4097: 136 CTAs at B = 1024)
constexpr uint32_t kHalfBytes = 128 * kBK * 2;        // 128 rows x 64 k of bf16
constexpr uint32_t kStageBytes2 = 2 * kHalfBytes;     // this CTA's W half + h half
constexpr size_t kSmem2 = (size_t)kStages2 * kStageBytes2 + (2 * kStages2 + 1) * 8 + 16 + 1024;

// shared::cluster address of the same object in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t peer_addr(const void *p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *tm, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(saddr(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void umma2_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrives on the mbarrier at a shared::cluster address once the issued MMAs complete
__device__ __forceinline__ void umma2_commit(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

constexpr int kGemm2Threads = 320;  // warp 0: TMA, warp 1: TMEM + MMA, warps 2-9: epilogue

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemm2Threads, 1)
    lmhead_gemm2_kernel(const __grid_constant__ CUtensorMap tmW,
                        const __grid_constant__ CUtensorMap tmH, __nv_bfloat16 *out,
                        int64_t ld_out, int V, int B, int KT, int32_t *error) {
  constexpr int S = kStages2;
  extern __shared__ unsigned char dsmem[];
  unsigned char *base = (unsigned char *)(((uintptr_t)dsmem + 1023) & ~(uintptr_t)1023);
  uint64_t *full = reinterpret_cast<uint64_t *>(base + (size_t)S * kStageBytes2);
  uint64_t *empty = full + S;
  uint64_t *accum = empty + S;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(accum + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank(), peer = rank ^ 1u;
  const bool leader = rank == 0;
  const int m0 = blockIdx.x * kBM;                       // this CTA's 128 W rows
  const int n0 = blockIdx.y * 256;                       // the pair's 256 batch rows
  const int nh = n0 + (int)rank * 128;                   // this CTA's half of them

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    bar_init(accum, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     saddr(tmem_slot)),
                 "r"(256)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any load or commit targets them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
    const uint32_t full0 = peer_addr(&full[0], 0);  // the leader's full barriers
    int issued = 0;
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % S;
      if (kt >= S && !bar_wait(&empty[s], ((kt / S) & 1) ^ 1, abort_flag)) break;
      unsigned char *st = base + (size_t)s * kStageBytes2;
      if (leader) bar_expect_tx(&full[s], 2 * kStageBytes2);  // both CTAs' halves
      tma_load_2d_pair(st, &tmW, kt * kBK, m0, full0 + 8 * s);
      tma_load_2d_pair(st + kHalfBytes, &tmH, kt * kBK, nh, full0 + 8 * s);
      ++issued;
    }
    if (*abort_flag && leader) {  // let the pair's copies in flight land before exiting
      for (int kt = issued - S > 0 ? issued - S : 0; kt < issued; ++kt) {
        const unsigned long long t0 = now_ns();
        while (!bar_try(&full[kt % S], (kt / S) & 1) && now_ns() - t0 < kLmWaitLimitNs) {
        }
      }
    }
    }
    __syncwarp();  // the warp reconverges before the CTA barrier
  } else if (warp == 1) {
    if (lane == 0 && leader) {
    constexpr uint32_t idesc = umma_idesc(2 * kBM, 256);
    const uint32_t empty_peer = peer_addr(&empty[0], peer), accum_peer = peer_addr(accum, peer);
    for (int kt = 0; kt < KT; ++kt) {
      const int s = kt % S;
      if (!bar_wait(&full[s], (kt / S) & 1, abort_flag)) break;
      tc_fence_after();
      const uint32_t a0 = saddr(base + (size_t)s * kStageBytes2);
      const uint32_t b0 = a0 + kHalfBytes;
#pragma unroll
      for (int kk = 0; kk < kBK / kUK; ++kk)
        umma2_bf16(tmem, sw128_desc(a0 + kk * kUK * 2), sw128_desc(b0 + kk * kUK * 2), idesc,
                   (kt | kk) != 0 ? 1u : 0u);
      umma2_commit(saddr(&empty[s]));  // the stage is free in both CTAs once these MMAs are done
      umma2_commit(empty_peer + 8 * s);
    }
    umma2_commit(saddr(accum));
    umma2_commit(accum_peer);
    }
    __syncwarp();
  } else {
    // epilogue, warps 2..9: warp w reads TMEM lanes 32 (w % 4) .. + 31 (this CTA's
    // W rows) and columns [128 h, 128 h + 128), h = (w - 2) / 4
    const int q = warp & 3, h = (warp - 2) >> 2;
    const bool ok = bar_wait(accum, 0, abort_flag);
    tc_fence_after();
    const int v = m0 + q * 32 + lane;
    const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(128 * h);
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      uint32_t r[32];
      tmem_ld32(ta + 32 * i, r);
      if (ok && !*abort_flag && v < V) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int b = n0 + 128 * h + 32 * i + j;
          if (b < B) out[(int64_t)b * ld_out + v] = __float2bfloat16_rn(__uint_as_float(r[j]));
        }
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs, loads and reads are over before TMEM and smem go away
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256)
                 : "memory");
  }
  if (threadIdx.x == 0 && *abort_flag) atomicOr(error, 2);
}

// ---- GEMV (B <= kGemvMaxB) ----

constexpr int kGemvRows = 2;   // W rows per warp task
constexpr int kGemvGroup = 8;  // 16-byte chunks per lane per pass (D = 2048: one pass)

template <int NB>
__device__ __forceinline__ void gemv_load(uint4 (&w)[kGemvRows][kGemvGroup], const __nv_bfloat16 *W,
                                          int64_t ld_w, int V, int chunks, int v0, int g,
                                          int lane) {
#pragma unroll
  for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
    for (int i = 0; i < kGemvGroup; ++i) {
      const int c = g + lane + 32 * i;
      w[r][i] = (v0 + r < V && c < chunks)
                    ? __ldg(reinterpret_cast<const uint4 *>(W + (int64_t)(v0 + r) * ld_w) + c)
                    : make_uint4(0, 0, 0, 0);
    }
}

// One warp per pair of W rows; each lane holds 8 16-byte chunks of both rows
// (all loads issued before any use, the first task's before h is staged), h
// is read from shared memory, the fp32 sums are reduced across the warp.
template <int NB>
__global__ void __launch_bounds__(32 * kGemvWarps)
    lmhead_gemv_kernel(const __nv_bfloat16 *h, int64_t ld_h, const __nv_bfloat16 *W,
                       int64_t ld_w, int B, int V, int D, __nv_bfloat16 *out, int64_t ld_out) {
  extern __shared__ __align__(16) unsigned char hs_raw[];
  const uint4 *hs = reinterpret_cast<const uint4 *>(hs_raw);  // [NB][chunks]
  const int chunks = D >> 3;                                   // 16-byte chunks per row
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * kGemvWarps + (threadIdx.x >> 5), nw = gridDim.x * kGemvWarps;
  int v0 = gw * kGemvRows;
  uint4 w[kGemvRows][kGemvGroup];
  if (v0 < V) gemv_load<NB>(w, W, ld_w, V, chunks, v0, 0, lane);
  for (int i = threadIdx.x; i < NB * chunks; i += blockDim.x) {
    const int b = i / chunks, c = i - b * chunks;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (b < B) v = *reinterpret_cast<const uint4 *>(h + (int64_t)b * ld_h + 8 * c);
    reinterpret_cast<uint4 *>(hs_raw)[i] = v;
  }
  __syncthreads();
  for (; v0 < V; v0 += nw * kGemvRows) {
    float acc[kGemvRows][NB];
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b) acc[r][b] = 0.0f;
    for (int g = 0; g < chunks; g += 32 * kGemvGroup) {
      if (g > 0) gemv_load<NB>(w, W, ld_w, V, chunks, v0, g, lane);
#pragma unroll
      for (int i = 0; i < kGemvGroup; ++i) {
        const int c = g + lane + 32 * i;
        if (c >= chunks) break;
        float wf[kGemvRows][8];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r) {
          const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&w[r][i]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(w2[e]);
            wf[r][2 * e] = f.x;
            wf[r][2 * e + 1] = f.y;
          }
        }
#pragma unroll
        for (int b = 0; b < NB; ++b) {
          const uint4 h4 = hs[b * chunks + c];
          const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&h4);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h2[e]);
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r) {
              acc[r][b] = __fmaf_rn(wf[r][2 * e], f.x, acc[r][b]);
              acc[r][b] = __fmaf_rn(wf[r][2 * e + 1], f.y, acc[r][b]);
            }
          }
        }
      }
    }
    const int vn = v0 + nw * kGemvRows;
    if (vn < V) gemv_load<NB>(w, W, ld_w, V, chunks, vn, 0, lane);  // next task's loads in flight
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
          acc[r][b] = __fadd_rn(acc[r][b], __shfl_xor_sync(0xffffffffu, acc[r][b], o));
    // lane r * NB + b writes (row v0 + r, batch b)
#pragma unroll
    for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
      for (int b = 0; b < NB; ++b)
        if (lane == r * NB + b && b < B && v0 + r < V)
          out[(int64_t)b * ld_out + v0 + r] = __float2bfloat16_rn(acc[r][b]);
  }
}

// ---- host: tensor maps ----

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                   const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 matrix [rows, cols] with row stride ld (elements), box [box_rows, 64].
bool make_map(CUtensorMap *m, const void *ptr, int rows, int cols, int64_t ld, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

// Split K when the output tiles leave most SMs idle (small B): about one CTA
// per SM, at least four k-tiles per split, and (the splits of a tile being one
// cluster) no more clusters than fit on the GPU at once.
template <int BN>
int gemm_splits(int B, int V, int D, int &kps) {
  const int KT = (D + kBK - 1) / kBK;
  const int tiles = ((V + kBM - 1) / kBM) * ((B + BN - 1) / BN);
  int want = std::max(1, std::min(8, sm_count() / std::max(tiles, 1)));
  want = std::min(want, std::max(1, KT / 4));
  // the partials of ranks 1 .. want - 1 must fit in rank 0's stages
  const size_t part_bytes = (size_t)kBM * BN * 4;
  want = std::min(want, 1 + (int)((size_t)GemmCfg<BN>::kStages * GemmCfg<BN>::kStageBytes / part_bytes));
  for (; want > 1; --want) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((V + kBM - 1) / kBM, (B + BN - 1) / BN, want);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmCfg<BN>::kSmem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 1;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = (unsigned)want;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, lmhead_gemm_kernel<BN>, &cfg) == cudaSuccess &&
        clusters >= tiles)
      break;
    cudaGetLastError();  // a refused query is not an error of the launch
  }
  kps = (KT + want - 1) / want;
  return (KT + kps - 1) / kps;
}

template <int BN>
int launch_gemm(const LmArgs &a, cudaStream_t st) {
  using Cfg = GemmCfg<BN>;
  CUtensorMap tw, th;
  if (!make_map(&tw, a.W, a.V, a.D, a.ld_w, kBM) || !make_map(&th, a.h, a.B, a.D, a.ld_h, BN))
    return D3S_ERR_CUDA;
  if (prepare_launch((const void *)lmhead_gemm_kernel<BN>, kGemmThreads, Cfg::kSmem) <= 0)
    return D3S_ERR_CUDA;
  const int KT = (a.D + kBK - 1) / kBK;
  int kps = KT;
  const int KS = gemm_splits<BN>(a.B, a.V, a.D, kps);
  if ((size_t)(KS - 1) * kBM * BN * 4 > (size_t)Cfg::kStages * Cfg::kStageBytes) return D3S_ERR_ARG;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.V + kBM - 1) / kBM, (a.B + BN - 1) / BN, KS);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = (unsigned)KS;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  __nv_bfloat16 *out = reinterpret_cast<__nv_bfloat16 *>(a.out);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, lmhead_gemm_kernel<BN>, tw, th, out, a.ld_out,
                                           a.V, a.B, KT, kps, KS, a.error);
  return e == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

int launch_gemm2(const LmArgs &a, cudaStream_t st) {
  CUtensorMap tw, th;
  if (!make_map(&tw, a.W, a.V, a.D, a.ld_w, kBM) || !make_map(&th, a.h, a.B, a.D, a.ld_h, 128))
    return D3S_ERR_CUDA;
  if (prepare_launch((const void *)lmhead_gemm2_kernel, kGemm2Threads, kSmem2) <= 0)
    return D3S_ERR_CUDA;
  const int mt = (a.V + kBM - 1) / kBM;
  const dim3 grid((mt + 1) & ~1, (a.B + 255) / 256);  // whole CTA pairs along W rows
  const int KT = (a.D + kBK - 1) / kBK;
  lmhead_gemm2_kernel<<<grid, kGemm2Threads, kSmem2, st>>>(
      tw, th, reinterpret_cast<__nv_bfloat16 *>(a.out), a.ld_out, a.V, a.B, KT, a.error);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

template <int NB>
int launch_gemv(const LmArgs &a, cudaStream_t st) {
  const size_t smem = (size_t)NB * a.D * 2;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(lmhead_gemv_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return D3S_ERR_CUDA;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int tasks = (a.V + kGemvRows - 1) / kGemvRows;
  const int blocks = std::max(1, std::min((tasks + kGemvWarps - 1) / kGemvWarps, 4 * sms));
  lmhead_gemv_kernel<NB><<<blocks, 32 * kGemvWarps, smem, st>>>(
      reinterpret_cast<const __nv_bfloat16 *>(a.h), a.ld_h,
      reinterpret_cast<const __nv_bfloat16 *>(a.W), a.ld_w, a.B, a.V, a.D,
      reinterpret_cast<__nv_bfloat16 *>(a.out), a.ld_out);
  return cudaGetLastError() == cudaSuccess ? D3S_OK : D3S_ERR_CUDA;
}

}  // namespace

int launch_lmhead(const LmArgs &a, cudaStream_t st) {
  if (a.B == 0 || a.V == 0) return D3S_OK;
  if (a.B <= 1) return launch_gemv<1>(a, st);
  if (a.B <= 2) return launch_gemv<2>(a, st);
  if (a.B <= 4) return launch_gemv<4>(a, st);
  if (a.B <= kGemvMaxB) return launch_gemv<kGemvMaxB>(a, st);
  if (a.B <= 32) return launch_gemm<32>(a, st);
  if (a.B <= 64) return launch_gemm<64>(a, st);
  if (a.B <= 128) return launch_gemm<128>(a, st);
  if (a.B < kPairMinB) return launch_gemm<256>(a, st);
  return launch_gemm2(a, st);
}

}  // namespace d3s

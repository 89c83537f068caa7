// BF16 GEMM on CTA pairs (tcgen05 cta_group::2), sm_100a.
//
//   C[M, N] = A[M, K] * B[N, K]^T, 256 x 256 output tiles per CTA pair.
//
// A cluster of two CTAs on two SMs computes one 256x256 tile: each CTA
// TMA-loads its own 128 rows of A and its own 128 rows of B (no multicast:
// every load lands in the issuing CTA's shared memory) and the leader CTA's
// single MMA thread issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16),
// which reads both CTAs' tiles and accumulates each CTA's 128 rows into its
// own TMEM.  Per SM this halves the B traffic of the one-CTA kernel (32 KB
// per 64-deep stage instead of 48 KB), which leaves room for 6 stages.
//
// Barriers: full[s] lives in the leader (both CTAs' loads complete_tx on it;
// the leader arms it with both byte counts); empty[s] and tfull[acc] live in
// both CTAs and are signalled by the leader's tcgen05.commit multicast; tempty[acc]
// lives in the leader and gets one arrive per epilogue warp of both CTAs.
// Epilogues are the one-CTA kernel's (gemm_sm100.cuh), per CTA on its 128
// rows x 256 columns.  All waits are bounded.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"

namespace clef {

struct Gemm2Shape {
  static constexpr int BM = 256, BN = 256, BK = 64;  // per CTA pair; each CTA: 128 rows of A and of B
  static constexpr int STAGES = 6;
  static constexpr uint32_t A_BYTES = 128 * BK * 2;
  static constexpr uint32_t B_BYTES = 128 * BK * 2;
  static constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators
  static constexpr size_t SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + 256;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster_addr, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` (same offset) in both CTAs of the pair once this thread's MMAs are done.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_sm100_pair(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                         GemmArgs args) {
  using S = Gemm2Shape;
  constexpr int BK = S::BK, STAGES = S::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(256, 256);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * S::B_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, num_clusters = gridDim.x >> 1;
  const int num_m = (args.M + S::BM - 1) / S::BM, num_n = (args.N + S::BN - 1) / S::BN;
  const int num_tiles = num_m * num_n;
  const int num_kb = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 8);  // one arrive per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, S::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);  // the leader's full[0]
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = cluster; tile < num_tiles && !*abort_flag; tile += num_clusters) {
        int m, n;
        gemm_tile_coords(tile, num_m, num_n, m, n);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.status, kTimeoutProducer) || *abort_flag) {
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * (S::A_BYTES + S::B_BYTES));
          const uint32_t bar = full0 + stage * 8;
          tma_load_2d_pair(sA + stage * S::A_BYTES, &tma_a, bar, kb * BK, m * S::BM + rank * 128);
          tma_load_2d_pair(sB + stage * S::B_BYTES, &tma_b, bar, kb * BK, n * S::BN + rank * 128);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = cluster; tile < num_tiles && !*abort_flag; tile += num_clusters, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.status, kTimeoutMma)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * S::BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.status, kTimeoutMma) || *abort_flag) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * S::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * S::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16_pair(d_tmem, smem_desc_k128(a_addr + k * 32), smem_desc_k128(b_addr + k * 32), IDESC,
                           (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit_pair(&tfull[acc]);
      }
      // Wait for this thread's pair MMAs before teardown (the commit must be a
      // cta_group::2 one to track them; it also arrives on the peer's drain).
      umma_commit_pair(drain);
      mbar_wait(drain, 0, args.status, kTimeoutDrain);
    }
  } else {
    const int q = warp & 3;
    const uint32_t tempty0 = mapa_shared(smem_u32(tempty), 0);
    int local = 0;
    for (int tile = cluster; tile < num_tiles; tile += num_clusters, ++local) {
      int m, n;
      gemm_tile_coords(tile, num_m, num_n, m, n);
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, args.status, kTimeoutEpilogue);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ok)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = m * S::BM + static_cast<int>(rank) * 128 + q * 32 + lane;
      const uint32_t taddr = tmem_base + acc * S::BN + (static_cast<uint32_t>(q * 32) << 16);
      gemm_epilogue<256, EPI>(args, taddr, row, n);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0 + acc * 8);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA frees TMEM while its pair may still use it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
}

}  // namespace clef

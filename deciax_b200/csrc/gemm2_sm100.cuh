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
//
// TPR (tensor parallelism): the o-proj / down-proj GEMM and the cross-rank
// reduction after it run as one kernel, so the NVLink transfer overlaps the
// MMAs of later tiles.  Every rank computes the same tiles in the same order
// (its FP32 partial, the kEpiF32 epilogue); each epilogue warp, once its 32
// rows of a tile are stored, publishes a flag in the memory of the tile's
// owner (tp_tile_owner).  Six more warps per CTA (warps 6..11) reduce the
// tiles this rank owns: they wait for the four epilogue warps' flags from
// every rank, sum the tp partial rows in rank order (peer loads), add the
// residual and write x = T(x + T(sum)) into every rank's x (peer stores) -- the semantics
// of the unfused path in tp.cuh (qwen3_5/pallas.py:66-69,121).  Flags carry a
// per-launch epoch, so they are never reset.  Plain peer loads and stores
// only; no multicast.
#pragma once

#include "common.cuh"
#include "gemm_sm100.cuh"
#include "tp.cuh"

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

// Peers of the fused TP reduction (TPR): index k = rank k's buffer.
struct TpFuse {
  const float* parts[kTpMaxRanks];  // FP32 partial [M, ldo] = this GEMM's output on rank k
  __nv_bfloat16* xs[kTpMaxRanks];   // residual stream x [M, ldx]
  unsigned* flags[kTpMaxRanks];     // tile flags [tiles][2 CTAs][4 warps][tp]
  int tp, rank, ldx;
  unsigned epoch;                   // this launch's flag value (every rank counts launches alike)
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Owner of a tile: alternates along each cluster's tiles and across the
// clusters of a wave, so every SM reduces 1/tp of its tiles and every rank
// pulls at every moment.
__device__ __forceinline__ int tp_tile_owner(int tile, int num_clusters, int tp) {
  return (tile / num_clusters + tile % num_clusters) % tp;
}

// tpf.flags[k] for a run-time k, without a run-time index into the kernel
// parameters (which would copy them to local memory).
__device__ __forceinline__ unsigned* tp_flag_array(const TpFuse& f, int k) {
  unsigned* r = f.flags[0];
#pragma unroll
  for (int j = 1; j < kTpMaxRanks; ++j)
    if (j == k) r = f.flags[j];
  return r;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The reduce warps' share of an owned tile: the CTA's rows [row0, row0 +
// nrows) x float4 columns [0, ncols4) from col0 (at most 128 x 64).  Item i is
// row i / 64, float4 column i % 64; warp w, lane l takes items w*32 + l +
// kTpReduceWarps*32*j, so each warp's loads are coalesced 512-byte runs.  R
// items per lane are in flight at once (R x TP peer loads of 16 bytes): the
// NVLink latency needs that much memory parallelism.
constexpr int kTpReduceWarps = 6;

template <int TP>
__device__ __forceinline__ void tp_reduce_rows(const TpFuse& f, const __nv_bfloat16* own_x, int ldo, int row0,
                                               int nrows, int col0, int ncols4, int item0) {
  constexpr int R = 8 / TP;
  constexpr int STRIDE = kTpReduceWarps * 32;
  const float* parts[TP];
  __nv_bfloat16* xs[TP];
#pragma unroll
  for (int k = 0; k < TP; ++k) {
    parts[k] = f.parts[k];
    xs[k] = f.xs[k];
  }
#pragma unroll 1
  for (int base = item0; base < 128 * 64; base += STRIDE * R) {
    float4 p[R][TP];
    uint2 rv[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int i = base + STRIDE * j;
      const int r = i >> 6, c = (i & 63) * 4;
      if (i < 128 * 64 && r < nrows && (i & 63) < ncols4) {
        const size_t po = static_cast<size_t>(row0 + r) * ldo + col0 + c;
#pragma unroll
        for (int k = 0; k < TP; ++k) p[j][k] = *reinterpret_cast<const float4*>(parts[k] + po);
        rv[j] = *reinterpret_cast<const uint2*>(own_x + static_cast<size_t>(row0 + r) * f.ldx + col0 + c);
      }
    }
#pragma unroll
    for (int j = 0; j < R; ++j) {
      const int i = base + STRIDE * j;
      const int r = i >> 6, c = (i & 63) * 4;
      if (!(i < 128 * 64 && r < nrows && (i & 63) < ncols4)) continue;
      const size_t xo = static_cast<size_t>(row0 + r) * f.ldx + col0 + c;
      float4 sum = p[j][0];
#pragma unroll
      for (int k = 1; k < TP; ++k) {  // rank order: the same bits on every rank
        sum.x += p[j][k].x;
        sum.y += p[j][k].y;
        sum.z += p[j][k].z;
        sum.w += p[j][k].w;
      }
      const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rv[j].x));
      const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rv[j].y));
      const uint2 o = make_uint2(pack_bf16x2(r0.x + round_to<__nv_bfloat16>(sum.x), r0.y + round_to<__nv_bfloat16>(sum.y)),
                                 pack_bf16x2(r1.x + round_to<__nv_bfloat16>(sum.z), r1.y + round_to<__nv_bfloat16>(sum.w)));
#pragma unroll
      for (int k = 0; k < TP; ++k) *reinterpret_cast<uint2*>(xs[k] + xo) = o;
    }
  }
}

template <int EPI, bool TPR = false>
__global__ void __launch_bounds__(TPR ? 192 + 32 * kTpReduceWarps : 192, 1)
    gemm_bf16_sm100_pair(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                         GemmArgs args, const __grid_constant__ TpFuse tpf) {
  static_assert(!TPR || EPI == kEpiF32, "the fused TP reduction follows the FP32-partial epilogue");
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
  } else if (warp < 6) {
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
      if constexpr (TPR) {
        // this warp's 32 partial rows are stored: tell the tile's owner
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
          const size_t slot = ((static_cast<size_t>(tile) * 2 + rank) * 4 + q) * tpf.tp + tpf.rank;
          st_release_sys(tp_flag_array(tpf, tp_tile_owner(tile, num_clusters, tpf.tp)) + slot, tpf.epoch);
        }
      }
    }
  } else if constexpr (TPR) {
    // ---- reduce warps: the tiles this rank owns, this CTA's 128 rows of each ----
    const int tp = tpf.tp;
    const __nv_bfloat16* own_x = tpf.xs[0];
    for (int k = 1; k < kTpMaxRanks; ++k)  // tpf.xs[tpf.rank] without a run-time index into the parameters
      if (k == tpf.rank) own_x = tpf.xs[k];
    const int item0 = (warp - 6) * 32 + lane;
    bool ok = true;
    for (int tile = cluster; ok && tile < num_tiles; tile += num_clusters) {
      if (tp_tile_owner(tile, num_clusters, tp) != tpf.rank) continue;
      int m, n;
      gemm_tile_coords(tile, num_m, num_n, m, n);
      // every rank's four epilogue warps have stored their rows of this tile:
      // flags [q][src] of this (tile, CTA), one per lane
      const unsigned* f = tp_flag_array(tpf, tpf.rank) + (static_cast<size_t>(tile) * 2 + rank) * 4 * tp;
      bool arrived = lane >= 4 * tp || ld_acquire_sys(f + lane) >= tpf.epoch;
      const long long t0 = clock64();
      while (!__all_sync(0xffffffffu, arrived)) {
        if (!arrived) arrived = ld_acquire_sys(f + lane) >= tpf.epoch;
        if (clock64() - t0 > 2 * kWaitCycles || *abort_flag) {
          record_status(args.status, kTimeoutTpFlag);
          arrived = true;
          ok = false;
        }
        __nanosleep(64);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      const int row0 = m * S::BM + static_cast<int>(rank) * 128;
      const int nrows = min(128, args.M - row0);
      const int ncols4 = (min(args.N, (n + 1) * S::BN) - n * S::BN) / 4;
      if (nrows > 0) {
        switch (tp) {
          case 2: tp_reduce_rows<2>(tpf, own_x, args.ldo, row0, nrows, n * S::BN, ncols4, item0); break;
          case 4: tp_reduce_rows<4>(tpf, own_x, args.ldo, row0, nrows, n * S::BN, ncols4, item0); break;
          case 8: tp_reduce_rows<8>(tpf, own_x, args.ldo, row0, nrows, n * S::BN, ncols4, item0); break;
          default: record_status(args.status, kBadTpRanks); break;  // the host launches only tp = 2, 4, 8
        }
      }
    }
    __threadfence_system();  // peer stores ordered before the barrier that follows the launch
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA frees TMEM while its pair may still use it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, S::TMEM_COLS);
}

}  // namespace clef

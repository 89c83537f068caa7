// BF16 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[M, N] = A[M, K] * B[N, K]^T        (A, B K-major: PyTorch [out, in] weights)
//
// Design (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte
//               swizzle, into a STAGES-deep shared-memory ring (no multicast).
//   warp 1      allocates 2*BN TMEM columns; one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M=128, N=BN, K=16) into one
//               of two TMEM accumulators and commits stage / tile barriers.
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time (thread = row),
//               apply the fused epilogue, store to global memory.
// The double-buffered accumulator lets tile i's epilogue overlap tile i+1's
// main loop.  All waits are bounded (see common.cuh).
//
// Epilogues (the reference rounding points, qwen3_5/text.py:21-22,94-102 and
// kernels/swiglu.py:100-101):
//   kEpiStore     out = T(acc + bias)                        dense() cast
//   kEpiSwiglu    B rows packed [128 gate | 128 up] per 256; out[:, j] =
//                 T(T(silu(T(g))) * T(u))                    fused SwiGLU
//   kEpiResidual  out = T(res + T(acc)) (may alias res)      x + dense(...)
//   kEpiF32       out = acc (float)                          TP partial sum
#pragma once

#include "common.cuh"

namespace clef {

enum GemmEpi : int { kEpiStore = 0, kEpiSwiglu = 1, kEpiResidual = 2, kEpiF32 = 3, kEpiQkv = 4 };

struct GemmArgs {
  int M, N, K;
  void* out;                       // bf16 (or float for kEpiF32), row stride ldo elements
  int ldo;
  const __nv_bfloat16* bias;       // [N] or nullptr (kEpiStore)
  const __nv_bfloat16* residual;   // [M, ldr] (kEpiResidual)
  int ldr;
  int* status;
  // kEpiQkv: the packed projection [Hq x (q d | gate d)] [Hkv x k d] [Hkv x v d]
  // leaves with q/k RMSNorm(1+w) + partial RoPE applied (text.py:83-88) and
  // the gate replaced by T(sigmoid(T(gate))) (text.py:91); v unchanged.
  const __nv_bfloat16* q_norm;
  const __nv_bfloat16* k_norm;
  const float* rope_cos;  // [seq, rot/2]
  const float* rope_sin;
  int hq, hkv, head_dim, rot, seq;
  float eps;
};

template <int BN>
struct GemmShape {
  static constexpr int BM = 128, BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr uint32_t A_BYTES = BM * BK * 2;
  static constexpr uint32_t B_BYTES = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = 2 * BN;
  static constexpr size_t SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + 256;
};

__device__ __forceinline__ void gemm_tile_coords(int tile, int num_m, int num_n, int& m, int& n) {
  // Group 16 M-tiles together so the CTAs in flight share A rows and B columns in L2.
  constexpr int GROUP = 16;
  const int per_group = GROUP * num_n;
  const int g = tile / per_group;
  const int first = g * GROUP;
  const int gm = min(num_m - first, GROUP);
  const int r = tile - g * per_group;
  m = first + r % gm;
  n = r / gm;
}

__device__ __forceinline__ float silu_f(float x) { return x * sigmoid_fast(x); }

__device__ __forceinline__ void store32_bf16(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    reinterpret_cast<uint4*>(dst)[q] =
        make_uint4(pack_bf16x2(v[8 * q + 0], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                   pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
}

__device__ __forceinline__ void load32_bf16(const __nv_bfloat16* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = reinterpret_cast<const uint4*>(src)[q];
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(h[e]);
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

__device__ __forceinline__ void load32_f32(const float* src, float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 f = reinterpret_cast<const float4*>(src)[q];
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

// kEpiQkv: the tile holds whole heads (head_dim divides BN).  Thread = row.
template <int BN>
__device__ __forceinline__ void qkv_epilogue(const GemmArgs& a, uint32_t taddr, int row, int n) {
  using bf = __nv_bfloat16;
  const bool live = row < a.M;
  const int d = a.head_dim, half = a.rot / 2;
  const int qcols = a.hq * 2 * d, kend = qcols + a.hkv * d;
  const int pos = live ? row % a.seq : 0;
  bf* out_row = static_cast<bf*>(a.out) + static_cast<size_t>(live ? row : 0) * a.ldo;
#pragma unroll 1
  for (int seg = 0; seg < BN; seg += d) {
    const int col = n * BN + seg;  // first column of this head segment (uniform across the warp)
    if (col >= a.N) break;
    const bool gate = col < qcols && (col % (2 * d)) >= d;
    const bool is_k = col >= qcols && col < kend;
    const bool norm = (col < qcols && !gate) || is_k;
    if (!norm) {  // v: T(x); gate: T(sigmoid(T(x)))
#pragma unroll 1
      for (int c = 0; c < d; c += 32) {
        uint32_t r[32];
        __syncwarp();
        tmem_ld32(taddr + seg + c, r);
        tmem_wait_ld();
        if (live) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float x = round_to<bf>(__uint_as_float(r[j]));
            v[j] = gate ? sigmoid_fast(x) : x;
          }
          store32_bf16(out_row + col + c, v);
        }
      }
      continue;
    }
    // RMSNorm over the head of T(x), scaling by (1 + w)
    float ps[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
    for (int c = 0; c < d; c += 32) {
      uint32_t r[32];
      __syncwarp();
      tmem_ld32(taddr + seg + c, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x = round_to<bf>(__uint_as_float(r[j]));
        ps[j & 3] = fmaf(x, x, ps[j & 3]);
      }
    }
    const float rs = rsqrtf(((ps[0] + ps[1]) + (ps[2] + ps[3])) / static_cast<float>(d) + a.eps);
    const bf* w = is_k ? a.k_norm : a.q_norm;
#pragma unroll 1
    for (int c = 0; c < d; c += 32) {
      if (half >= 32 && c >= half && c < a.rot) continue;  // written together with its rotate-half partner
      uint32_t ra[32];
      float wa[32], ya[32];
      __syncwarp();
      tmem_ld32(taddr + seg + c, ra);
      tmem_wait_ld();
      load32_bf16(w + c, wa);
#pragma unroll
      for (int j = 0; j < 32; ++j) ya[j] = round_to<bf>(round_to<bf>(__uint_as_float(ra[j])) * rs * (wa[j] + 1.f));
      if (half == 16 && c == 0) {  // rot = 32: both rotate-half partners lie in this chunk
        float cs[16], sn[16];
        const float4* cp = reinterpret_cast<const float4*>(a.rope_cos + static_cast<size_t>(pos) * 16);
        const float4* sp = reinterpret_cast<const float4*>(a.rope_sin + static_cast<size_t>(pos) * 16);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const float4 c4 = cp[v], s4 = sp[v];
          cs[4 * v] = c4.x, cs[4 * v + 1] = c4.y, cs[4 * v + 2] = c4.z, cs[4 * v + 3] = c4.w;
          sn[4 * v] = s4.x, sn[4 * v + 1] = s4.y, sn[4 * v + 2] = s4.z, sn[4 * v + 3] = s4.w;
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float co = round_to<bf>(cs[j]), si = round_to<bf>(sn[j]);
          const float lo = round_to<bf>(round_to<bf>(ya[j] * co) + round_to<bf>(-ya[j + 16] * si));
          const float hi = round_to<bf>(round_to<bf>(ya[j + 16] * co) + round_to<bf>(ya[j] * si));
          ya[j] = lo;
          ya[j + 16] = hi;
        }
      } else if (c < half) {
        uint32_t rb[32];
        float wb[32], yb[32], cs[32], sn[32];
        tmem_ld32(taddr + seg + c + half, rb);
        tmem_wait_ld();
        load32_bf16(w + c + half, wb);
        load32_f32(a.rope_cos + static_cast<size_t>(pos) * half + c, cs);
        load32_f32(a.rope_sin + static_cast<size_t>(pos) * half + c, sn);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          yb[j] = round_to<bf>(round_to<bf>(__uint_as_float(rb[j])) * rs * (wb[j] + 1.f));
          const float co = round_to<bf>(cs[j]), si = round_to<bf>(sn[j]);
          const float lo = round_to<bf>(round_to<bf>(ya[j] * co) + round_to<bf>(-yb[j] * si));
          const float hi = round_to<bf>(round_to<bf>(yb[j] * co) + round_to<bf>(ya[j] * si));
          ya[j] = lo;
          yb[j] = hi;
        }
        if (live) store32_bf16(out_row + col + c + half, yb);
      }
      if (live) store32_bf16(out_row + col + c, ya);
    }
  }
}

template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& a, uint32_t taddr, int row, int n) {
  const bool live = row < a.M;
  if constexpr (EPI == kEpiQkv) {
    qkv_epilogue<BN>(a, taddr, row, n);
  } else if constexpr (EPI == kEpiSwiglu) {
    // Tile n covers packed columns [n*BN, n*BN+BN): gate j at c, up j at c + BN/2.
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(a.out);
#pragma unroll 1
    for (int c = 0; c < BN / 2; c += 32) {
      uint32_t g[32], u[32];
      __syncwarp();
      tmem_ld32(taddr + c, g);
      tmem_ld32(taddr + BN / 2 + c, u);
      tmem_wait_ld();
      if (live) {
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(row) * a.ldo + n * (BN / 2) + c);
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float r2[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int idx = v * 8 + j * 2 + e;
              const float gt = round_to<__nv_bfloat16>(__uint_as_float(g[idx]));
              const float ut = round_to<__nv_bfloat16>(__uint_as_float(u[idx]));
              r2[e] = round_to<__nv_bfloat16>(silu_f(gt)) * ut;
            }
            w[j] = pack_bf16x2(r2[0], r2[1]);
          }
          dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
      const int col0 = n * BN + c;
      if (live && col0 < a.N) {
      const bool full = col0 + 32 <= a.N;
      if constexpr (EPI == kEpiF32) {
        float* dst = static_cast<float*>(a.out) + static_cast<size_t>(row) * a.ldo + col0;
        if (full) {
#pragma unroll
          for (int v = 0; v < 8; ++v)
            reinterpret_cast<float4*>(dst)[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                            __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < a.N) dst[j] = __uint_as_float(r[j]);
        }
      } else {
        __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(a.out) + static_cast<size_t>(row) * a.ldo + col0;
        float vals[32];
        if constexpr (EPI == kEpiStore) {
#pragma unroll
          for (int j = 0; j < 32; ++j) vals[j] = __uint_as_float(r[j]);
          if (a.bias) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < a.N) vals[j] += __bfloat162float(a.bias[col0 + j]);
          }
        } else {  // kEpiResidual
          const __nv_bfloat16* res = a.residual + static_cast<size_t>(row) * a.ldr + col0;
          if (full) {
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              const uint4 q = reinterpret_cast<const uint4*>(res)[v];
              const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                vals[v * 8 + j] = __bfloat162float(h[j]) + round_to<__nv_bfloat16>(__uint_as_float(r[v * 8 + j]));
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              vals[j] = col0 + j < a.N ? __bfloat162float(res[j]) + round_to<__nv_bfloat16>(__uint_as_float(r[j])) : 0.f;
          }
        }
        if (full) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            reinterpret_cast<uint4*>(dst)[v] =
                make_uint4(pack_bf16x2(vals[v * 8 + 0], vals[v * 8 + 1]), pack_bf16x2(vals[v * 8 + 2], vals[v * 8 + 3]),
                           pack_bf16x2(vals[v * 8 + 4], vals[v * 8 + 5]), pack_bf16x2(vals[v * 8 + 6], vals[v * 8 + 7]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < a.N) dst[j] = __float2bfloat16_rn(vals[j]);
        }
      }
      }
      __syncwarp();  // converge before the next tcgen05.ld.sync.aligned
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_bf16_sm100(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b, GemmArgs args) {
  using S = GemmShape<BN>;
  constexpr int BM = S::BM, BK = S::BK, STAGES = S::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN);

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
  const int num_m = (args.M + BM - 1) / BM, num_n = (args.N + BN - 1) / BN;
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
      mbar_init(&tempty[i], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        int m, n;
        gemm_tile_coords(tile, num_m, num_n, m, n);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.status, kTimeoutProducer) || *abort_flag) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], S::A_BYTES + S::B_BYTES);
          tma_load_2d(sA + stage * S::A_BYTES, &tma_a, &full[stage], kb * BK, m * BM);
          tma_load_2d(sB + stage * S::B_BYTES, &tma_b, &full[stage], kb * BK, n * BN);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every issued load must land before the CTA may exit.
      for (int i = 0; i < STAGES && i < issued; ++i) {
        if (stage == 0) {
          stage = STAGES - 1;
          phase ^= 1;
        } else {
          --stage;
        }
        mbar_wait(&full[stage], phase, args.status, kTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, args.status, kTimeoutMma)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
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
          for (int k = 0; k < BK / 16; ++k) {
            umma_bf16(d_tmem, smem_desc_k128(a_addr + k * 32), smem_desc_k128(b_addr + k * 32), IDESC,
                      (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&tfull[acc]);
      }
      // Wait for this thread's MMAs to finish before the CTA can tear down.
      umma_commit(drain);
      mbar_wait(drain, 0, args.status, kTimeoutDrain);
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
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
      const int row = m * BM + q * 32 + lane;
      const uint32_t taddr = tmem_base + acc * BN + (static_cast<uint32_t>(q * 32) << 16);
      gemm_epilogue<BN, EPI>(args, taddr, row, n);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, S::TMEM_COLS);
}

}  // namespace clef

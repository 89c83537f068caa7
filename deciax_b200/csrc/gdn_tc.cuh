// Gated DeltaNet mixer core on the 5th-generation tensor cores (sm_100a),
// BF16 activations, head dim 128: qwen3_5/text.py:48-67 with the chunked rule
// of kernels/gdn/reference.py:40-92.
//
// One CTA per (state, value head) walks the sequence in 64-token chunks.  The
// FP32 state S [dk, dv] stays in shared memory in the layout of a tcgen05
// B operand.  Per chunk (c, c' tokens of the chunk):
//   L  conv + SiLU, L2 norms and gates as the CUDA-core kernel (gdn.cuh),
//      written straight into operand layouts: A0 = [k; q] (128 rows), v.
//   M0 D0 = A0 k^T (M = 128, N = 64, K = 128): rows 0-63 k k^T, rows 64-127 q k^T.
//   M1 D1 = A0 S (N = 128): rows 0-63 k S, rows 64-127 q S.
//   P  rows 0-63 of D0 -> the strictly lower system A = -(k beta k^T) * decay;
//      rows 64-127 -> M = (q k^T) * decay (c' <= c), written back into tensor
//      memory as the A operand of M3; K~^T = (k e^{g_C - g})^T into tensor
//      memory (the A operand of M4); R = v - e^g * (k S) in place of v.
//   T  the inverse T = (I - A)^{-1} (reference.py:73-80) by exact forward
//      substitution on the CUDA cores, one column per thread, stored as
//      T diag(beta).
//   MV V_new = T diag(beta) R (K = 64).  This is reference.py:81-83's
//      T (v beta) - T (k beta e^g) S, regrouped so that neither product with
//      T runs over the value and the key dims separately.
//   M3 D3 = M V_new (A from tensor memory, K = 64).
//   M4 D2 = K~^T V_new (M = 128, N = 128, K = 64); S = S e^{g_C} + D2
//      (reference.py:86).
//   O  rows c: e^{g_c} (q S)_c + D3_c (reference.py:85), then the gated
//      RMSNorm x SiLU(z) (text.py:61-67).
// Products run as kind::tf32 (operands rounded to TF32, FP32 accumulation);
// the inverse, the gates and every elementwise step are FP32.  The FP32
// parity mode keeps the all-FP32 CUDA-core kernel.
//
// Operand tiles are rows of 32 fp32 (128 B) in atoms of `rows` rows per 32
// columns: a K-major operand [M or N rows][K] with the 128-byte swizzle
// (16-byte chunks XOR row % 8), an MN-major one [K rows][M or N] with the
// 128-byte swizzle of 32-byte atomicity (32-byte chunks XOR row % 4), the only
// swizzle tcgen05 takes for 32-bit MN-major operands.  Tensor memory (512
// columns): D0 [0, 64), D1 [64, 192), V_new product then D3 [192, 320), D2
// [320, 448), K~^T [448, 512).  One thread issues the MMAs and commits to one
// mbarrier; every wait is bounded.  Rows past the sequence end are zero with
// g = beta = 0, as the reference's padding.
#pragma once

#include "attention_sm100.cuh"
#include "common.cuh"
#include "gdn.cuh"

namespace clef {

constexpr int kGdnTcDim = 128;

struct GdnTcShape {
  static constexpr int C = kGdnChunk, DH = kGdnTcDim, LDA = C + 4;
  static constexpr uint32_t S_BYTES = DH * DH * 4;        // state, MN-major B [dk rows][dv]
  static constexpr uint32_t A0_BYTES = 2 * C * DH * 4;    // [k; q], K-major [128 rows][dk]
  static constexpr uint32_t V_BYTES = C * DH * 4;         // v -> R -> V_new, MN-major [tokens][dv]
  static constexpr uint32_t T_BYTES = 2 * C * C * 4;      // T diag(beta), K-major [128 rows][64]; rows 64-127 the unscaled T
  static constexpr uint32_t AS_BYTES = C * LDA * 4;       // system matrix, row-major
  static constexpr uint32_t MISC_FLOATS = 4 * C + 2 * C + 32 * 33 + DH;  // gates, norm sums, inverse blocks, norm weight
  static constexpr int ZLD = DH + 8;  // z rows staged over the system matrix: bf16, 272-byte rows
  static_assert(C * ZLD * 2 <= AS_BYTES, "z staging");
  static constexpr size_t SMEM = 1024 + S_BYTES + A0_BYTES + V_BYTES + T_BYTES + AS_BYTES + MISC_FLOATS * 4 + 64;
  static constexpr uint32_t D0 = 0, D1 = 64, DV = 192, D2 = 320, KT = 448, TMEM_COLS = 512;
};

// Byte offset of element (row, col) of a K-major fp32 operand tile (rows =
// M or N, col = K) in atoms of `rows` rows x 32 columns, with the 128-byte
// swizzle: the eight 16-byte chunks of a 128-byte row XOR-permuted by row % 8.
__device__ __forceinline__ uint32_t gdn_sw(int row, int col, int rows) {
  return static_cast<uint32_t>((col >> 5) * (rows * 128) + row * 128 + ((((col & 31) >> 2) ^ (row & 7)) << 4) +
                               ((col & 3) << 2));
}

// The same for an MN-major fp32 operand tile (row = K, col = M or N).  For
// 32-bit MN-major operands tcgen05 takes only the 128-byte swizzle with
// 32-byte atomicity: the four 32-byte chunks of a 128-byte row XOR-permuted
// by row % 4, K rows in groups of four (512 bytes).
__device__ __forceinline__ uint32_t gdn_sw_mn(int row, int col, int rows) {
  return static_cast<uint32_t>((col >> 5) * (rows * 128) + row * 128 + ((((col & 31) >> 3) ^ (row & 3)) << 5) +
                               ((col & 7) << 2));
}

// Shared-memory descriptor of such an MN-major tile: `lbo` bytes between
// 32-column atoms, 512 bytes between 4-row K groups, layout type 1
// (SWIZZLE_128B_BASE32B), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_mn128_32b(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(512 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(1) << 61;
  return d;
}

// Round to TF32 (10-bit mantissa, to nearest, ties away), the operand precision of kind::tf32.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Instruction descriptor, kind::tf32: TF32 A/B, FP32 D; a_mn / b_mn = MN-major operands.
__host__ __device__ constexpr uint32_t idesc_tf32_f32(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// A from tensor memory: row i of A in lane i, one TF32 per 32-bit column, K = 8 over 8 columns.
__device__ __forceinline__ void umma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Stage L as its own pass: causal conv + SiLU (text.py:31-39) of every q, k
// and v channel and the L2 norms of q and k (reference.py:14-21), written as
// bf16 rows [B*S, 2*nh*dh + nv*dh] (q heads, k heads, v heads, in projection
// column order).  Every value is one the reference rounds to bf16, so the
// chunk kernel reads exactly what it used to compute itself; q leaves without
// the dk^-1/2 factor.  One CTA per (256-token span, q/k/v head, state): the
// q and k heads are computed once, not once per value head that shares them,
// and the pass runs at full occupancy (each CTA walks kGdnConvBlocks blocks
// with its taps in registers).  The sliding-window arithmetic is
// gdn_load_chunk's (same taps, same order of operations).
constexpr int kGdnConvBlocks = 4;  // 64-token blocks per CTA of the conv pass

template <int W>
__global__ void __launch_bounds__(kGdnThreads) gdn_conv_bf16_kernel(GdnArgs a) {
  using T = __nv_bfloat16;
  constexpr int C = kGdnChunk, DH = kGdnTcDim, VN = GdnVec<T>::N, GL = DH / VN, RPP = kGdnThreads / GL;
  constexpr int RT = C / RPP, NX = RT + W - 1;
  const int tid = threadIdx.x, g = tid % GL, r0 = (tid / GL) * RT;
  const int kh = blockIdx.y, b = blockIdx.z;
  const int kind = kh < a.nh ? 0 : kh < 2 * a.nh ? 1 : 2;
  const int col = (kind == 0 ? kh * DH : kind == 1 ? a.k_col + (kh - a.nh) * DH : a.v_col + (kh - 2 * a.nh) * DH) +
                  g * VN;
  const T* proj = static_cast<const T*>(a.proj);
  const T* convw = static_cast<const T*>(a.conv);
  T* dst = static_cast<T*>(a.qkv_conv);
  const long long row0 = static_cast<long long>(b) * a.S;
  const int shift = W - a.width;
  float w[VN][W];  // this thread's taps, loaded once for all its blocks
#pragma unroll
  for (int c = 0; c < VN; ++c)
#pragma unroll
    for (int i = 0; i < W; ++i)
      w[c][i] = i >= shift ? to_f32(convw[static_cast<long long>(col + c) * a.width + (i - shift)]) : 0.f;
  for (int blk = 0; blk < kGdnConvBlocks; ++blk) {
    const int t0 = (blockIdx.x * kGdnConvBlocks + blk) * C;  // uniform across the CTA
    if (t0 >= a.S) break;
    float x[NX][VN];
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      const int tt = t0 + r0 - (W - 1) + i;
      const uint4 raw = (tt >= 0 && tt < a.S) ? *reinterpret_cast<const uint4*>(proj + (row0 + tt) * a.ldp + col)
                                              : make_uint4(0u, 0u, 0u, 0u);
      const T* hv = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int c = 0; c < VN; ++c) x[i][c] = __bfloat162float(hv[c]);
    }
#pragma unroll
    for (int j = 0; j < RT; ++j) {
      const int t = t0 + r0 + j;
      GdnVec<T> y;
#pragma unroll
      for (int c = 0; c < VN; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < W; ++i) acc = __fadd_rn(acc, __fmul_rn(x[j + i][c], w[c][i]));
        const float z = round_to<T>(acc);
        y.v[c] = t < a.S ? round_to<T>(z * sigmoid_fast(z)) : 0.f;
      }
      if (kind < 2) {
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < VN; ++c) ss += y.v[c] * y.v[c];
        const float inv = rsqrtf(group_sum<GL>(ss) + 1e-6f);
#pragma unroll
        for (int c = 0; c < VN; ++c) y.v[c] = round_to<T>(y.v[c] * inv);
      }
      if (t < a.S) y.store(dst + (row0 + t) * a.ldc + kh * DH + g * VN);
    }
  }
}

__global__ void __launch_bounds__(kGdnThreads, 1) gdn_tc_kernel(GdnArgs a) {
  using Sh = GdnTcShape;
  using T = __nv_bfloat16;
  constexpr int C = Sh::C, DH = Sh::DH, LDA = Sh::LDA;
  constexpr uint32_t IDESC_G = idesc_tf32_f32(128, C, false, false);  // A0 k^T: both K-major
  constexpr uint32_t IDESC_N = idesc_tf32_f32(128, DH, false, true);  // x S, T R, (tmem A) V_new: B MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sS = smem;
  uint8_t* sA0 = sS + Sh::S_BYTES;
  uint8_t* sV = sA0 + Sh::A0_BYTES;
  uint8_t* sT = sV + Sh::V_BYTES;
  float* As = reinterpret_cast<float*>(sT + Sh::T_BYTES);  // [C][LDA]
  float* gs = As + C * LDA;                                // cumulative g
  float* bs = gs + C;                                      // beta
  float* es = bs + C;                                      // e^g
  float* ws = es + C;                                      // e^(g_last - g)
  float* red = ws + C;                                     // [2][C] output-row partial sums of squares
  float* yb = red + 2 * C;                                 // [32][33] products of the blocked inverse
  float* nws = yb + 32 * 33;                               // gated-norm weight
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(nws + DH);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;  // tensor-memory lane quarter, column half
  const int lrow = quarter * 32 + lane;            // this thread's tensor-memory lane
  const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
  const int hk = h / (a.nv / a.nh);
  const T* proj = static_cast<const T*>(a.proj);
  const T* nw = static_cast<const T*>(a.norm_w);
  const T* qkv = static_cast<const T*>(a.qkv_conv);
  T* out = static_cast<T*>(a.out);
  const float neg_a = -expf(to_f32(static_cast<const T*>(a.A_log)[h]));
  const float dt_bias = to_f32(static_cast<const T*>(a.dt_bias)[h]);
  const long long row0 = static_cast<long long>(b) * a.S;
  const int q_col = hk * DH, k_col = (a.nh + hk) * DH, v_col = (2 * a.nh + h) * DH;  // columns of the conv pass

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Sh::TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = tid; i < DH * DH; i += kGdnThreads) reinterpret_cast<float*>(sS)[i] = 0.f;  // S = 0 (any layout)
  // the T tile starts zero: blocks above the diagonal are never written
  for (int i = tid; i < 2 * C * C; i += kGdnThreads) reinterpret_cast<float*>(sT)[i] = 0.f;
  if (tid < DH) nws[tid] = to_f32(nw[tid]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint32_t mma_phase = 0;

  // One thread issues a group of MMAs and commits; everyone waits for it.
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mma_bar, mma_phase, a.status, kTimeoutMma);
    mma_phase ^= 1;
    tc_fence_after();
    return __syncthreads_and(ok) != 0;
  };

  const uint32_t a0 = smem_u32(sA0), sv = smem_u32(sV), st = smem_u32(sT), ss_addr = smem_u32(sS);
  const int chunks = (a.S + C - 1) / C;
  for (int ci = 0; ci < chunks; ++ci) {
    const int t0 = ci * C;
    // ---- L: q, k, v rows of the conv pass into the operand tiles (k -> A0
    // rows 0-63, q x dk^-1/2 -> A0 rows 64-127, v -> V), and the gates ----
    float ga = 0.f, gb = 0.f;
    const bool gate_row = tid < C && t0 + tid < a.S;
    if (gate_row) {
      const T* pr = proj + (row0 + t0 + tid) * a.ldp;
      ga = to_f32(pr[a.a_col + h]);
      gb = to_f32(pr[a.b_col + h]);
    }
    {
      constexpr int RS = kGdnThreads / 16;  // rows per pass: 16 threads x 8 channels per row
      uint4 raw[3][C / RS];
#pragma unroll
      for (int i = 0; i < C / RS; ++i) {
        const int r = tid / 16 + RS * i, t = t0 + r, g8 = (tid % 16) * 8;
        const T* src = qkv + (row0 + t) * a.ldc + g8;
#pragma unroll
        for (int kind = 0; kind < 3; ++kind)
          raw[kind][i] = t < a.S ? *reinterpret_cast<const uint4*>(src + (kind == 0 ? q_col : kind == 1 ? k_col : v_col))
                                 : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < C / RS; ++i) {
        const int r = tid / 16 + RS * i, g8 = (tid % 16) * 8;
#pragma unroll
        for (int kind = 0; kind < 3; ++kind) {
          const T* hv = reinterpret_cast<const T*>(&raw[kind][i]);
          float y[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) y[c] = kind == 0 ? to_tf32(__bfloat162float(hv[c]) * a.qscale) : __bfloat162float(hv[c]);
#pragma unroll
          for (int c = 0; c < 8; c += 4) {
            const float4 v4 = make_float4(y[c], y[c + 1], y[c + 2], y[c + 3]);
            if (kind == 2)
              *reinterpret_cast<float4*>(sV + gdn_sw_mn(r, g8 + c, C)) = v4;
            else
              *reinterpret_cast<float4*>(sA0 + gdn_sw(kind == 0 ? C + r : r, g8 + c, 2 * C)) = v4;
          }
        }
      }
    }
    if (tid < C) {
      gs[tid] = gate_row ? neg_a * softplus_f(ga + dt_bias) : 0.f;
      bs[tid] = gate_row ? round_to<T>(sigmoid_fast(gb)) : 0.f;
    }
    fence_async_smem();
    __syncthreads();
    // cumulative gate (sequential, as cumsum) and its exponentials; M0 and M1 meanwhile
    if (warp == 0) {
      if (lane == 0) {
        float acc = 0.f;
        for (int r = 0; r < C; ++r) {
          acc += gs[r];
          gs[r] = acc;
        }
      }
      __syncwarp();
      const float last = gs[C - 1];
      for (int r = lane; r < C; r += 32) {
        es[r] = expf(gs[r]);
        ws[r] = expf(last - gs[r]);
      }
    }
    if (tid == 32) {
      // ---- M0: D0 = [k; q] k^T;  M1: D1 = [k; q] S (the k operand values
      // are exact in TF32: bf16 after the norm) ----
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < DH / 8; ++kk) {
        const uint32_t off = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
        umma_tf32(tmem + Sh::D0, smem_desc_k128(a0 + off), smem_desc_k128(a0 + off), IDESC_G, kk > 0 ? 1u : 0u);
        umma_tf32(tmem + Sh::D1, smem_desc_k128(a0 + off), smem_desc_mn128_32b(ss_addr + kk * 1024, DH * 128),
                  IDESC_N, kk > 0 ? 1u : 0u);
      }
      umma_commit(mma_bar);
    }
    if (!mma_wait()) break;
    // ---- P: system matrix (lanes 0-63) or M (lanes 64-127); K~^T; R (lanes 0-63) ----
    {
      // this thread: tensor-memory lane lrow, D0 columns [32 half, +32)
      uint32_t d[32];
      tmem_ld32(tmem + t_lane + Sh::D0 + 32 * half, d);
      tmem_wait_ld();
      if (lrow < C) {
        const int i = lrow;
        const float gi = gs[i], bi = bs[i];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = 32 * half + e;
          As[i * LDA + j] = j < i ? -(__uint_as_float(d[e]) * bi) * exp_fast(gi - gs[j]) : 0.f;
        }
      } else {
        const int i = lrow - C;
        const float gi = gs[i];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int j = 32 * half + e;
          d[e] = __float_as_uint(j <= i ? to_tf32(__uint_as_float(d[e]) * exp_fast(gi - gs[j])) : 0.f);
        }
        tmem_st32(tmem + t_lane + Sh::D0 + 32 * half, d);
      }
      // K~^T: lane (key dim) x columns c in [32 half, +32): k[c][key] e^{g_last - g_c}
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int c = 32 * half + e;
        d[e] = __float_as_uint(to_tf32(*reinterpret_cast<const float*>(sA0 + gdn_sw(c, lrow, 2 * C)) * ws[c]));
      }
      tmem_st32(tmem + t_lane + Sh::KT + 32 * half, d);
      if (lrow < C) {
        // R = v - e^g (k S), value dims [64 half, +64)
        const int c = lrow;
        const float ec = es[c];
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int j0 = 64 * half + 32 * part;
          tmem_ld32(tmem + t_lane + Sh::D1 + j0, d);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            float4* p = reinterpret_cast<float4*>(sV + gdn_sw_mn(c, j0 + e, C));
            float4 u = *p;
            u.x = to_tf32(fmaf(-ec, __uint_as_float(d[e]), u.x));
            u.y = to_tf32(fmaf(-ec, __uint_as_float(d[e + 1]), u.y));
            u.z = to_tf32(fmaf(-ec, __uint_as_float(d[e + 2]), u.z));
            u.w = to_tf32(fmaf(-ec, __uint_as_float(d[e + 3]), u.w));
            *p = u;
          }
        }
      }
      tmem_wait_st();
    }
    __syncthreads();
    // ---- T: (I - A)^{-1} by blocks.  The unscaled inverse is built in rows
    // 64-127 of the T tile (rows the MV product computes but nobody reads);
    // each block, once final, also goes to rows 0-63 scaled by beta per column
    // and rounded to TF32: the A operand of MV.  Diagonal 16 x 16 blocks by
    // forward substitution; then for [[P, 0], [Q, R]] with known inverses P', R'
    // the lower-left block of the inverse is R' (Q~ P'), Q~ = the system
    // entries (A holds minus the matrix's off-diagonal), first for the 16 x 16
    // pairs of blocks, then for the two 32 x 32 halves.  Blocks above the
    // diagonal are never written and stay zero in both copies. ----
    {
      auto tw = [&](int r, int c) -> float& { return *reinterpret_cast<float*>(sT + gdn_sw(C + r, c, 2 * C)); };
      auto tw4 = [&](int r, int c4) -> float4 {  // working row r, columns c4..c4+3
        return *reinterpret_cast<const float4*>(sT + gdn_sw(C + r, c4, 2 * C));
      };
      auto put = [&](int r, int c, float v) {
        tw(r, c) = v;
        *reinterpret_cast<float*>(sT + gdn_sw(r, c, 2 * C)) = to_tf32(v * bs[c]);
      };
      if (tid < C) {
        const int b0 = (tid >> 4) * 16, c = tid & 15;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
          const float* arow = As + (b0 + r) * LDA + b0;
          float acc0 = r == c ? 1.f : 0.f, acc1 = 0.f;
#pragma unroll
          for (int j = 0; j < r; ++j) {
            if (j & 1)
              acc1 = fmaf(arow[j], x[j], acc1);
            else
              acc0 = fmaf(arow[j], x[j], acc0);
          }
          x[r] = acc0 + acc1;
          put(b0 + r, b0 + c, x[r]);
        }
      }
      __syncthreads();
      // pairs of 16-blocks: Y = A[B0 + r][A0 + k] T[A0 + k][A0 + c]  (T's upper parts are zero)
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int a0b = 32 * m, b0b = a0b + 16, r = tid >> 4, c = tid & 15;
        const float* arow = As + (b0b + r) * LDA + a0b;
        float acc = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < 16; k4 += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(arow + k4);
          acc = fmaf(a4.x, tw(a0b + k4, a0b + c), acc);
          acc = fmaf(a4.y, tw(a0b + k4 + 1, a0b + c), acc);
          acc = fmaf(a4.z, tw(a0b + k4 + 2, a0b + c), acc);
          acc = fmaf(a4.w, tw(a0b + k4 + 3, a0b + c), acc);
        }
        yb[m * 16 * 17 + r * 17 + c] = acc;
      }
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const int a0b = 32 * m, b0b = a0b + 16, r = tid >> 4, c = tid & 15;
        float acc = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < 16; k4 += 4) {
          const float4 t4 = tw4(b0b + r, b0b + k4);
          acc = fmaf(t4.x, yb[m * 16 * 17 + k4 * 17 + c], acc);
          acc = fmaf(t4.y, yb[m * 16 * 17 + (k4 + 1) * 17 + c], acc);
          acc = fmaf(t4.z, yb[m * 16 * 17 + (k4 + 2) * 17 + c], acc);
          acc = fmaf(t4.w, yb[m * 16 * 17 + (k4 + 3) * 17 + c], acc);
        }
        put(b0b + r, a0b + c, acc);
      }
      __syncthreads();
      // the two halves: Y = A[32 + r][k] T[k][c], then T[32 + r][c] = T[32 + r][32 + k] Y[k][c]
      {
        const int c = tid & 31, r0 = tid >> 5;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int k4 = 0; k4 < 32; k4 += 4) {
          float t[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) t[e] = tw(k4 + e, c);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float4 a4 = *reinterpret_cast<const float4*>(As + (32 + r0 + 8 * m) * LDA + k4);
            acc[m] = fmaf(a4.x, t[0], acc[m]);
            acc[m] = fmaf(a4.y, t[1], acc[m]);
            acc[m] = fmaf(a4.z, t[2], acc[m]);
            acc[m] = fmaf(a4.w, t[3], acc[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) yb[(r0 + 8 * m) * 33 + c] = acc[m];
        __syncthreads();
#pragma unroll
        for (int m = 0; m < 4; ++m) acc[m] = 0.f;
#pragma unroll
        for (int k4 = 0; k4 < 32; k4 += 4) {
          float y[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) y[e] = yb[(k4 + e) * 33 + c];
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const float4 t4 = tw4(32 + r0 + 8 * m, 32 + k4);
            acc[m] = fmaf(t4.x, y[0], acc[m]);
            acc[m] = fmaf(t4.y, y[1], acc[m]);
            acc[m] = fmaf(t4.z, y[2], acc[m]);
            acc[m] = fmaf(t4.w, y[3], acc[m]);
          }
        }
#pragma unroll
        for (int m = 0; m < 4; ++m) put(32 + r0 + 8 * m, c, acc[m]);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // the system matrix is done with: each output thread stages its z row
    // segment (64 bf16) there for the O phase
    if (lrow >= C) {
      const int c = lrow - C, t = t0 + c;
      const T* src = proj + (row0 + (t < a.S ? t : 0)) * a.ldp + a.z_col + h * DH + 64 * half;
      T* dst = reinterpret_cast<T*>(As) + c * Sh::ZLD + 64 * half;
#pragma unroll
      for (int e8 = 0; e8 < 64; e8 += 8) cp_async16(dst + e8, src + e8, t < a.S);
      cp_async_commit();
    }
    // ---- MV: D_V = [T diag(beta); T] R (lanes 64-127 unused) ----
    if (tid == 32) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < C / 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
        umma_tf32(tmem + Sh::DV, smem_desc_k128(st + aoff), smem_desc_mn128_32b(sv + kk * 1024, C * 128), IDESC_N,
                  kk > 0 ? 1u : 0u);
      }
      umma_commit(mma_bar);
    }
    if (!mma_wait()) break;
    // ---- V_new (lanes 0-63) -> the B operand tile, in place of R ----
    if (lrow < C) {
      const int c = lrow;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t d[32];
        const int j0 = 64 * half + 32 * part;
        tmem_ld32(tmem + t_lane + Sh::DV + j0, d);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(sV + gdn_sw_mn(c, j0 + e, C)) =
              make_float4(to_tf32(__uint_as_float(d[e])), to_tf32(__uint_as_float(d[e + 1])),
                          to_tf32(__uint_as_float(d[e + 2])), to_tf32(__uint_as_float(d[e + 3])));
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- M3: D3 = M V_new (over the MV product);  M4: D2 = K~^T V_new ----
    if (tid == 32) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < C / 8; ++kk) {
        const uint64_t bdesc = smem_desc_mn128_32b(sv + kk * 1024, C * 128);
        umma_tf32_ts(tmem + Sh::DV, tmem + Sh::D0 + kk * 8, bdesc, IDESC_N, kk > 0 ? 1u : 0u);
        umma_tf32_ts(tmem + Sh::D2, tmem + Sh::KT + kk * 8, bdesc, IDESC_N, kk > 0 ? 1u : 0u);
      }
      umma_commit(mma_bar);
    }
    if (!mma_wait()) break;
    // ---- O1 (lanes 64-127): o = T(e^g (q S) + M V_new) into the A0 tile, which
    // no MMA reads any more this chunk (rows of 132 floats), and each row
    // half's sum of squares ----
    constexpr int OLD = DH + 4;
    float* ob = reinterpret_cast<float*>(sA0);
    if (lrow >= C) {
      const int c = lrow - C;
      const float ec = es[c];
      float sq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t d[32], m[32];
        const int j0 = 64 * half + 32 * part;
        tmem_ld32(tmem + t_lane + Sh::D1 + j0, d);
        tmem_ld32(tmem + t_lane + Sh::DV + j0, m);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float4 o4;
          o4.x = round_to<T>(fmaf(ec, __uint_as_float(d[e]), __uint_as_float(m[e])));
          o4.y = round_to<T>(fmaf(ec, __uint_as_float(d[e + 1]), __uint_as_float(m[e + 1])));
          o4.z = round_to<T>(fmaf(ec, __uint_as_float(d[e + 2]), __uint_as_float(m[e + 2])));
          o4.w = round_to<T>(fmaf(ec, __uint_as_float(d[e + 3]), __uint_as_float(m[e + 3])));
          sq[0] = fmaf(o4.x, o4.x, sq[0]);
          sq[1] = fmaf(o4.y, o4.y, sq[1]);
          sq[2] = fmaf(o4.z, o4.z, sq[2]);
          sq[3] = fmaf(o4.w, o4.w, sq[3]);
          *reinterpret_cast<float4*>(ob + c * OLD + j0 + e) = o4;
        }
      }
      red[half * C + c] = (sq[0] + sq[1]) + (sq[2] + sq[3]);
      cp_async_wait<0>();  // this thread's z copies, read by others after the barrier
    }
    // ---- S = S e^{g_last} + D2 (lane = key dim, 64 value columns per thread) ----
    {
      const float decay = es[C - 1];
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        uint32_t d[32];
        const int j0 = 64 * half + 32 * part;
        tmem_ld32(tmem + t_lane + Sh::D2 + j0, d);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; e += 4) {
          float4* p = reinterpret_cast<float4*>(sS + gdn_sw_mn(lrow, j0 + e, DH));
          float4 s = *p;
          s.x = to_tf32(fmaf(s.x, decay, __uint_as_float(d[e])));
          s.y = to_tf32(fmaf(s.y, decay, __uint_as_float(d[e + 1])));
          s.z = to_tf32(fmaf(s.z, decay, __uint_as_float(d[e + 2])));
          s.w = to_tf32(fmaf(s.w, decay, __uint_as_float(d[e + 3])));
          *p = s;
        }
      }
    }
    __syncthreads();
    // ---- O2 (all threads, one row per lane, 32 columns per warp quarter of
    // the CTA): gated RMSNorm x SiLU(z) (text.py:61-67) ----
    {
      const int c = tid & (C - 1), q32 = (tid >> 6) * 32, t = t0 + c;
      if (t < a.S) {
        const float rs = rsqrtf((red[c] + red[C + c]) / DH + a.eps);
        const T* zrow = reinterpret_cast<const T*>(As) + c * Sh::ZLD + q32;
        const float* orow_s = ob + c * OLD + q32;
        T* orow = out + (row0 + t) * a.ldo + h * DH + q32;
#pragma unroll
        for (int e8 = 0; e8 < 32; e8 += 8) {
          GdnVec<T> z, res;
          z.load(zrow + e8);
          const float4 o0 = *reinterpret_cast<const float4*>(orow_s + e8);
          const float4 o1 = *reinterpret_cast<const float4*>(orow_s + e8 + 4);
          const float o[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float n = round_to<T>(round_to<T>(o[e] * rs) * nws[q32 + e8 + e]);
            res.v[e] = n * (z.v[e] * sigmoid_fast(z.v[e]));
          }
          res.store(orow + e8);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, Sh::TMEM_COLS);
}

}  // namespace clef

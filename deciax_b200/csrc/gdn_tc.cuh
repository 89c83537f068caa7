// Gated DeltaNet mixer core on the 5th-generation tensor cores (sm_100a),
// BF16 activations, head dim 128: qwen3_5/text.py:48-67 with the chunked rule
// of kernels/gdn/reference.py:40-92, in three passes over 64-token chunks.
//
//   conv   causal conv + SiLU and the q/k L2 norms of every head
//          (text.py:31-39, reference.py:14-21), bf16 rows [B*S, (2 nh + nv) 128].
//   prep   per (chunk, value head, state), all in parallel: the gates
//          g = cumsum(-e^A_log softplus(a + dt_bias)), beta = sigmoid(b)
//          (text.py:54-55); k k^T and q k^T (tcgen05 kind::f16, exact on the
//          bf16 values); the system A = -(k beta k^T) * decay and its inverse
//          T = (I - A)^{-1} (reference.py:73-80, blocked, FP32 on the CUDA
//          cores); M = (q k^T dk^-1/2) * decay (c' <= c).  Writes one record:
//          the A operand tile [T diag(beta); M] in the chain's layout and the
//          gates e^g, e^{g_C - g}.
//   chain  per (value head, state), the chunks in sequence with the FP32
//          state S [dk, dv] in shared memory as a tcgen05 B operand:
//            M1 D1 = [k; q] S;  R = v - e^g (k S);
//            MV V_new = T diag(beta) R  (reference.py:81-83's
//               T (v beta) - T (k beta e^g) S, regrouped so that no product
//               with T runs over the value and the key dims separately);
//            M3 M V_new;  M4 D2 = K~^T V_new, K~ = k e^{g_C - g};
//            o = e^g (q S) + M V_new (reference.py:85), S = S e^{g_C} + D2
//            (reference.py:86), then the gated RMSNorm x SiLU(z)
//            (text.py:61-67).
// Products in the chain run as kind::tf32 (operands rounded to TF32, FP32
// accumulation); the inverse, the gates and every elementwise step are FP32.
// The FP32 parity mode keeps the all-FP32 CUDA-core kernel (gdn.cuh).
//
// Operand tiles are rows of 32 fp32 (128 B) in atoms of `rows` rows per 32
// columns: a K-major operand [M or N rows][K] with the 128-byte swizzle
// (16-byte chunks XOR row % 8), an MN-major one [K rows][M or N] with the
// 128-byte swizzle of 32-byte atomicity (32-byte chunks XOR row % 4), the only
// swizzle tcgen05 takes for 32-bit MN-major operands.  One thread issues the
// MMAs and commits to one mbarrier; every wait is bounded.  Rows past the
// sequence end are zero with g = beta = 0, as the reference's padding.
#pragma once

#include "attention_sm100.cuh"
#include "common.cuh"
#include "gdn.cuh"

namespace clef {

constexpr int kGdnTcDim = 128;

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

// gdn_mn_half: a thread that updates row r of such a tile visits the two
// 16-byte halves of each 32-byte chunk in the order given by bit 2 of r.  Rows
// r and r + 4 put a column in the same chunk position under the swizzle, so a
// warp of 32 consecutive rows then covers all 32 banks per float4 access (4
// wavefronts instead of 8).

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

// Conv pass: causal conv + SiLU (text.py:31-39) of every q, k and v channel
// and the L2 norms of q and k (reference.py:14-21).  q and k leave as bf16
// rows [B*S, 2*nh*dh] (q heads, k heads; q without the dk^-1/2 factor) for the
// prep pass and as the chain's TF32 operand tiles [k; q dk^-1/2] per (state,
// key head, chunk); v leaves as the chain's MN-major tile per (state, value
// head, chunk).  Every value is one the reference rounds to bf16, so the prep
// and chain passes read exactly the values the CUDA-core kernel computes in
// place; rows past the sequence end are zero in the tiles.  One CTA per (256-token span, q/k/v head, state): the
// q and k heads are computed once, not once per value head that shares them,
// and the pass runs at full occupancy (each CTA walks kGdnConvBlocks blocks
// with its taps in registers).  The sliding-window arithmetic is
// gdn_load_chunk's (same taps, same order of operations).
constexpr int kGdnConvBlocks = 4;  // 64-token blocks per CTA of the conv pass

template <int W>
__global__ void __launch_bounds__(kGdnThreads, W <= 4 ? 3 : 1) gdn_conv_bf16_kernel(GdnArgs a) {
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
  const int shift = W - a.width, chunks = (a.S + C - 1) / C;
  float w[VN][W];  // this thread's taps, loaded once for all its blocks
#pragma unroll
  for (int c = 0; c < VN; ++c)
#pragma unroll
    for (int i = 0; i < W; ++i)
      w[c][i] = i >= shift ? to_f32(convw[static_cast<long long>(col + c) * a.width + (i - shift)]) : 0.f;
  for (int blk = 0; blk < kGdnConvBlocks; ++blk) {
    const int t0 = (blockIdx.x * kGdnConvBlocks + blk) * C;  // uniform across the CTA
    if (t0 >= a.S) break;
    uint32_t x[NX][VN / 2];  // the window's bf16 pairs, widened where used (exact)
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      const int tt = t0 + r0 - (W - 1) + i;
      const uint4 raw = (tt >= 0 && tt < a.S) ? *reinterpret_cast<const uint4*>(proj + (row0 + tt) * a.ldp + col)
                                              : make_uint4(0u, 0u, 0u, 0u);
      x[i][0] = raw.x;
      x[i][1] = raw.y;
      x[i][2] = raw.z;
      x[i][3] = raw.w;
    }
    auto xv = [&](int i, int c) -> float {  // channel c of window row i
      const uint32_t u = x[i][c >> 1];
      return __uint_as_float((c & 1) ? (u & 0xFFFF0000u) : (u << 16));
    };
#pragma unroll
    for (int j = 0; j < RT; ++j) {
      const int t = t0 + r0 + j;
      GdnVec<T> y;
#pragma unroll
      for (int c = 0; c < VN; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < W; ++i) acc = __fadd_rn(acc, __fmul_rn(xv(j + i, c), w[c][i]));
        y.v[c] = acc;
      }
      // bf16 roundings in pairs: z = T(acc), y = T(z sigmoid(z)) (text.py:31-39)
#pragma unroll
      for (int c = 0; c < VN; c += 2) round2_bf16(y.v[c], y.v[c + 1]);
#pragma unroll
      for (int c = 0; c < VN; ++c) y.v[c] *= sigmoid_fast(y.v[c]);
#pragma unroll
      for (int c = 0; c < VN; c += 2) round2_bf16(y.v[c], y.v[c + 1]);
      if (t >= a.S) y.zero();
      if (kind < 2) {
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < VN; ++c) ss += y.v[c] * y.v[c];
        const float inv = rsqrtf(group_sum<GL>(ss) + 1e-6f);
#pragma unroll
        for (int c = 0; c < VN; c += 2) {
          y.v[c] *= inv;
          y.v[c + 1] *= inv;
          round2_bf16(y.v[c], y.v[c + 1]);
        }
      }
      const int rr = r0 + j, ci = t0 / C;
      if (kind < 2) {
        if (t < a.S) y.store(dst + (row0 + t) * a.ldc + kh * DH + g * VN);
        // the chain's operand tile: k -> rows 0-63, q x dk^-1/2 (TF32) -> rows 64-127
        const int hk = kind == 0 ? kh : kh - a.nh;
        uint8_t* tile = static_cast<uint8_t*>(a.a0_tiles) +
                        ((static_cast<long long>(b) * a.nh + hk) * chunks + ci) * static_cast<long long>(2 * C * DH * 4);
        float o[VN];
#pragma unroll
        for (int c = 0; c < VN; ++c) o[c] = kind == 0 ? to_tf32(y.v[c] * a.qscale) : y.v[c];
        const int row = kind == 1 ? rr : C + rr;
#pragma unroll
        for (int c = 0; c < VN; c += 4)
          *reinterpret_cast<float4*>(tile + gdn_sw(row, g * VN + c, 2 * C)) = make_float4(o[c], o[c + 1], o[c + 2], o[c + 3]);
      } else {
        // the chain's v tile (MN-major: token rows, value-dim columns)
        uint8_t* tile = static_cast<uint8_t*>(a.v_tiles) +
                        ((static_cast<long long>(b) * a.nv + (kh - 2 * a.nh)) * chunks + ci) * static_cast<long long>(C * DH * 4);
#pragma unroll
        for (int c = 0; c < VN; c += 4)
          *reinterpret_cast<float4*>(tile + gdn_sw_mn(rr, g * VN + c, C)) =
              make_float4(y.v[c], y.v[c + 1], y.v[c + 2], y.v[c + 3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Prep pass: the state-independent half of every chunk, all chunks at once.
// ---------------------------------------------------------------------------

// Per (chunk, value head, state): the A operand tile [T diag(beta); M] of the
// chain kernel's V_new and output products (K-major fp32, 128 rows x 64,
// the 128-byte swizzle of gdn_sw) and the chunk's gates e^g and e^(g_C - g).
struct GdnPrepShape {
  static constexpr int C = kGdnChunk, DH = kGdnTcDim, LDA = C + 4;
  static constexpr uint32_t TILE_BYTES = 2 * C * C * 4;           // [T diag(beta); M]
  static constexpr uint32_t GATE_BYTES = 2 * C * 4;               // e^g, e^(g_C - g)
  static constexpr uint32_t OUT_BYTES = TILE_BYTES + GATE_BYTES;  // per (chunk, value head, state)
  static constexpr uint32_t A0_BYTES = 2 * C * DH * 2;            // [k; q] bf16, K-major [128 rows][dk];
                                                                  // after the MMA: system matrix + inverse blocks
  static constexpr uint32_t TW_BYTES = C * LDA * 4;               // the unscaled inverse, row-major
  static constexpr uint32_t MISC_FLOATS = 4 * C;                  // gates
  static_assert(C * LDA * 4 + 32 * 33 * 4 <= A0_BYTES, "system matrix and blocks over the operand tile");
  static constexpr size_t SMEM = 1024 + A0_BYTES + TW_BYTES + MISC_FLOATS * 4 + 32;  // + 2 mbarriers, TMEM slot
  static constexpr uint32_t TMEM_COLS = 64;                       // D0 = [k; q] k^T
  static constexpr int CTAS_PER_SM = 4;
};

// Byte offset of element (row, col) of a K-major bf16 operand tile in atoms
// of `rows` rows x 64 columns, with the 128-byte swizzle.
__device__ __forceinline__ uint32_t gdn_sw16(int row, int col, int rows) {
  return static_cast<uint32_t>((col >> 6) * (rows * 128) + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) +
                               ((col & 7) << 1));
}

// The blocked inverse T = (I - A)^{-1} of a chunk's unit lower-triangular
// system (reference.py:73-80) into Tw [C][LDA] (zero on entry: blocks above
// the diagonal are never written).  As [C][LDA] holds A (minus the matrix's
// off-diagonal).  Diagonal 16 x 16 blocks by forward substitution; then for
// [[P, 0], [Q, R]] with known inverses P', R' the lower-left block of the
// inverse is R' (Q~ P'), first for the 16 x 16 pairs of blocks, then for the
// two 32 x 32 halves.  All threads of the CTA (kGdnThreads) take part.
__device__ __forceinline__ void gdn_blocked_inverse(float* Tw, const float* As, float* yb, int tid) {
  constexpr int C = kGdnChunk, LDA = C + 4;
  auto tw4 = [&](int r, int c4) -> float4 { return *reinterpret_cast<const float4*>(Tw + r * LDA + c4); };
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
      Tw[(b0 + r) * LDA + b0 + c] = x[r];
    }
  }
  __syncthreads();
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    const int a0b = 32 * m, b0b = a0b + 16, r = tid >> 4, c = tid & 15;
    const float* arow = As + (b0b + r) * LDA + a0b;
    float acc = 0.f;
#pragma unroll
    for (int k4 = 0; k4 < 16; k4 += 4) {
      const float4 a4 = *reinterpret_cast<const float4*>(arow + k4);
      acc = fmaf(a4.x, Tw[(a0b + k4) * LDA + a0b + c], acc);
      acc = fmaf(a4.y, Tw[(a0b + k4 + 1) * LDA + a0b + c], acc);
      acc = fmaf(a4.z, Tw[(a0b + k4 + 2) * LDA + a0b + c], acc);
      acc = fmaf(a4.w, Tw[(a0b + k4 + 3) * LDA + a0b + c], acc);
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
    Tw[(b0b + r) * LDA + a0b + c] = acc;
  }
  __syncthreads();
  {
    const int c = tid & 31, r0 = tid >> 5;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k4 = 0; k4 < 32; k4 += 4) {
      float t[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t[e] = Tw[(k4 + e) * LDA + c];
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
    for (int m = 0; m < 4; ++m) Tw[(32 + r0 + 8 * m) * LDA + c] = acc[m];
  }
}

// Untiled bulk copy of `bytes` (a multiple of 16) from this CTA's shared
// memory to global memory (both 16-byte aligned), in the current bulk group.
__device__ __forceinline__ void gdn_bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}

// 3-D tiled load (x = column, y = row, z = state) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// One CTA per (chunk, key head, state), for each value head of the key head's
// group in turn: gates (text.py:54-55: g = -e^A_log softplus(a + dt_bias),
// beta = sigmoid(b); their in-chunk cumsum), the system matrix A = -(k beta
// k^T) * decay (strictly lower), M = (q k^T dk^-1/2) * decay (c' <= c, TF32)
// and the inverse; writes [T diag(beta); M] in the chain kernel's operand
// layout and the gates e^g, e^(g_C - g).  k k^T and q k^T are shared by the
// group: one TMA load of the bf16 [k; q] tile (the conv pass's rows, as a
// [state][token][column] tensor: tokens past the sequence end read zero) and
// one tcgen05 kind::f16 product (exact on bf16 values; dk^-1/2 applied after),
// kept in tensor memory.  Four CTAs per SM hide each other's phase latencies.
__global__ void __launch_bounds__(kGdnThreads, GdnPrepShape::CTAS_PER_SM)
    gdn_prep_kernel(const __grid_constant__ CUtensorMap qk_map, GdnArgs a) {
  using Sh = GdnPrepShape;
  using T = __nv_bfloat16;
  constexpr int C = Sh::C, DH = Sh::DH, LDA = Sh::LDA;
  constexpr uint32_t IDESC = idesc_bf16_f32(2 * C, C);  // [k; q] k^T: both K-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA0 = smem;
  float* As = reinterpret_cast<float*>(sA0);  // over the operand tile once the MMA is done: [C][LDA]
  float* yb = As + C * LDA;                   // [32][33]
  float* Tw = reinterpret_cast<float*>(sA0 + Sh::A0_BYTES);
  float* gs = Tw + C * LDA;  // cumulative g
  float* bs = gs + C;        // beta
  float* es = bs + C;        // e^g
  float* ws = es + C;        // e^(g_last - g)
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(ws + C);
  uint64_t* load_bar = mma_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(load_bar + 1);

  const int ci = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const int lrow = quarter * 32 + lane;
  const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
  const int group = a.nv / a.nh, t0 = ci * C;
  const T* proj = static_cast<const T*>(a.proj);
  const long long row0 = static_cast<long long>(b) * a.S;
  const int chunks = (a.S + C - 1) / C;

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    mbar_init(load_bar, 1);
    fence_barrier_init();
    prefetch_tmap(&qk_map);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Sh::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tid == 0) {  // k -> rows 0-63, q -> rows 64-127 of each 64-column atom
    mbar_arrive_expect_tx(load_bar, Sh::A0_BYTES);
#pragma unroll
    for (int atom = 0; atom < DH / 64; ++atom) {
      uint8_t* dst = sA0 + atom * (2 * C * 128);
      tma_load_3d(dst, &qk_map, load_bar, (a.nh + hk) * DH + 64 * atom, t0, b);
      tma_load_3d(dst + C * 128, &qk_map, load_bar, hk * DH + 64 * atom, t0, b);
    }
  }
  const bool load_ok = mbar_wait(load_bar, 0, a.status, kTimeoutMma);
  const bool loaded = __syncthreads_and(load_ok) != 0;
  if (loaded && tid == 32) {
    tc_fence_after();
    const uint32_t a0 = smem_u32(sA0);
#pragma unroll
    for (int kk = 0; kk < DH / 16; ++kk) {
      const uint32_t off = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
      umma_bf16(tmem, smem_desc_k128(a0 + off), smem_desc_k128(a0 + off), IDESC, kk > 0 ? 1u : 0u);
    }
    umma_commit(mma_bar);
  }
  const bool ok = loaded && mbar_wait(mma_bar, 0, a.status, kTimeoutMma);
  tc_fence_after();
  if (!__syncthreads_and(ok)) {
    // a load that a failed wait left in flight lands before shared memory is
    // released (bounded: the status is already set)
    if (tid == 0 && !load_ok) mbar_wait(load_bar, 0, a.status, kTimeoutMma);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, Sh::TMEM_COLS);
    return;
  }

  for (int g = 0; g < group; ++g) {
    const int h = hk * group + g;
    uint8_t* outp = static_cast<uint8_t*>(a.prep) +
                    ((static_cast<long long>(b) * a.nv + h) * chunks + ci) * static_cast<long long>(Sh::OUT_BYTES);
    if (tid < C) {
      const bool row = t0 + tid < a.S;
      float ga = 0.f, gb = 0.f;
      if (row) {
        const T* pr = proj + (row0 + t0 + tid) * a.ldp;
        ga = to_f32(pr[a.a_col + h]);
        gb = to_f32(pr[a.b_col + h]);
      }
      const float neg_a = -expf(to_f32(static_cast<const T*>(a.A_log)[h]));
      const float dt_bias = to_f32(static_cast<const T*>(a.dt_bias)[h]);
      gs[tid] = row ? neg_a * softplus_f(ga + dt_bias) : 0.f;
      bs[tid] = row ? round_to<T>(sigmoid_fast(gb)) : 0.f;
    }
    for (int i = tid; i < C * LDA / 4; i += kGdnThreads) reinterpret_cast<float4*>(Tw)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g > 0 && tid == 0) tma_store_wait_read();  // the previous record has left shared memory
    __syncthreads();
    if (warp == 0) {  // cumulative gate (sequential, as cumsum) and its exponentials
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
    __syncthreads();
    // system matrix (lanes 0-63, over the operand tile the MMA has read)
    if (lrow < C) {
      uint32_t d[32];
      tmem_ld32(tmem + t_lane + 32 * half, d);
      tmem_wait_ld();
      const int i = lrow;
      const float gi = gs[i], bi = bs[i];
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float a4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = 32 * half + e + u;
          a4[u] = j < i ? -(__uint_as_float(d[e + u]) * bi) * exp_fast(gi - gs[j]) : 0.f;
        }
        *reinterpret_cast<float4*>(As + i * LDA + 32 * half + e) = make_float4(a4[0], a4[1], a4[2], a4[3]);
      }
    }
    __syncthreads();
    gdn_blocked_inverse(Tw, As, yb, tid);
    __syncthreads();
    // the record in shared memory, over the system matrix: rows 0-63 T diag(beta),
    // rows 64-127 M = (q k^T dk^-1/2) * decay (c' <= c), both rounded to TF32
    if (lrow < C) {
      const int r = lrow;
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const int c4 = 32 * half + e;
        const float4 t4 = *reinterpret_cast<const float4*>(Tw + r * LDA + c4);
        *reinterpret_cast<float4*>(sA0 + gdn_sw(r, c4, 2 * C)) =
            make_float4(to_tf32(t4.x * bs[c4]), to_tf32(t4.y * bs[c4 + 1]), to_tf32(t4.z * bs[c4 + 2]),
                        to_tf32(t4.w * bs[c4 + 3]));
      }
    } else {
      uint32_t d[32];
      tmem_ld32(tmem + t_lane + 32 * half, d);
      tmem_wait_ld();
      const int i = lrow - C;
      const float gi = gs[i];
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float m4[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = 32 * half + e + u;
          m4[u] = j <= i ? to_tf32(__uint_as_float(d[e + u]) * a.qscale * exp_fast(gi - gs[j])) : 0.f;
        }
        *reinterpret_cast<float4*>(sA0 + gdn_sw(lrow, 32 * half + e, 2 * C)) = make_float4(m4[0], m4[1], m4[2], m4[3]);
      }
    }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {  // tile and gates (es, ws adjacent) by two bulk stores
      gdn_bulk_store(outp, sA0, Sh::TILE_BYTES);
      gdn_bulk_store(outp + Sh::TILE_BYTES, es, Sh::GATE_BYTES);
      tma_store_commit();
    }
  }
  if (tid == 0) tma_store_wait_read();  // shared memory stays valid until the copies have read it
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, Sh::TMEM_COLS);
}

// ---------------------------------------------------------------------------
// Chain pass: the state-dependent half of every chunk, in sequence.
// ---------------------------------------------------------------------------

struct GdnChainShape {
  static constexpr int C = kGdnChunk, DH = kGdnTcDim;
  static constexpr uint32_t S_BYTES = DH * DH * 4;        // state, MN-major B [dk rows][dv]
  static constexpr uint32_t A0_BYTES = 2 * C * DH * 4;    // [k; q dk^-1/2], K-major [128 rows][dk]
  static constexpr uint32_t V_BYTES = C * DH * 4;         // v -> R -> V_new, MN-major [tokens][dv]
  static constexpr uint32_t T_BYTES = GdnPrepShape::TILE_BYTES;  // [T diag(beta); M] of the prep pass
  static constexpr uint32_t G_BYTES = 2 * GdnPrepShape::GATE_BYTES;  // two chunks' gates
  static constexpr int ZLD = DH + 8;                      // z rows: bf16, 272-byte rows
  static constexpr uint32_t Z_BYTES = C * ZLD * 2;
  static constexpr uint32_t MISC_FLOATS = 2 * C + DH;     // output-row sums of squares, norm weight
  static constexpr size_t SMEM = 1024 + S_BYTES + A0_BYTES + V_BYTES + T_BYTES + G_BYTES + Z_BYTES + MISC_FLOATS * 4 + 64;  // + 5 mbarriers, TMEM slot
  static constexpr uint32_t D1 = 0, DV = 128, D2 = 256, KT = 384, TMEM_COLS = 512;
  static_assert(GdnPrepShape::TILE_BYTES % 16 == 0 && GdnPrepShape::GATE_BYTES % 16 == 0 &&
                    GdnPrepShape::OUT_BYTES % 16 == 0,
                "bulk copies move 16-byte multiples from 16-byte aligned records");
};

// Scratch of the tensor-core path for B states of S tokens, in order, each part
// 256-byte aligned: the conv pass's bf16 q/k rows [B*S, 2 nh 128] (q heads, k
// heads), the chain's [k; q dk^-1/2] operand tiles (GdnChainShape::A0_BYTES per
// state, key head and chunk), its v tiles (V_BYTES per state, value head and
// chunk), and the prep pass's records (GdnPrepShape::OUT_BYTES per state, value
// head and chunk).
struct GdnTcScratch {
  size_t rows = 0, a0 = 0, v = 0, prep = 0, total = 0;
  GdnTcScratch(int B, int S, int nh, int nv);
};

inline GdnTcScratch::GdnTcScratch(int B, int S, int nh, int nv) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t chunks = (static_cast<size_t>(S) + kGdnChunk - 1) / kGdnChunk;
  rows = 0;
  a0 = up(static_cast<size_t>(B) * S * 2 * nh * kGdnTcDim * 2);
  v = a0 + up(static_cast<size_t>(B) * nh * chunks * GdnChainShape::A0_BYTES);
  prep = v + up(static_cast<size_t>(B) * nv * chunks * GdnChainShape::V_BYTES);
  total = prep + static_cast<size_t>(B) * nv * chunks * GdnPrepShape::OUT_BYTES;
}

inline size_t gdn_tc_scratch_bytes(int B, int S, int nh, int nv) { return GdnTcScratch(B, S, nh, nv).total; }

// Point a's tensor-core buffers into `base` (gdn_tc_scratch_bytes(a.B, a.S, a.nh, a.nv) bytes).
inline void gdn_tc_bind_scratch(GdnArgs& a, void* base) {
  const GdnTcScratch sc(a.B, a.S, a.nh, a.nv);
  uint8_t* p = static_cast<uint8_t*>(base);
  a.qkv_conv = p + sc.rows;
  a.ldc = 2LL * a.nh * kGdnTcDim;
  a.a0_tiles = p + sc.a0;
  a.v_tiles = p + sc.v;
  a.prep = p + sc.prep;
}

// Untiled bulk copy global -> this CTA's shared memory, completing on `bar`
// (both addresses 16-byte aligned, `bytes` a multiple of 16).
__device__ __forceinline__ void gdn_bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Output row staging over the (read) operand tile: row c, columns j, 128
// floats per row with 16-byte chunks XOR-permuted by c % 32 (a warp's 32 rows
// at one column fall in distinct chunks).
__device__ __forceinline__ int gdn_ob(int c, int j) { return c * 128 + (((j >> 2) ^ (c & 31)) << 2) + (j & 3); }

// One CTA per (value head, state) walks the chunks with the FP32 state S in
// shared memory.  Per chunk, everything it reads arrives by bulk copy while
// the previous chunk finishes: the conv pass's TF32 operand tiles A0 = [k; q
// dk^-1/2] (once the previous chunk's K~^T has read A0) and V (once its last
// products have read V), the prep pass's gates (with V) and its tile
// [T diag(beta); M] (once the previous chunk's output rows are read);
//   M1 D1 = A0 S (rows 0-63 k S, rows 64-127 q S);
//   P  K~^T = (k e^{g_C - g})^T into tensor memory (lanes 0-63: during the previous
//      chunk's output phase); R = v - e^g (k S) in place of v;
//   MV D_V = [T diag(beta); M] R: rows 0-63 V_new, stored in place of R;
//   M3 D_V = [T diag(beta); M] V_new: rows 64-127 M V_new; M4 D2 = K~^T V_new;
//   O  lanes 64-127 (warps 2, 3, 6, 7): rows e^g (q S) + M V_new
//      (reference.py:85) over the tile, S = S e^{g_C} + D2 (reference.py:86)
//      on their lanes; lanes 0-63 (warps 0, 1, 4, 5): the state update on
//      theirs; then the next chunk's M1 is issued and all warps apply the
//      gated RMSNorm x SiLU(z) (text.py:61-67) while it runs.
// Tensor memory: D1 [0, 128), D_V [128, 256), D2 [256, 384), K~^T [384, 448).
__global__ void __launch_bounds__(kGdnThreads, 1) gdn_chain_kernel(GdnArgs a) {
  using Sh = GdnChainShape;
  using T = __nv_bfloat16;
  constexpr int C = Sh::C, DH = Sh::DH;
  constexpr uint32_t IDESC_N = idesc_tf32_f32(128, DH, false, true);  // x S, [T; M] R, [T; M] V_new, (tmem A) V_new

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sS = smem;
  uint8_t* sA0 = sS + Sh::S_BYTES;
  uint8_t* sV = sA0 + Sh::A0_BYTES;
  uint8_t* sT = sV + Sh::V_BYTES;
  float* ob = reinterpret_cast<float*>(sT);                       // output rows, once the tile is read
  float* gates = reinterpret_cast<float*>(sT + Sh::T_BYTES);      // [2][e^g (C), e^(g_C - g) (C)]
  T* zs = reinterpret_cast<T*>(gates + 4 * C);                    // [C][ZLD]
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(zs) + Sh::Z_BYTES);  // [2][C]
  float* nws = red + 2 * C;                                       // gated-norm weight
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(nws + DH);
  uint64_t* tile_bar = mma_bar + 1;
  uint64_t* gate_bar = tile_bar + 1;
  uint64_t* a0_bar = gate_bar + 1;
  uint64_t* v_bar = a0_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(v_bar + 1);
  static_assert(C * 128 * 4 <= Sh::T_BYTES, "output rows over the tile");

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, half = warp >> 2;  // tensor-memory lane quarter, column half
  const int lrow = quarter * 32 + lane;            // this thread's tensor-memory lane
  const uint32_t t_lane = static_cast<uint32_t>(quarter * 32) << 16;
  const int hk = h / (a.nv / a.nh);
  const T* proj = static_cast<const T*>(a.proj);
  const T* nw = static_cast<const T*>(a.norm_w);
  T* out = static_cast<T*>(a.out);
  const long long row0 = static_cast<long long>(b) * a.S;
  const int chunks = (a.S + C - 1) / C;
  // the conv pass's operand tiles of this CTA's key head and value head, chunk 0
  const uint8_t* a0_src = static_cast<const uint8_t*>(a.a0_tiles) +
                          (static_cast<long long>(b) * a.nh + hk) * chunks * static_cast<long long>(Sh::A0_BYTES);
  const uint8_t* v_src = static_cast<const uint8_t*>(a.v_tiles) +
                         (static_cast<long long>(b) * a.nv + h) * chunks * static_cast<long long>(Sh::V_BYTES);
  const uint8_t* prep = static_cast<const uint8_t*>(a.prep) +
                        (static_cast<long long>(b) * a.nv + h) * chunks * static_cast<long long>(GdnPrepShape::OUT_BYTES);

  if (tid == 0) {
    mbar_init(mma_bar, 1);
    mbar_init(tile_bar, 1);
    mbar_init(gate_bar, 1);
    mbar_init(a0_bar, 1);
    mbar_init(v_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, Sh::TMEM_COLS);
    tmem_relinquish();
  }
  for (int i = tid; i < DH * DH; i += kGdnThreads) reinterpret_cast<float*>(sS)[i] = 0.f;  // S = 0 (any layout)
  if (tid < DH) nws[tid] = to_f32(nw[tid]);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint32_t mma_phase = 0, tile_phase = 0, gate_phase = 0, a0_phase = 0, v_phase = 0;
  bool tile_pending = false, gate_pending = false, a0_pending = false, v_pending = false;  // thread 0: copies in flight
  // chunk ci's record: the tile into sT, the gates into gates[ci & 1]
  auto load_tile = [&](int ci) {
    mbar_arrive_expect_tx(tile_bar, GdnPrepShape::TILE_BYTES);
    gdn_bulk_load(sT, prep + static_cast<long long>(ci) * GdnPrepShape::OUT_BYTES, GdnPrepShape::TILE_BYTES, tile_bar);
    tile_pending = true;
  };
  auto load_gates = [&](int ci) {
    mbar_arrive_expect_tx(gate_bar, GdnPrepShape::GATE_BYTES);
    gdn_bulk_load(gates + (ci & 1) * 2 * C,
                  prep + static_cast<long long>(ci) * GdnPrepShape::OUT_BYTES + GdnPrepShape::TILE_BYTES,
                  GdnPrepShape::GATE_BYTES, gate_bar);
    gate_pending = true;
  };
  // chunk ci's operand tiles: [k; q dk^-1/2] into A0, v into V
  auto load_a0 = [&](int ci) {
    mbar_arrive_expect_tx(a0_bar, Sh::A0_BYTES);
    gdn_bulk_load(sA0, a0_src + static_cast<long long>(ci) * Sh::A0_BYTES, Sh::A0_BYTES, a0_bar);
    a0_pending = true;
  };
  auto load_v = [&](int ci) {
    mbar_arrive_expect_tx(v_bar, Sh::V_BYTES);
    gdn_bulk_load(sV, v_src + static_cast<long long>(ci) * Sh::V_BYTES, Sh::V_BYTES, v_bar);
    v_pending = true;
  };
  if (tid == 0) {
    load_a0(0);
    load_v(0);
    load_gates(0);
    load_tile(0);
  }

  // One thread issues a group of MMAs and commits; everyone waits for it.
  auto mma_wait = [&]() -> bool {
    const bool ok = mbar_wait(mma_bar, mma_phase, a.status, kTimeoutMma);
    mma_phase ^= 1;
    tc_fence_after();
    return __syncthreads_and(ok) != 0;
  };
  // A bulk copy's wait: every thread sees its bytes; thread 0 tracks what is in flight.
  auto copy_wait = [&](uint64_t* bar, uint32_t& phase, bool& pending) -> bool {
    const bool ok = mbar_wait(bar, phase, a.status, kTimeoutMma);
    if (ok) {
      phase ^= 1;
      if (tid == 0) pending = false;
    }
    return ok;
  };

  const uint32_t a0 = smem_u32(sA0), sv = smem_u32(sV), st = smem_u32(sT), ss_addr = smem_u32(sS);
  // ---- M1: D1 = [k; q] S (the k operand values are exact in TF32: bf16 after
  // the norm), issued as soon as a chunk's A0 tile has landed and S is updated ----
  auto issue_m1 = [&]() {
#pragma unroll
    for (int kk = 0; kk < DH / 8; ++kk) {
      const uint32_t off = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
      umma_tf32(tmem + Sh::D1, smem_desc_k128(a0 + off), smem_desc_mn128_32b(ss_addr + kk * 1024, DH * 128), IDESC_N,
                kk > 0 ? 1u : 0u);
    }
    umma_commit(mma_bar);
  };
  if (tid == 32 && mbar_wait(a0_bar, a0_phase, a.status, kTimeoutMma)) issue_m1();
  for (int ci = 0; ci < chunks; ++ci) {
    const int t0 = ci * C;
    const float* es = gates + (ci & 1) * 2 * C;  // e^g
    const float* ws = es + C;                    // e^(g_last - g)
    // the chunk's z rows for the gated norm (16 threads per 256-byte row), and
    // the next chunk's z rows head for L2, while M1 runs
#pragma unroll
    for (int i = 0; i < C * 16 / kGdnThreads; ++i) {
      const int idx = tid + kGdnThreads * i, c = idx >> 4, e8 = (idx & 15) * 8, t = t0 + c;
      cp_async16(zs + c * Sh::ZLD + e8, proj + (row0 + (t < a.S ? t : 0)) * a.ldp + a.z_col + h * DH + e8, t < a.S);
    }
    cp_async_commit();
    if (tid < 2 * C && t0 + C + (tid >> 1) < a.S)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(proj + (row0 + t0 + C + (tid >> 1)) * a.ldp + a.z_col + h * DH +
                                                      64 * (tid & 1)));
    {
      const bool gate_ok = copy_wait(gate_bar, gate_phase, gate_pending);
      const bool a0_ok = copy_wait(a0_bar, a0_phase, a0_pending);
      const bool v_ok = copy_wait(v_bar, v_phase, v_pending);
      const bool mma_ok = mbar_wait(mma_bar, mma_phase, a.status, kTimeoutMma);
      mma_phase ^= 1;
      tc_fence_after();
      if (!__syncthreads_and(gate_ok && a0_ok && v_ok && mma_ok)) break;
    }
    // ---- P: K~^T (lane = key dim, columns c in [32 half, +32)) and R = v - e^g (k S)
    // (lanes 0-63, value dims [64 half, +64)) ----
    {
      uint32_t d[32];
      if (lrow >= C || ci == 0) {  // lanes 0-63 of later chunks: written during the previous chunk
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int c = 32 * half + e;
          d[e] = __float_as_uint(to_tf32(*reinterpret_cast<const float*>(sA0 + gdn_sw(c, lrow, 2 * C)) * ws[c]));
        }
        tmem_st32(tmem + t_lane + Sh::KT + 32 * half, d);
      }
      if (lrow < C) {
        const int c = lrow;
        const float ec = es[c];
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int j0 = 64 * half + 32 * part;
          tmem_ld32(tmem + t_lane + Sh::D1 + j0, d);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const bool hi = (hh ^ ((c >> 2) & 1)) != 0;  // half order: gdn_mn_half
              float x[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) x[k] = __uint_as_float(hi ? d[e + 4 + k] : d[e + k]);
              float4* p = reinterpret_cast<float4*>(sV + gdn_sw_mn(c, j0 + e + (hi ? 4 : 0), C));
              float4 u = *p;
              u.x = to_tf32(fmaf(-ec, x[0], u.x));
              u.y = to_tf32(fmaf(-ec, x[1], u.y));
              u.z = to_tf32(fmaf(-ec, x[2], u.z));
              u.w = to_tf32(fmaf(-ec, x[3], u.w));
              *p = u;
            }
          }
        }
      }
      tmem_wait_st();
    }
    fence_async_smem();
    tc_fence_before();
    {
      const bool tile_ok = copy_wait(tile_bar, tile_phase, tile_pending);
      if (!__syncthreads_and(tile_ok)) break;
    }
    // A0 is read (M1, K~^T): the next chunk's [k; q] tile comes in
    if (tid == 0 && ci + 1 < chunks) load_a0(ci + 1);
    // ---- MV: D_V = [T diag(beta); M] R (lanes 0-63: V_new; lanes 64-127 unused) ----
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
        for (int e = 0; e < 32; e += 8) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const bool hi = (hh ^ ((c >> 2) & 1)) != 0;  // half order: gdn_mn_half
            float x[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) x[k] = to_tf32(__uint_as_float(hi ? d[e + 4 + k] : d[e + k]));
            *reinterpret_cast<float4*>(sV + gdn_sw_mn(c, j0 + e + (hi ? 4 : 0), C)) = make_float4(x[0], x[1], x[2], x[3]);
          }
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- M3: D_V = [T diag(beta); M] V_new (lanes 64-127: M V_new);  M4: D2 = K~^T V_new ----
    if (tid == 32) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < C / 8; ++kk) {
        const uint32_t aoff = (kk >> 2) * (2 * C * 128) + (kk & 3) * 32;
        const uint64_t bdesc = smem_desc_mn128_32b(sv + kk * 1024, C * 128);
        umma_tf32(tmem + Sh::DV, smem_desc_k128(st + aoff), bdesc, IDESC_N, kk > 0 ? 1u : 0u);
        umma_tf32_ts(tmem + Sh::D2, tmem + Sh::KT + kk * 8, bdesc, IDESC_N, kk > 0 ? 1u : 0u);
      }
      umma_commit(mma_bar);
    }
    if (!mma_wait()) break;
    // every operand tile is read: the next chunk's gates and v tile come in now,
    // its record tile once the output rows (over the tile) are read
    if (tid == 0 && ci + 1 < chunks) {
      load_gates(ci + 1);
      load_v(ci + 1);
    }
    const float decay = es[C - 1];
    if (lrow >= C) {
      // ---- O1 (lanes 64-127): o = T(e^g (q S) + M V_new) into the output
      // rows, and each row half's sum of squares ----
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
          o4.x = fmaf(ec, __uint_as_float(d[e]), __uint_as_float(m[e]));
          o4.y = fmaf(ec, __uint_as_float(d[e + 1]), __uint_as_float(m[e + 1]));
          o4.z = fmaf(ec, __uint_as_float(d[e + 2]), __uint_as_float(m[e + 2]));
          o4.w = fmaf(ec, __uint_as_float(d[e + 3]), __uint_as_float(m[e + 3]));
          round2_bf16(o4.x, o4.y);
          round2_bf16(o4.z, o4.w);
          sq[0] = fmaf(o4.x, o4.x, sq[0]);
          sq[1] = fmaf(o4.y, o4.y, sq[1]);
          sq[2] = fmaf(o4.z, o4.z, sq[2]);
          sq[3] = fmaf(o4.w, o4.w, sq[3]);
          *reinterpret_cast<float4*>(ob + gdn_ob(c, j0 + e)) = o4;
        }
      }
      red[half * C + c] = (sq[0] + sq[1]) + (sq[2] + sq[3]);
    }
    // ---- S = S e^{g_last} + D2 (lane = key dim, 64 value columns per thread) ----
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      uint32_t d[32];
      const int j0 = 64 * half + 32 * part;
      tmem_ld32(tmem + t_lane + Sh::D2 + j0, d);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; e += 8) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const bool hi = (hh ^ ((lrow >> 2) & 1)) != 0;  // half order: gdn_mn_half
          float x[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) x[k] = __uint_as_float(hi ? d[e + 4 + k] : d[e + k]);
          float4* p = reinterpret_cast<float4*>(sS + gdn_sw_mn(lrow, j0 + e + (hi ? 4 : 0), DH));
          float4 s = *p;
          s.x = to_tf32(fmaf(s.x, decay, x[0]));
          s.y = to_tf32(fmaf(s.y, decay, x[1]));
          s.z = to_tf32(fmaf(s.z, decay, x[2]));
          s.w = to_tf32(fmaf(s.w, decay, x[3]));
          *p = s;
        }
      }
    }
    // ---- the next chunk's K~^T on lanes 0-63, while warps 2, 3, 6, 7 finish the
    // output rows (its A0 tile and gates have arrived by now; a failed wait
    // leaves it to the loop head's waits, which then end the walk) ----
    if (lrow < C && ci + 1 < chunks && mbar_wait(a0_bar, a0_phase, a.status, kTimeoutMma) &&
        mbar_wait(gate_bar, gate_phase, a.status, kTimeoutMma)) {
      const float* wsn = gates + ((ci + 1) & 1) * 2 * C + C;
      uint32_t d[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int c = 32 * half + e;
        d[e] = __float_as_uint(to_tf32(*reinterpret_cast<const float*>(sA0 + gdn_sw(c, lrow, 2 * C)) * wsn[c]));
      }
      tmem_st32(tmem + t_lane + Sh::KT + 32 * half, d);
      tmem_wait_st();
    }
    cp_async_wait<0>();  // this thread's z copies, read by others after the barrier
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 32 && ci + 1 < chunks && mbar_wait(a0_bar, a0_phase, a.status, kTimeoutMma))
      issue_m1();  // overlaps the gated norm below
    // ---- O2 (all threads; 16 per row, 8 columns each, so that a warp's
    // loads and stores cover two whole rows): gated RMSNorm x SiLU(z)
    // (text.py:61-67) ----
    {
      const int col = (tid & 15) * 8;
      float wn[8];  // this thread's columns of the norm weight
#pragma unroll
      for (int e = 0; e < 8; ++e) wn[e] = nws[col + e];
#pragma unroll
      for (int pass = 0; pass < C * 16 / kGdnThreads; ++pass) {
        const int c = pass * (kGdnThreads / 16) + (tid >> 4), t = t0 + c;
        if (t < a.S) {
          const float rs = rsqrtf((red[c] + red[C + c]) / DH + a.eps);
          GdnVec<T> z, res;
          z.load(zs + c * Sh::ZLD + col);
          const float4 o0 = *reinterpret_cast<const float4*>(ob + gdn_ob(c, col));
          const float4 o1 = *reinterpret_cast<const float4*>(ob + gdn_ob(c, col + 4));
          float n[8] = {o0.x * rs, o0.y * rs, o0.z * rs, o0.w * rs, o1.x * rs, o1.y * rs, o1.z * rs, o1.w * rs};
#pragma unroll
          for (int e = 0; e < 8; e += 2) round2_bf16(n[e], n[e + 1]);
#pragma unroll
          for (int e = 0; e < 8; ++e) n[e] *= wn[e];
#pragma unroll
          for (int e = 0; e < 8; e += 2) round2_bf16(n[e], n[e + 1]);
#pragma unroll
          for (int e = 0; e < 8; ++e) res.v[e] = n[e] * (z.v[e] * sigmoid_fast(z.v[e]));
          res.store(out + (row0 + t) * a.ldo + h * DH + col);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0 && ci + 1 < chunks) load_tile(ci + 1);
  }

  // copies that a failed wait left in flight land before the CTA's shared
  // memory is released (bounded: the status is already set)
  if (tid == 0 && tile_pending) mbar_wait(tile_bar, tile_phase, a.status, kTimeoutMma);
  if (tid == 0 && gate_pending) mbar_wait(gate_bar, gate_phase, a.status, kTimeoutMma);
  if (tid == 0 && a0_pending) mbar_wait(a0_bar, a0_phase, a.status, kTimeoutMma);
  if (tid == 0 && v_pending) mbar_wait(v_bar, v_phase, a.status, kTimeoutMma);
  cp_async_wait<0>();  // and this thread's z copies
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, Sh::TMEM_COLS);
}

}  // namespace clef

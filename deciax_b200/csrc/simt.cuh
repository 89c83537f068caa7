// CUDA-core kernels: the generic GEMM (fp32 mode and the joint head's
// small-M projections), row norms, embedding gather, q/k-norm + partial RoPE
// and elementwise epilogues.  Templated on the activation type T (float or
// __nv_bfloat16); all arithmetic is fp32 with T rounding at the reference's
// cast points.
#pragma once

#include "common.cuh"

namespace clef {

// ---------------------------------------------------------------------------
// generic GEMM: C[M,N] = A[M,K] * B[N,K]^T, fp32 accumulate
// ---------------------------------------------------------------------------

enum SimtEpi : int {
  kSimtStore = 0,     // out = T(acc + bias)
  kSimtGelu = 1,      // out = T(gelu(T(acc + bias)))   dense() followed by exact GELU
  kSimtResidual = 2,  // out = T(res + T(acc))
  kSimtF32 = 3,       // out(float) = acc
};

template <typename T>
struct SimtGemmArgs {
  const T* A;
  int lda;
  const T* B;
  int ldb;
  int M, N, K;
  const T* bias;
  const T* residual;
  int ldr;
  void* out;
  int ldo;
};

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

template <typename T, int EPI>
__global__ void __launch_bounds__(256) simt_gemm(SimtGemmArgs<T> a) {
  constexpr int BM = 64, BN = 64, BK = 16;
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < a.K; k0 += BK) {
    for (int i = threadIdx.x; i < BM * BK; i += 256) {
      const int r = i / BK, c = i % BK;
      const int gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < a.M && gk < a.K) ? to_f32(a.A[static_cast<size_t>(gm) * a.lda + gk]) : 0.f;
      const int gn = n0 + r;
      Bs[c][r] = (gn < a.N && gk < a.K) ? to_f32(a.B[static_cast<size_t>(gn) * a.ldb + gk]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float av[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= a.N) continue;
      float v = acc[i][j];
      if constexpr (EPI == kSimtF32) {
        static_cast<float*>(a.out)[static_cast<size_t>(gm) * a.ldo + gn] = v;
      } else {
        if constexpr (EPI == kSimtStore || EPI == kSimtGelu) {
          if (a.bias) v += to_f32(a.bias[gn]);
          if constexpr (EPI == kSimtGelu) v = gelu_erf(round_to<T>(v));
        } else {
          v = to_f32(a.residual[static_cast<size_t>(gm) * a.ldr + gn]) + round_to<T>(v);
        }
        static_cast<T*>(a.out)[static_cast<size_t>(gm) * a.ldo + gn] = from_f32<T>(v);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// row norms (one warp per row)
// ---------------------------------------------------------------------------

// RMSNorm scaling by (1 + w): qwen3_5/text.py:25-28.  With row_mask, rows
// whose mask byte is 0 are written as zeros (the Gated DeltaNet input
// x * mask of text.py:43).
template <typename T>
__global__ void rmsnorm_kernel(const T* __restrict__ x, int ldx, const T* __restrict__ w, T* __restrict__ out, int ldo,
                               int rows, int dim, float eps, const uint8_t* __restrict__ row_mask) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + static_cast<size_t>(row) * ldx;
  T* orow = out + static_cast<size_t>(row) * ldo;
  if (row_mask != nullptr && row_mask[row] == 0) {
    for (int i = lane; i < dim; i += 32) orow[i] = from_f32<T>(0.f);
    return;
  }
  float ss = 0.f;
  if constexpr (sizeof(T) == 2) {
    if ((dim & 7) == 0) {
      for (int i = lane * 8; i < dim; i += 256) {
        const uint4 q = *reinterpret_cast<const uint4*>(xr + i);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float v = __bfloat162float(h[j]);
          ss += v * v;
        }
      }
      const float r = rsqrtf(warp_sum(ss) / dim + eps);
      for (int i = lane * 8; i < dim; i += 256) {
        const uint4 q = *reinterpret_cast<const uint4*>(xr + i);
        const uint4 wq = *reinterpret_cast<const uint4*>(w + i);
        const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
        const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wq);
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = pack_bf16x2(__bfloat162float(h[2 * j]) * r * (__bfloat162float(wh[2 * j]) + 1.f),
                             __bfloat162float(h[2 * j + 1]) * r * (__bfloat162float(wh[2 * j + 1]) + 1.f));
        *reinterpret_cast<uint4*>(orow + i) = make_uint4(o[0], o[1], o[2], o[3]);
      }
      return;
    }
  }
  for (int i = lane; i < dim; i += 32) {
    const float v = to_f32(xr[i]);
    ss += v * v;
  }
  const float r = rsqrtf(warp_sum(ss) / dim + eps);
  for (int i = lane; i < dim; i += 32) orow[i] = from_f32<T>(to_f32(xr[i]) * r * (to_f32(w[i]) + 1.f));
}

// The same RMSNorm for bf16 rows of at most kRmsSmemMaxDim elements (dim and
// ldx multiples of 8): each warp stages its row in shared memory with 16-byte
// cp.async copies all in flight, then reads it twice from there, so DRAM sees
// one read of x.  4 rows (warps) per block.
constexpr int kRmsSmemMaxDim = 8192;
constexpr int kRmsSmemRows = 4;
__global__ void __launch_bounds__(32 * kRmsSmemRows)
    rmsnorm_bf16_smem_kernel(const __nv_bfloat16* __restrict__ x, int ldx, const __nv_bfloat16* __restrict__ w,
                             __nv_bfloat16* __restrict__ out, int ldo, int rows, int dim, float eps,
                             const uint8_t* __restrict__ row_mask) {
  extern __shared__ uint4 rms_stage[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRmsSmemRows + warp;
  if (row >= rows) return;
  const int nvec = dim / 8;
  uint4* buf = rms_stage + static_cast<size_t>(warp) * nvec;
  __nv_bfloat16* orow = out + static_cast<size_t>(row) * ldo;
  if (row_mask != nullptr && row_mask[row] == 0) {
    for (int v = lane; v < nvec; v += 32) reinterpret_cast<uint4*>(orow)[v] = make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * ldx);
  for (int v = lane; v < nvec; v += 32) cp_async16(buf + v, xr + v, true);
  cp_async_commit();
  cp_async_wait<0>();
  __syncwarp();
  float ss = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    const uint4 q = buf[v];
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float f = __bfloat162float(h[j]);
      ss += f * f;
    }
  }
  const float r = rsqrtf(warp_sum(ss) / dim + eps);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  for (int v = lane; v < nvec; v += 32) {
    const uint4 q = buf[v];
    const uint4 wq = wv[v];
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wq);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      o[j] = pack_bf16x2(__bfloat162float(h[2 * j]) * r * (__bfloat162float(wh[2 * j]) + 1.f),
                         __bfloat162float(h[2 * j + 1]) * r * (__bfloat162float(wh[2 * j + 1]) + 1.f));
    reinterpret_cast<uint4*>(orow)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// LayerNorm with weight and bias, eps 1e-5 (nn.py:22-28, head.py:16-17).
template <typename T>
__global__ void layernorm_kernel(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
                                 T* __restrict__ out, int rows, int dim, float eps) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + static_cast<size_t>(row) * dim;
  float s = 0.f;
  for (int i = lane; i < dim; i += 32) s += to_f32(xr[i]);
  const float mean = warp_sum(s) / dim;
  float ss = 0.f;
  for (int i = lane; i < dim; i += 32) {
    const float z = to_f32(xr[i]) - mean;
    ss += z * z;
  }
  const float r = rsqrtf(warp_sum(ss) / dim + eps);
  T* orow = out + static_cast<size_t>(row) * dim;
  for (int i = lane; i < dim; i += 32) orow[i] = from_f32<T>((to_f32(xr[i]) - mean) * r * to_f32(w[i]) + to_f32(b[i]));
}

// ---------------------------------------------------------------------------
// embedding gather (models/clef/model.py:67,95), one warp per token
// ---------------------------------------------------------------------------

template <typename T>
__global__ void embed_kernel(const int32_t* __restrict__ ids, const T* __restrict__ table, T* __restrict__ out,
                             int tokens, int dim, int vocab, float scale, int* status) {
  const int t = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  int id = ids[t];
  if (id < 0 || id >= vocab) {
    if (lane == 0) record_status(status, kBadIndex);
    id = 0;
  }
  const T* src = table + static_cast<size_t>(id) * dim;
  T* dst = out + static_cast<size_t>(t) * dim;
  if (scale == 0.f && (dim * sizeof(T)) % 16 == 0) {
    const int nv = dim * sizeof(T) / 16;
    for (int i = lane; i < nv; i += 32) reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (int i = lane; i < dim; i += 32) {
      const float v = to_f32(src[i]);
      dst[i] = from_f32<T>(scale == 0.f ? v : v * round_to<T>(scale));
    }
  }
}

// ---------------------------------------------------------------------------
// per-head q/k RMSNorm + partial rotate-half RoPE, in place (text.py:79-88, nn.py:35-44)
// ---------------------------------------------------------------------------
// Row layout of the packed projection: [Hq x (q d | gate d)] [Hkv x k d] [Hkv x v d].
// One warp per (token, head); heads [0, hq) are q heads, [hq, hq+hkv) k heads.
// cos/sin tables are [S, rot/2] float; they are rounded to T before use.
template <typename T>
__global__ void qk_norm_rope_kernel(T* __restrict__ qkv, int ld, int tokens, int seq, int hq, int hkv, int d, int rot,
                                    const T* __restrict__ qw, const T* __restrict__ kw, const float* __restrict__ cos_t,
                                    const float* __restrict__ sin_t, float eps) {
  extern __shared__ float rowbuf[];  // (blockDim/32) * d floats
  const int wib = threadIdx.x / 32, lane = threadIdx.x & 31;
  const long long item = static_cast<long long>(blockIdx.x) * (blockDim.x / 32) + wib;
  const int heads = hq + hkv;
  if (item >= static_cast<long long>(tokens) * heads) return;
  const int t = static_cast<int>(item / heads), h = static_cast<int>(item % heads);
  const int pos = t % seq;
  T* x = qkv + static_cast<size_t>(t) * ld + (h < hq ? h * 2 * d : hq * 2 * d + (h - hq) * d);
  const T* w = h < hq ? qw : kw;
  float* buf = rowbuf + wib * d;
  float ss = 0.f;
  for (int i = lane; i < d; i += 32) {
    const float v = to_f32(x[i]);
    buf[i] = v;
    ss += v * v;
  }
  const float r = rsqrtf(warp_sum(ss) / d + eps);
  for (int i = lane; i < d; i += 32) buf[i] = round_to<T>(buf[i] * r * (to_f32(w[i]) + 1.f));
  __syncwarp();
  const int half = rot / 2;
  for (int i = lane; i < d; i += 32) {
    float v = buf[i];
    if (i < rot) {
      const int f = i < half ? i : i - half;
      const float c = round_to<T>(cos_t[static_cast<size_t>(pos) * half + f]);
      const float s = round_to<T>(sin_t[static_cast<size_t>(pos) * half + f]);
      const float other = i < half ? -buf[i + half] : buf[i - half];
      v = round_to<T>(v * c) + round_to<T>(other * s);
    }
    x[i] = from_f32<T>(v);
  }
}

// ---------------------------------------------------------------------------
// elementwise
// ---------------------------------------------------------------------------

// x = T(x + T(y)): residual add after a reduced fp32 projection (text.py:98,102).
template <typename T>
__global__ void residual_add_f32_kernel(T* __restrict__ x, const float* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    x[i] = from_f32<T>(to_f32(x[i]) + round_to<T>(y[i]));
}

// act[m, j] = T(T(silu(g)) * u) from a packed [M, 2F] gate/up product whose
// 256-column blocks are [128 gate | 128 up] (text.py:101).
template <typename T>
__global__ void swiglu_packed_kernel(const T* __restrict__ gu, T* __restrict__ act, int rows, int f) {
  const long long n = static_cast<long long>(rows) * f;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / f;
    const int j = static_cast<int>(i % f);
    const long long base = r * 2 * f + (j / 128) * 256 + (j % 128);
    const float g = to_f32(gu[base]), u = to_f32(gu[base + 128]);
    act[i] = from_f32<T>(round_to<T>(g / (1.f + expf(-g))) * u);
  }
}

}  // namespace clef

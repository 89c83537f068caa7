// Gated DeltaNet mixer core: qwen3_5/text.py:31-67 and kernels/gdn/reference.py:14-92.
//
// One CTA per (state, value head) walks the sequence in 64-token chunks with
// the head's FP32 state S [dk, dv] resident in shared memory.  Per chunk it
//   1. reads the projection rows straight from the GEMM output and applies the
//      depthwise causal convolution + SiLU (text.py:31-39) to this head's q, k
//      and v channels (q and k of key head h / (nv / nh): jnp.repeat order),
//      L2-normalises q and k (eps 1e-6, rounded to the activation dtype, q
//      then scaled by dk^-1/2), and forms g = -exp(A_log) softplus(a + dt_bias)
//      and beta = sigmoid(b) (text.py:57-58);
//   2. runs the chunked delta rule (reference.py:54-89): cumulative g, the
//      strictly lower system A = -(k beta k^T) * decay, an exact forward
//      substitution (I - A) X = [v beta | k beta e^g] (one column per thread,
//      the column held in registers), value = X_v - X_k S,
//      out = (q e^g) S + (q k^T * decay) value, S = S e^{g_last} + (k e^{g_last-g})^T value;
//   3. applies the gated RMSNorm and SiLU(z) gate (text.py:61-67) to the
//      chunk's output rows and writes them in the activation dtype.
// All arithmetic after the casts is FP32 on CUDA cores (the reference uses
// Precision.HIGHEST); exp, sigmoid and rsqrt use the hardware approximations
// (a few fp32 ulps).  Rows past the sequence end are zero with g = beta = 0,
// as the reference's padding.  No waits on other CTAs.
#pragma once

#include "common.cuh"

namespace clef {

struct GdnArgs {
  const void* proj;  // [B*S, ldp] activation dtype: q | k | v | z | a | b column groups (q at column 0)
  long long ldp;
  int k_col, v_col, z_col, a_col, b_col;
  const void* conv;  // [v_col + nv*dh, width]: one row per q/k/v channel, in projection column order
  int width;
  const void* A_log;    // [nv]
  const void* dt_bias;  // [nv]
  const void* norm_w;   // [dh]
  void* out;            // [B*S, ldo]: head h at columns h*dh
  long long ldo;
  int B, S, nh, nv;
  float qscale;  // dk^-1/2 as a float32
  float eps;     // rms_norm_eps of the gated norm
  int* status;   // device status word for a bounded wait that gives up (tensor-core kernel); may be null
  // tensor-core path only: the conv pass's bf16 rows [B*S, ldc] (q heads, k heads, v heads)
  void* qkv_conv;
  long long ldc;
  // tensor-core path only: the prep pass's per-(chunk, value head, state) records
  void* prep;
  // tensor-core path only: the conv pass's operand tiles for the chain pass, per
  // (state, key head, chunk) [k; q dk^-1/2] and per (state, value head, chunk) v
  void* a0_tiles;
  void* v_tiles;
};

constexpr int kGdnChunk = 64;
constexpr int kGdnThreads = 256;

template <int DH>
struct GdnShape {
  static constexpr int C = kGdnChunk;
  static constexpr int LDQ = DH + 4;  // q (later the output rows), k and the solved key rows: 16-byte rows
  static constexpr int LDA = C + 4;
  static constexpr int TCOL = DH < 16 ? DH : 16;  // threads across output columns
  static constexpr int TROW = kGdnThreads / TCOL;
  static constexpr int NC = DH / TCOL;                           // columns per thread
  static constexpr int RM = C / TROW;                            // rows per thread, 64-row outputs
  static constexpr int RS = DH / TROW > 0 ? DH / TROW : 1;       // rows per thread, DH-row state
  static constexpr size_t floats = size_t(DH) * DH + 3 * C * LDQ + C * DH + C * LDA + 4 * C + 3 * DH * 4;
  static constexpr size_t bytes = floats * 4;
};

// e^x through the hardware ex2 (a few fp32 ulps; the parity bars are 1e-4
// relative in FP32 and one bf16 step in BF16).
__device__ __forceinline__ float exp_fast(float x) { return ex2_approx(1.4426950408889634f * x); }

__device__ __forceinline__ float softplus_f(float x) {  // logaddexp(0, x)
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

// 16-byte vectors of the activation dtype (8 bf16 or 4 float) as floats.
template <typename T>
struct GdnVec {
  static constexpr int N = 16 / static_cast<int>(sizeof(T));
  float v[N];
  __device__ __forceinline__ void load(const T* p) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    if constexpr (sizeof(T) == 2) {
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = __bfloat162float(h[i]);
    } else {
      const float* f = reinterpret_cast<const float*>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) v[i] = f[i];
    }
  }
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = 0.f;
  }
  __device__ __forceinline__ void store(T* p) const {
    uint4 raw;
    if constexpr (sizeof(T) == 2) {
      uint32_t* w = reinterpret_cast<uint32_t*>(&raw);
#pragma unroll
      for (int i = 0; i < N / 2; ++i) w[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    } else {
      float* f = reinterpret_cast<float*>(&raw);
#pragma unroll
      for (int i = 0; i < N; ++i) f[i] = v[i];
    }
    *reinterpret_cast<uint4*>(p) = raw;
  }
};

// Sum over aligned groups of G lanes (G a power of two <= 32).
template <int G>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = G / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Stage 1 of a chunk: conv + SiLU (text.py:31-39) of this head's q, k and v
// channels for rows t0..t0+63, L2 norms of q and k (reference.py:14-21: eps
// 1e-6, cast, q then x dk^-1/2), into shared memory.  GL threads cover one
// row of a vector in 16-byte pieces; each thread convolves RT consecutive
// rows from a sliding window of RT + W - 1 loaded rows, all loads in flight
// before the arithmetic.  The taps are right-aligned in W slots (zero weights
// first), so each output is 0 + x_0 w_0 + ... in the reference's order.
template <typename T, int DH, int W>
__device__ __forceinline__ void gdn_load_chunk(const GdnArgs& a, const T* proj, const T* convw, const float* wsm,
                                               long long row0, int t0, int q_col, int k_col, int v_col, float* Qs,
                                               float* Ks, float* Vs) {
  constexpr int C = kGdnChunk, LDQ = GdnShape<DH>::LDQ, VN = GdnVec<T>::N, GL = DH / VN, RPP = kGdnThreads / GL;
  constexpr int RT = C / RPP > 0 ? C / RPP : 1, NX = RT + W - 1;
  const int tid = threadIdx.x, g = tid % GL, r0 = (tid / GL) * RT;
  const int shift = W - a.width;
  if (r0 >= C) return;  // warp-uniform: RT * (32 / GL) divides 64
  // conv width <= 4: every tap row of q, k and v in flight before any
  // arithmetic; wider convs load one kind at a time (register budget)
  constexpr int NK = W <= 4 ? 3 : 1;
  uint4 raw[NK][NX];
  auto load_kind = [&](int kind, uint4 (&dst)[NX]) {
    const int col = (kind == 0 ? q_col : kind == 1 ? k_col : v_col) + g * VN;
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      const int tt = t0 + r0 - (W - 1) + i;
      dst[i] = (tt >= 0 && tt < a.S) ? *reinterpret_cast<const uint4*>(proj + (row0 + tt) * a.ldp + col)
                                     : make_uint4(0u, 0u, 0u, 0u);
    }
  };
  if constexpr (NK == 3) {
#pragma unroll
    for (int kind = 0; kind < 3; ++kind) load_kind(kind, raw[kind]);
  }
#pragma unroll
  for (int kind = 0; kind < 3; ++kind) {
    const int col = (kind == 0 ? q_col : kind == 1 ? k_col : v_col) + g * VN;
    if constexpr (NK == 1) load_kind(kind, raw[0]);
    const uint4 (&rk)[NX] = raw[NK == 3 ? kind : 0];
    float w[VN][W];
#pragma unroll
    for (int c = 0; c < VN; ++c)
#pragma unroll
      for (int i = 0; i < W; ++i)
        w[c][i] = wsm ? wsm[(kind * DH + g * VN + c) * W + i]
                      : (i >= shift ? to_f32(convw[static_cast<long long>(col + c) * a.width + (i - shift)]) : 0.f);
    GdnVec<T> x[NX];
#pragma unroll
    for (int i = 0; i < NX; ++i) {
      if constexpr (sizeof(T) == 2) {
        const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&rk[i]);
#pragma unroll
        for (int c = 0; c < VN; ++c) x[i].v[c] = __bfloat162float(hv[c]);
      } else {
        const float* fv = reinterpret_cast<const float*>(&rk[i]);
#pragma unroll
        for (int c = 0; c < VN; ++c) x[i].v[c] = fv[c];
      }
    }
    float* dst = kind == 0 ? Qs : kind == 1 ? Ks : Vs;
    const int ld = kind == 2 ? DH : LDQ;
#pragma unroll
    for (int j = 0; j < RT; ++j) {
      const int r = r0 + j;
      GdnVec<T> y;
#pragma unroll
      for (int c = 0; c < VN; ++c) {
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < W; ++i) acc = __fadd_rn(acc, __fmul_rn(x[j + i].v[c], w[c][i]));
        const float z = round_to<T>(acc);
        y.v[c] = t0 + r < a.S ? round_to<T>(z * sigmoid_fast(z)) : 0.f;
      }
      if (kind < 2) {
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < VN; ++c) ss += y.v[c] * y.v[c];
        const float inv = rsqrtf(group_sum<GL>(ss) + 1e-6f);
        const float scale = kind == 0 ? a.qscale : 1.f;
#pragma unroll
        for (int c = 0; c < VN; ++c) y.v[c] = round_to<T>(y.v[c] * inv) * scale;
      }
#pragma unroll
      for (int c = 0; c < VN; c += 4)
        *reinterpret_cast<float4*>(dst + r * ld + g * VN + c) = make_float4(y.v[c], y.v[c + 1], y.v[c + 2], y.v[c + 3]);
    }
  }
}

// acc[m][n] = sum_d X[i_m][d] * Y[j_n][d] over 64x64 pairs, i_m = ti + 16m,
// j_n = tj + 16n; rows 16-byte aligned, d in order, 4 at a time.
template <int LD>
__device__ __forceinline__ void gdn_gram(float (&acc)[4][4], const float* X, const float* Y, int kd, int ti, int tj) {
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[m][n] = 0.f;
  for (int d = 0; d < kd; d += 4) {
    float4 x[4], y[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) x[m] = *reinterpret_cast<const float4*>(X + (ti + 16 * m) * LD + d);
#pragma unroll
    for (int n = 0; n < 4; ++n) y[n] = *reinterpret_cast<const float4*>(Y + (tj + 16 * n) * LD + d);
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        float v = acc[m][n];
        v = fmaf(x[m].x, y[n].x, v);
        v = fmaf(x[m].y, y[n].y, v);
        v = fmaf(x[m].z, y[n].z, v);
        acc[m][n] = fmaf(x[m].w, y[n].w, v);
      }
  }
}

__device__ __forceinline__ float f4_at(const float4& v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }

// acc[m][n][q] = sum_{d<kd} L[(tr + 16 m) * ldl + d] * R[d * ldr + 4 tc + 64 n + q]
// (kd a multiple of 4, rows 16-byte aligned): 16 threads across 4-column
// groups, d in order.
template <int RM, int NV>
__device__ __forceinline__ void gdn_mm4(float (&acc)[RM][NV][4], const float* L, int ldl, const float* R, int ldr,
                                        int kd, int tr, int tc) {
#pragma unroll
  for (int m = 0; m < RM; ++m)
#pragma unroll
    for (int n = 0; n < NV; ++n)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[m][n][q] = 0.f;
  for (int d = 0; d < kd; d += 4) {
    float4 l[RM];
#pragma unroll
    for (int m = 0; m < RM; ++m) l[m] = *reinterpret_cast<const float4*>(L + (tr + 16 * m) * ldl + d);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float4 r[NV];
#pragma unroll
      for (int n = 0; n < NV; ++n) r[n] = *reinterpret_cast<const float4*>(R + (d + e) * ldr + 4 * tc + 64 * n);
#pragma unroll
      for (int m = 0; m < RM; ++m) {
        const float lv = f4_at(l[m], e);
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          acc[m][n][0] = fmaf(lv, r[n].x, acc[m][n][0]);
          acc[m][n][1] = fmaf(lv, r[n].y, acc[m][n][1]);
          acc[m][n][2] = fmaf(lv, r[n].z, acc[m][n][2]);
          acc[m][n][3] = fmaf(lv, r[n].w, acc[m][n][3]);
        }
      }
    }
  }
}

// acc[m][n] = sum_{d<kd} L[(tr + TROW m) * ldl + d] * R[d * ldr + tc + TCOL n]
template <int RM, int NC, int TROW, int TCOL>
__device__ __forceinline__ void gdn_mm(float (&acc)[RM][NC], const float* L, int ldl, const float* R, int ldr, int kd,
                                       int tr, int tc) {
#pragma unroll
  for (int m = 0; m < RM; ++m)
#pragma unroll
    for (int n = 0; n < NC; ++n) acc[m][n] = 0.f;
  for (int d = 0; d < kd; ++d) {
    float l[RM], r[NC];
#pragma unroll
    for (int m = 0; m < RM; ++m) l[m] = L[(tr + TROW * m) * ldl + d];
#pragma unroll
    for (int n = 0; n < NC; ++n) r[n] = R[d * ldr + tc + TCOL * n];
#pragma unroll
    for (int m = 0; m < RM; ++m)
#pragma unroll
      for (int n = 0; n < NC; ++n) acc[m][n] = fmaf(l[m], r[n], acc[m][n]);
  }
}

template <typename T, int DH>
__global__ void __launch_bounds__(kGdnThreads, 1) gdn_chunk_kernel(GdnArgs a) {
  using G = GdnShape<DH>;
  constexpr int C = G::C, LDQ = G::LDQ, LDA = G::LDA, TCOL = G::TCOL, TROW = G::TROW, NC = G::NC, RM = G::RM,
                RS = G::RS, NV = DH >= 64 ? DH / 64 : 1;
  extern __shared__ float smem_f[];
  float* St = smem_f;        // [DH][DH] state
  float* Qs = St + DH * DH;  // [C][LDQ] scaled q, then the chunk's output rows
  float* Ks = Qs + C * LDQ;  // [C][LDQ] normalised k
  float* Cs = Ks + C * LDQ;  // [C][LDQ] k beta e^g, solved in place
  float* Vs = Cs + C * LDQ;  // [C][DH] v beta, solved in place, then value
  float* As = Vs + C * DH;   // [C][LDA] system matrix, then q k^T * decay
  float* gs = As + C * LDA;  // cumulative g
  float* bs = gs + C;        // beta
  float* es = bs + C;        // e^g
  float* ws = es + C;        // e^(g_last - g)
  float* wconv = ws + C;     // [3][DH][4] this head's q / k / v conv taps, right-aligned (width <= 4)

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = h / (a.nv / a.nh);
  const T* proj = static_cast<const T*>(a.proj);
  const T* convw = static_cast<const T*>(a.conv);
  const T* nw = static_cast<const T*>(a.norm_w);
  T* out = static_cast<T*>(a.out);
  const float neg_a = -expf(to_f32(static_cast<const T*>(a.A_log)[h]));
  const float dt_bias = to_f32(static_cast<const T*>(a.dt_bias)[h]);
  const long long row0 = static_cast<long long>(b) * a.S;
  const int q_col = hk * DH, k_col = a.k_col + hk * DH, v_col = a.v_col + h * DH;
  const int ti = tid >> 4, tj = tid & 15;            // 64x64 products
  const int tr = tid / TCOL, tc = tid % TCOL;        // 64xDH and DHxDH products

  for (int i = tid; i < DH * DH; i += kGdnThreads) St[i] = 0.f;
  if (a.width <= 4) {
    const int shift = 4 - a.width;
    for (int i = tid; i < 3 * DH * 4; i += kGdnThreads) {
      const int kind = i / (DH * 4), c = (i / 4) % DH, tap = i % 4;
      const int col = (kind == 0 ? q_col : kind == 1 ? k_col : v_col) + c;
      wconv[i] = tap >= shift ? to_f32(convw[static_cast<long long>(col) * a.width + (tap - shift)]) : 0.f;
    }
  }
  __syncthreads();
  GdnVec<T> nwv;  // this thread's slice of the gated norm's weight
  nwv.load(nw + (tid % (DH / GdnVec<T>::N)) * GdnVec<T>::N);

  const int chunks = (a.S + C - 1) / C;
  for (int ci = 0; ci < chunks; ++ci) {
    const int t0 = ci * C;
    // 1. conv + SiLU, L2 norms, gates
    {
      if (a.width <= 4)
        gdn_load_chunk<T, DH, 4>(a, proj, convw, wconv, row0, t0, q_col, k_col, v_col, Qs, Ks, Vs);
      else
        gdn_load_chunk<T, DH, 8>(a, proj, convw, nullptr, row0, t0, q_col, k_col, v_col, Qs, Ks, Vs);
      if (tid < C) {
        const int t = t0 + tid;
        if (t < a.S) {
          const T* pr = proj + (row0 + t) * a.ldp;
          gs[tid] = neg_a * softplus_f(to_f32(pr[a.a_col + h]) + dt_bias);
          bs[tid] = round_to<T>(sigmoid_fast(to_f32(pr[a.b_col + h])));
        } else {
          gs[tid] = 0.f;
          bs[tid] = 0.f;
        }
      }
    }
    __syncthreads();
    // 2. cumulative gate (sequential, as cumsum) and its exponentials
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
    __syncthreads();
    // 3. right-hand sides and the strictly lower system matrix
    for (int i = tid; i < C * DH; i += kGdnThreads) {
      const int r = i / DH, c = i % DH;
      Cs[r * LDQ + c] = Ks[r * LDQ + c] * bs[r] * es[r];
      Vs[r * DH + c] *= bs[r];
    }
    {
      float acc[4][4];
      gdn_gram<LDQ>(acc, Ks, Ks, DH, ti, tj);
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int i = ti + 16 * m, j = tj + 16 * n;
          As[i * LDA + j] = j < i ? -(acc[m][n] * bs[i]) * exp_fast(gs[i] - gs[j]) : 0.f;
        }
    }
    __syncthreads();
    // 4. forward substitution, one right-hand-side column per thread
    if (tid < 2 * DH) {
      float* col = tid < DH ? Vs + tid : Cs + (tid - DH);
      const int ld = tid < DH ? DH : LDQ;
      float x[C];
#pragma unroll
      for (int r = 0; r < C; ++r) {
        float acc = col[r * ld];
#pragma unroll
        for (int j4 = 0; j4 + 4 <= r; j4 += 4) {
          const float4 a4 = *reinterpret_cast<const float4*>(As + r * LDA + j4);
          acc = fmaf(a4.x, x[j4], acc);
          acc = fmaf(a4.y, x[j4 + 1], acc);
          acc = fmaf(a4.z, x[j4 + 2], acc);
          acc = fmaf(a4.w, x[j4 + 3], acc);
        }
#pragma unroll
        for (int j = r & ~3; j < r; ++j) acc = fmaf(As[r * LDA + j], x[j], acc);
        x[r] = acc;
        col[r * ld] = acc;
      }
    }
    __syncthreads();
    // 5. value = X_v - X_k S; q k^T * decay (j <= i) into As
    if constexpr (DH >= 64) {
      float acc[4][NV][4];
      gdn_mm4<4, NV>(acc, Cs, LDQ, St, DH, DH, tr, tc);
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          float4* p = reinterpret_cast<float4*>(Vs + (tr + 16 * m) * DH + 4 * tc + 64 * n);
          float4 v = *p;
          v.x -= acc[m][n][0];
          v.y -= acc[m][n][1];
          v.z -= acc[m][n][2];
          v.w -= acc[m][n][3];
          *p = v;
        }
    } else {
      float acc[RM][NC];
      gdn_mm<RM, NC, TROW, TCOL>(acc, Cs, LDQ, St, DH, DH, tr, tc);
#pragma unroll
      for (int m = 0; m < RM; ++m)
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          const int i = tr + TROW * m, c = tc + TCOL * n;
          Vs[i * DH + c] -= acc[m][n];
        }
    }
    {
      float acc[4][4];
      gdn_gram<LDQ>(acc, Qs, Ks, DH, ti, tj);
#pragma unroll
      for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          const int i = ti + 16 * m, j = tj + 16 * n;
          As[i * LDA + j] = j <= i ? acc[m][n] * exp_fast(gs[i] - gs[j]) : 0.f;
        }
    }
    __syncthreads();
    // 6. out = (q e^g) S + (q k^T * decay) value -> the rows of Qs
    if constexpr (DH >= 64) {
      float acc[4][NV][4], acc2[4][NV][4];
      gdn_mm4<4, NV>(acc, Qs, LDQ, St, DH, DH, tr, tc);
      gdn_mm4<4, NV>(acc2, As, LDA, Vs, DH, C, tr, tc);
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int i = tr + 16 * m;
        const float e = es[i];
#pragma unroll
        for (int n = 0; n < NV; ++n)
          *reinterpret_cast<float4*>(Qs + i * LDQ + 4 * tc + 64 * n) =
              make_float4(acc[m][n][0] * e + acc2[m][n][0], acc[m][n][1] * e + acc2[m][n][1],
                          acc[m][n][2] * e + acc2[m][n][2], acc[m][n][3] * e + acc2[m][n][3]);
      }
    } else {
      float acc[RM][NC], acc2[RM][NC];
      gdn_mm<RM, NC, TROW, TCOL>(acc, Qs, LDQ, St, DH, DH, tr, tc);
      gdn_mm<RM, NC, TROW, TCOL>(acc2, As, LDA, Vs, DH, C, tr, tc);
      __syncthreads();
#pragma unroll
      for (int m = 0; m < RM; ++m)
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          const int i = tr + TROW * m, c = tc + TCOL * n;
          Qs[i * LDQ + c] = acc[m][n] * es[i] + acc2[m][n];
        }
    }
    __syncthreads();
    // 7a. S = S e^{g_last} + (k e^{g_last - g})^T value
    if constexpr (DH >= 64) {
      constexpr int RSV = DH / 16;
      float acc[RSV][NV][4];
#pragma unroll
      for (int m = 0; m < RSV; ++m)
#pragma unroll
        for (int n = 0; n < NV; ++n)
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[m][n][q] = 0.f;
      for (int r = 0; r < C; ++r) {
        const float wr = ws[r];
        float l[RSV];
        float4 v[NV];
#pragma unroll
        for (int m = 0; m < RSV; ++m) l[m] = Ks[r * LDQ + tr + 16 * m] * wr;
#pragma unroll
        for (int n = 0; n < NV; ++n) v[n] = *reinterpret_cast<const float4*>(Vs + r * DH + 4 * tc + 64 * n);
#pragma unroll
        for (int m = 0; m < RSV; ++m)
#pragma unroll
          for (int n = 0; n < NV; ++n) {
            acc[m][n][0] = fmaf(l[m], v[n].x, acc[m][n][0]);
            acc[m][n][1] = fmaf(l[m], v[n].y, acc[m][n][1]);
            acc[m][n][2] = fmaf(l[m], v[n].z, acc[m][n][2]);
            acc[m][n][3] = fmaf(l[m], v[n].w, acc[m][n][3]);
          }
      }
      const float decay = es[C - 1];
#pragma unroll
      for (int m = 0; m < RSV; ++m)
#pragma unroll
        for (int n = 0; n < NV; ++n) {
          float4* p = reinterpret_cast<float4*>(St + (tr + 16 * m) * DH + 4 * tc + 64 * n);
          float4 sv = *p;
          sv.x = sv.x * decay + acc[m][n][0];
          sv.y = sv.y * decay + acc[m][n][1];
          sv.z = sv.z * decay + acc[m][n][2];
          sv.w = sv.w * decay + acc[m][n][3];
          *p = sv;
        }
    } else if (tr < DH) {
      float acc[RS][NC];
#pragma unroll
      for (int m = 0; m < RS; ++m)
#pragma unroll
        for (int n = 0; n < NC; ++n) acc[m][n] = 0.f;
      for (int r = 0; r < C; ++r) {
        float l[RS], v[NC];
        const float wr = ws[r];
#pragma unroll
        for (int m = 0; m < RS; ++m) l[m] = Ks[r * LDQ + tr + TROW * m] * wr;
#pragma unroll
        for (int n = 0; n < NC; ++n) v[n] = Vs[r * DH + tc + TCOL * n];
#pragma unroll
        for (int m = 0; m < RS; ++m)
#pragma unroll
          for (int n = 0; n < NC; ++n) acc[m][n] = fmaf(l[m], v[n], acc[m][n]);
      }
      const float decay = es[C - 1];
#pragma unroll
      for (int m = 0; m < RS; ++m)
#pragma unroll
        for (int n = 0; n < NC; ++n) {
          float& s = St[(tr + TROW * m) * DH + tc + TCOL * n];
          s = s * decay + acc[m][n];
        }
    }
    // 7b. gated RMSNorm x SiLU(z) of the output rows (text.py:61-67), G threads per row
    {
      constexpr int VN = GdnVec<T>::N, GL = DH / VN, RPP = kGdnThreads / GL;
      const int g = tid % GL, rr = tid / GL;
      for (int r = rr; r < C; r += RPP) {
        const int t = t0 + r;
        const bool live = t < a.S;
        GdnVec<T> z, o;
        if (live) z.load(proj + (row0 + t) * a.ldp + a.z_col + h * DH + g * VN);
        float ss = 0.f;
#pragma unroll
        for (int c = 0; c < VN; ++c) {
          o.v[c] = round_to<T>(Qs[r * LDQ + g * VN + c]);
          ss += o.v[c] * o.v[c];
        }
        const float rs = rsqrtf(group_sum<GL>(ss) / DH + a.eps);
        if (live) {
#pragma unroll
          for (int c = 0; c < VN; ++c) {
            const float n = round_to<T>(round_to<T>(o.v[c] * rs) * nwv.v[c]);
            o.v[c] = n * (z.v[c] * sigmoid_fast(z.v[c]));
          }
          o.store(out + (row0 + t) * a.ldo + h * DH + g * VN);
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace clef

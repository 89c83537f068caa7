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
// Precision.HIGHEST).  Rows past the sequence end are zero with g = beta = 0,
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
};

constexpr int kGdnChunk = 64;
constexpr int kGdnThreads = 256;

template <int DH>
struct GdnShape {
  static constexpr int C = kGdnChunk;
  static constexpr int LDQ = DH + 1;  // q (later the output rows), k and the solved key rows
  static constexpr int LDA = C + 1;
  static constexpr int TCOL = DH < 16 ? DH : 16;  // threads across output columns
  static constexpr int TROW = kGdnThreads / TCOL;
  static constexpr int NC = DH / TCOL;                           // columns per thread
  static constexpr int RM = C / TROW;                            // rows per thread, 64-row outputs
  static constexpr int RS = DH / TROW > 0 ? DH / TROW : 1;       // rows per thread, DH-row state
  static constexpr size_t floats = size_t(DH) * DH + 3 * C * LDQ + C * DH + C * LDA + 4 * C;
  static constexpr size_t bytes = floats * 4;
};

__device__ __forceinline__ float softplus_f(float x) {  // logaddexp(0, x)
  return fmaxf(x, 0.f) + log1pf(expf(-fabsf(x)));
}

// Depthwise causal conv of projection column `col` at token t (left zero
// padding), FP32 multiply-then-add per tap as text.py:35-37, cast, SiLU, cast.
template <typename T>
__device__ __forceinline__ float gdn_conv_silu(const T* proj, long long ldp, const T* w, int width, long long row0,
                                               int t, int col) {
  float acc = 0.f;
  const T* wr = w + static_cast<long long>(col) * width;
  for (int i = 0; i < width; ++i) {
    const int tt = t - (width - 1) + i;
    const float x = tt >= 0 ? to_f32(proj[(row0 + tt) * ldp + col]) : 0.f;
    acc = __fadd_rn(acc, __fmul_rn(x, to_f32(wr[i])));
  }
  const float y = round_to<T>(acc);
  return round_to<T>(y * sigmoidf_exact(y));
}

// acc[m][n] = sum_d X[i_m][d] * Y[j_n][d] over 64x64 pairs, i_m = ti + 16m, j_n = tj + 16n.
template <int LD>
__device__ __forceinline__ void gdn_gram(float (&acc)[4][4], const float* X, const float* Y, int kd, int ti, int tj) {
#pragma unroll
  for (int m = 0; m < 4; ++m)
#pragma unroll
    for (int n = 0; n < 4; ++n) acc[m][n] = 0.f;
  for (int d = 0; d < kd; ++d) {
    float x[4], y[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) x[m] = X[(ti + 16 * m) * LD + d];
#pragma unroll
    for (int n = 0; n < 4; ++n) y[n] = Y[(tj + 16 * n) * LD + d];
#pragma unroll
    for (int m = 0; m < 4; ++m)
#pragma unroll
      for (int n = 0; n < 4; ++n) acc[m][n] = fmaf(x[m], y[n], acc[m][n]);
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
                RS = G::RS;
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

  const int chunks = (a.S + C - 1) / C;
  for (int ci = 0; ci < chunks; ++ci) {
    const int t0 = ci * C;
    // 1. conv + SiLU, L2 norms, gates
    for (int r = warp; r < C; r += kGdnThreads / 32) {
      const int t = t0 + r;
      if (t < a.S) {
        float qss = 0.f, kss = 0.f;
        for (int c = lane; c < DH; c += 32) {
          const float qv = gdn_conv_silu<T>(proj, a.ldp, convw, a.width, row0, t, q_col + c);
          const float kv = gdn_conv_silu<T>(proj, a.ldp, convw, a.width, row0, t, k_col + c);
          Qs[r * LDQ + c] = qv;
          Ks[r * LDQ + c] = kv;
          Vs[r * DH + c] = gdn_conv_silu<T>(proj, a.ldp, convw, a.width, row0, t, v_col + c);
          qss += qv * qv;
          kss += kv * kv;
        }
        const float qinv = 1.f / sqrtf(warp_sum(qss) + 1e-6f);
        const float kinv = 1.f / sqrtf(warp_sum(kss) + 1e-6f);
        for (int c = lane; c < DH; c += 32) {
          Qs[r * LDQ + c] = round_to<T>(Qs[r * LDQ + c] * qinv) * a.qscale;
          Ks[r * LDQ + c] = round_to<T>(Ks[r * LDQ + c] * kinv);
        }
        if (lane == 0) {
          const T* pr = proj + (row0 + t) * a.ldp;
          gs[r] = neg_a * softplus_f(to_f32(pr[a.a_col + h]) + dt_bias);
          bs[r] = round_to<T>(sigmoidf_exact(to_f32(pr[a.b_col + h])));
        }
      } else {
        for (int c = lane; c < DH; c += 32) {
          Qs[r * LDQ + c] = 0.f;
          Ks[r * LDQ + c] = 0.f;
          Vs[r * DH + c] = 0.f;
        }
        if (lane == 0) {
          gs[r] = 0.f;
          bs[r] = 0.f;
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
          As[i * LDA + j] = j < i ? -(acc[m][n] * bs[i]) * expf(gs[i] - gs[j]) : 0.f;
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
        for (int j = 0; j < r; ++j) acc = fmaf(As[r * LDA + j], x[j], acc);
        x[r] = acc;
        col[r * ld] = acc;
      }
    }
    __syncthreads();
    // 5. value = X_v - X_k S; q k^T * decay (j <= i) into As
    {
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
          As[i * LDA + j] = j <= i ? acc[m][n] * expf(gs[i] - gs[j]) : 0.f;
        }
    }
    __syncthreads();
    // 6. out = (q e^g) S + (q k^T * decay) value -> the rows of Qs
    {
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
    if (tr < DH) {
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
    // 7b. gated RMSNorm x SiLU(z) of the output rows (text.py:61-67)
    for (int r = warp; r < C; r += kGdnThreads / 32) {
      const int t = t0 + r;
      if (t >= a.S) continue;
      float ss = 0.f;
      for (int c = lane; c < DH; c += 32) {
        const float y = round_to<T>(Qs[r * LDQ + c]);
        ss += y * y;
      }
      const float rs = 1.f / sqrtf(warp_sum(ss) / DH + a.eps);
      const T* zr = proj + (row0 + t) * a.ldp + a.z_col + h * DH;
      T* orow = out + (row0 + t) * a.ldo + h * DH;
      for (int c = lane; c < DH; c += 32) {
        const float y = round_to<T>(Qs[r * LDQ + c]);
        const float n = round_to<T>(round_to<T>(y * rs) * to_f32(nw[c]));
        const float z = to_f32(zr[c]);
        orow[c] = from_f32<T>(n * (z * sigmoidf_exact(z)));
      }
    }
    __syncthreads();
  }
}

}  // namespace clef

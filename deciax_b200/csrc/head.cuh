// Joint schema head kernels (models/clef/head.py:50-107) and the lexical
// option means (models/clef/model.py:100, head.py:20-25).  Small, memory-
// or latency-bound work: one block per (batch row, option/field), fp32
// reductions, rounding to T at the reference's cast points.  The dense
// projections and attention between these steps run on the GEMM and
// attention kernels.
#pragma once

#include "common.cuh"

namespace clef {

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x / 32, lane = threadIdx.x & 31, nw = blockDim.x / 32;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}

// out[b, n, :] = T(sum_{s in [lo, hi)} x[b, s, :] / max(hi - lo, 1)), spans [B, N, 2].
// When `ids` is given the rows are table[ids[b, s]] (lexical means over lm_head rows).
template <typename T>
__global__ void span_means_kernel(const T* __restrict__ x, long long ldx, int S, const int32_t* __restrict__ ids,
                                  int vocab, const int32_t* __restrict__ spans, int N, int D, T* __restrict__ out,
                                  int* status) {
  const int n = blockIdx.x, b = blockIdx.y;
  const int lo_raw = spans[(static_cast<long long>(b) * N + n) * 2];
  const int hi_raw = spans[(static_cast<long long>(b) * N + n) * 2 + 1];
  // Positions outside [0, S) never match in the reference's mask formulation.
  const int lo = max(lo_raw, 0), hi = min(hi_raw, S);
  const int cnt = max(hi - lo, 0);
  const float inv = 1.f / static_cast<float>(max(cnt, 1));
  T* orow = out + (static_cast<long long>(b) * N + n) * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    for (int s = lo; s < hi; ++s) {
      long long r;
      if (ids) {
        int id = ids[static_cast<long long>(b) * S + s];
        if (id < 0 || id >= vocab) {
          record_status(status, kBadIndex);
          id = 0;
        }
        r = id;
      } else {
        r = static_cast<long long>(b) * S + s;
      }
      acc += to_f32(x[r * ldx + c]);
    }
    orow[c] = from_f32<T>(acc * inv);
  }
}

// gv[b, :] = h[b, max(sum(mask[b]) - 1, 0), :]   (head.py:55-56)
template <typename T>
__global__ void last_token_kernel(const T* __restrict__ h, int S, int D, const uint8_t* __restrict__ mask,
                                  T* __restrict__ out) {
  const int b = blockIdx.x;
  __shared__ int last;
  if (threadIdx.x == 0) {
    int c = 0;
    for (int s = 0; s < S; ++s) c += mask[static_cast<long long>(b) * S + s] != 0;
    last = max(c - 1, 0);
  }
  __syncthreads();
  const T* src = h + (static_cast<long long>(b) * S + last) * D;
  for (int c = threadIdx.x; c < D; c += blockDim.x) out[static_cast<long long>(b) * D + c] = src[c];
}

// options = T(T(ctx + lex) + qproj[b, owner[b, o]])   (head.py:62-63)
template <typename T>
__global__ void options_init_kernel(const T* __restrict__ ctx, const T* __restrict__ lex, const T* __restrict__ qp,
                                    const int32_t* __restrict__ owner, int O, int Q, int W, T* __restrict__ out) {
  const int o = blockIdx.x, b = blockIdx.y;
  int f = owner[static_cast<long long>(b) * O + o];
  f = min(max(f, 0), Q - 1);
  const long long r = static_cast<long long>(b) * O + o;
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    const float v = round_to<T>(to_f32(ctx[r * W + c]) + to_f32(lex[r * W + c]));
    out[r * W + c] = from_f32<T>(v + to_f32(qp[(static_cast<long long>(b) * Q + f) * W + c]));
  }
}

// Per (b, q): logits over options, field-owned masked softmax, routed summary
// (head.py:73-79).  routing is [B, Q, O]; summary [B, Q, W].
template <typename T>
__global__ void route_summary_kernel(const T* __restrict__ options, const T* __restrict__ base,
                                     const int32_t* __restrict__ owner, const uint8_t* __restrict__ option_mask, int O,
                                     int Q, int W, T* __restrict__ summary) {
  extern __shared__ float sm[];  // O logits/probs + 32 reduction slots
  float* p = sm;
  float* red = sm + O;
  const int q = blockIdx.x, b = blockIdx.y;
  const T* brow = base + (static_cast<long long>(b) * Q + q) * W;
  const float sqrt_w = round_to<T>(sqrtf(static_cast<float>(W)));  // weakly typed Python float -> T
  const int wib = threadIdx.x / 32, lane = threadIdx.x & 31, nw = blockDim.x / 32;
  for (int o = wib; o < O; o += nw) {
    const T* orow = options + (static_cast<long long>(b) * O + o) * W;
    float acc = 0.f;
    for (int c = lane; c < W; c += 32) acc = fmaf(to_f32(orow[c]), to_f32(brow[c]), acc);
    acc = warp_sum(acc);
    if (lane == 0) {
      const float logit = round_to<T>(round_to<T>(acc) / sqrt_w);
      const bool owns = owner[static_cast<long long>(b) * O + o] == q && option_mask[static_cast<long long>(b) * O + o];
      p[o] = owns ? logit : kMaskFill;
    }
  }
  __syncthreads();
  float mx = -INFINITY;
  for (int o = threadIdx.x; o < O; o += blockDim.x) mx = fmaxf(mx, p[o]);
  mx = warp_max(mx);
  __syncthreads();
  if (lane == 0) red[wib] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int i = 0; i < nw; ++i) mx = fmaxf(mx, red[i]);
  __syncthreads();
  float s = 0.f;
  for (int o = threadIdx.x; o < O; o += blockDim.x) s += expf(p[o] - mx);
  s = block_sum(s, red);
  __syncthreads();
  for (int o = threadIdx.x; o < O; o += blockDim.x) p[o] = round_to<T>(expf(p[o] - mx) / s);
  __syncthreads();
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    float acc = 0.f;
    for (int o = 0; o < O; ++o) acc += round_to<T>(p[o] * to_f32(options[(static_cast<long long>(b) * O + o) * W + c]));
    summary[(static_cast<long long>(b) * Q + q) * W + c] = from_f32<T>(acc);
  }
}

// fields = T(T(T(base + sn) + gproj[b]) + type_embedding[types[b, q]])   (head.py:80-82)
template <typename T>
__global__ void fields_init_kernel(const T* __restrict__ base, const T* __restrict__ sn, const T* __restrict__ gp,
                                   const T* __restrict__ type_emb, int n_types, const int32_t* __restrict__ types, int Q,
                                   int W, T* __restrict__ out) {
  const int q = blockIdx.x, b = blockIdx.y;
  const long long r = static_cast<long long>(b) * Q + q;
  int t = types[r];
  t = min(max(t, 0), n_types - 1);
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    float v = round_to<T>(to_f32(base[r * W + c]) + to_f32(sn[r * W + c]));
    v = round_to<T>(v + to_f32(gp[static_cast<long long>(b) * W + c]));
    out[r * W + c] = from_f32<T>(v + to_f32(type_emb[static_cast<long long>(t) * W + c]));
  }
}

// x = T(x + y)
template <typename T>
__global__ void add_inplace_kernel(T* __restrict__ x, const T* __restrict__ y, long long n) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    x[i] = from_f32<T>(to_f32(x[i]) + to_f32(y[i]));
}

// Per (b, o): prior (hidden space), cosine (head space) and the residual
// scorer's feature row [f, o, T(f*o), T(|T(f - o)|)]   (head.py:92-99).
// fn = field_norm(fields) [B,Q,W], on = option_norm(options) [B,O,W].
template <typename T>
__global__ void prior_cosine_kernel(const T* __restrict__ questions, const T* __restrict__ gv,
                                    const T* __restrict__ lexical, const T* __restrict__ fn, const T* __restrict__ on,
                                    const int32_t* __restrict__ owner, int O, int Q, int D, int W,
                                    T* __restrict__ features, float* __restrict__ prior_out,
                                    float* __restrict__ cos_out) {
  __shared__ float red[32];
  const int o = blockIdx.x, b = blockIdx.y;
  const long long r = static_cast<long long>(b) * O + o;
  int f = owner[r];
  f = min(max(f, 0), Q - 1);
  const T* qrow = questions + (static_cast<long long>(b) * Q + f) * D;
  const T* grow = gv + static_cast<long long>(b) * D;
  const T* lrow = lexical + r * D;
  // anchor = normalize(T(q + g)); lexn = normalize(lex)
  float sa = 0.f, sl = 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const float a = round_to<T>(to_f32(qrow[c]) + to_f32(grow[c]));
    const float l = to_f32(lrow[c]);
    sa += a * a;
    sl += l * l;
  }
  sa = block_sum(sa, red);
  sl = block_sum(sl, red);
  const float eps12 = round_to<T>(1e-12f);
  const float la = fmaxf(round_to<T>(sqrtf(sa)), eps12), ll = fmaxf(round_to<T>(sqrtf(sl)), eps12);
  float pr = 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    const float a = round_to<T>(round_to<T>(to_f32(qrow[c]) + to_f32(grow[c])) / la);
    const float l = round_to<T>(to_f32(lrow[c]) / ll);
    pr += round_to<T>(a * l);
  }
  pr = block_sum(pr, red);
  // cosine in head space
  const T* frow = fn + (static_cast<long long>(b) * Q + f) * W;
  const T* orow = on + r * W;
  float sf = 0.f, so = 0.f;
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    const float x = to_f32(frow[c]), y = to_f32(orow[c]);
    sf += x * x;
    so += y * y;
  }
  sf = block_sum(sf, red);
  so = block_sum(so, red);
  const float eps8 = round_to<T>(1e-8f);
  const float lf = fmaxf(round_to<T>(sqrtf(sf)), eps8), lo = fmaxf(round_to<T>(sqrtf(so)), eps8);
  float cs = 0.f;
  T* feat = features + r * 4 * W;
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    const float x = to_f32(frow[c]), y = to_f32(orow[c]);
    cs += round_to<T>(round_to<T>(x / lf) * round_to<T>(y / lo));
    feat[c] = from_f32<T>(x);
    feat[W + c] = from_f32<T>(y);
    feat[2 * W + c] = from_f32<T>(x * y);
    feat[3 * W + c] = from_f32<T>(fabsf(round_to<T>(x - y)));
  }
  cs = block_sum(cs, red);
  if (threadIdx.x == 0) {
    prior_out[r] = round_to<T>(pr);
    cos_out[r] = round_to<T>(cs);
  }
}

// logits = where(option_mask, T(prior*ps) + T(sig(g) * T(T(js*cos) + residual)), -1e9)   (head.py:95-107)
template <typename T>
__global__ void final_logits_kernel(const float* __restrict__ prior, const float* __restrict__ cosine,
                                    const T* __restrict__ residual, const uint8_t* __restrict__ option_mask,
                                    const T* __restrict__ prior_scale, const T* __restrict__ joint_scale,
                                    const T* __restrict__ gate, int n, float max_log_scale, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float ps = round_to<T>(expf(round_to<T>(fminf(to_f32(prior_scale[0]), round_to<T>(max_log_scale)))));
  const float js = round_to<T>(expf(round_to<T>(fminf(to_f32(joint_scale[0]), round_to<T>(max_log_scale)))));
  const float g = round_to<T>(sigmoidf_exact(to_f32(gate[0])));
  const float p = round_to<T>(prior[i] * ps);
  const float joint = round_to<T>(round_to<T>(js * cosine[i]) + to_f32(residual[i]));
  const float score = round_to<T>(p + round_to<T>(g * joint));
  out[i] = option_mask[i] ? score : -1e9f;
}

}  // namespace clef

// Softmax attention, [B, Lq, H, hd] x [B, Lk, Hk, hd] -> [B, Lq, H, hd], GQA.
//
// Semantics follow the reference's blocked attention
// (kernels/attention/blocked.py:9-32): FP32 scores scaled by hd^-1/2, masked
// entries set to MASK_FILL = -1e30 (so a row with no valid key averages
// every key uniformly), FP32 softmax, probabilities rounded to the activation
// type before P.V, FP32 accumulation, output rounded.  The full-attention
// layer's sigmoid output gate (text.py:91) is fused into the store:
// out = T(T(o) * T(sigmoid(gate))).
//
// Beyond-reference flags (off = reference): softcap > 0 applies
// softcap*tanh(s/softcap) to scaled scores; window > 0 keeps keys with
// i - j < window.
//
// attn_simt_kernel      exact two-pass, any head size, one warp per query
//                       row; fp32 mode and the joint head's attention.
// attn_fa2_bf16_kernel  bf16 mma.sync m16n8k16 flash attention (online
//                       softmax), head size 64/128/256, causal backbone path.
#pragma once

#include "common.cuh"

namespace clef {

template <typename T>
struct AttnArgs {
  const T* q;
  long long ldq, hsq;  // token stride, head stride (elements)
  const T* k;
  long long ldk, hsk;
  const T* v;
  long long ldv, hsv;
  const T* gate;  // nullable; indexed like q
  long long ldg, hsg;
  T* out;
  long long ldo, hso;
  const uint8_t* key_mask;  // [B, Lk], nullable = all valid
  int B, Lq, Lk, H, Hk, hd;
  int causal;
  float softcap;
  int window;
  int* status;
  // q, k, v and gate are column offsets of one row-major [B*L, ldq] buffer
  // starting at q (the packed QKV projection); enables the tcgen05 kernel.
  int packed;
  // the gate slots already hold T(sigmoid(T(gate))) (QKV GEMM epilogue)
  int gate_presig;
};

// T(sigmoid(g)) of a raw gate, or the value itself when it was precomputed.
template <typename T>
__device__ __forceinline__ float gate_factor(float g, int presig) {
  return presig ? g : round_to<T>(sigmoidf_exact(g));
}

__device__ __forceinline__ float attn_score_transform(float s, float softcap) {
  return softcap > 0.f ? softcap * tanhf(s / softcap) : s;
}

// ---------------------------------------------------------------------------
// exact two-pass SIMT attention
// ---------------------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(AttnArgs<T> a) {
  extern __shared__ float qbuf[];  // 4 warps x hd
  const int wib = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int i = blockIdx.x * 4 + wib;  // query row
  const int h = blockIdx.y, b = blockIdx.z;
  if (i >= a.Lq) return;
  const int hk = h / (a.H / a.Hk);
  const int hd = a.hd;
  float* qs = qbuf + wib * hd;
  const T* qrow = a.q + (static_cast<long long>(b) * a.Lq + i) * a.ldq + h * a.hsq;
  for (int c = lane; c < hd; c += 32) qs[c] = to_f32(qrow[c]);
  __syncwarp();
  const float scale = rsqrtf(static_cast<float>(hd));
  const T* kbase = a.k + static_cast<long long>(b) * a.Lk * a.ldk + hk * a.hsk;
  const T* vbase = a.v + static_cast<long long>(b) * a.Lk * a.ldv + hk * a.hsv;
  const uint8_t* mrow = a.key_mask ? a.key_mask + static_cast<long long>(b) * a.Lk : nullptr;
  int lo = 0, hi = a.Lk;
  if (a.causal) {
    hi = min(i + 1, a.Lk);
    if (a.window > 0) lo = max(0, i - a.window + 1);
  }
  auto score = [&](int j) -> float {
    const T* kr = kbase + static_cast<long long>(j) * a.ldk;
    float s = 0.f;
    for (int c = 0; c < hd; ++c) s = fmaf(qs[c], to_f32(kr[c]), s);
    s = attn_score_transform(s * scale, a.softcap);
    const bool valid = (!mrow || mrow[j]) && (!a.causal || (j <= i && (a.window <= 0 || i - j < a.window)));
    return valid ? s : kMaskFill;
  };
  // pass 1: running max and normaliser
  float m = -INFINITY, l = 0.f;
  for (int j0 = lo; j0 < hi; j0 += 32) {
    const int j = j0 + lane;
    const float s = j < hi ? score(j) : -INFINITY;
    const float cm = warp_max(s);
    const float mn = fmaxf(m, cm);
    const float p = j < hi ? expf(s - mn) : 0.f;
    l = l * expf(m - mn) + warp_sum(p);
    m = mn;
  }
  // A causal row with no valid key: the reference averages all Lk keys.
  const bool uniform = a.causal && m <= kMaskFill;
  if (uniform) {
    lo = 0;
    hi = a.Lk;
  }
  const float inv_l = 1.f / l;
  const float pu = round_to<T>(1.f / static_cast<float>(a.Lk));
  // pass 2: P.V with probabilities rounded to T
  constexpr int MAXC = 8;  // hd <= 256
  float o[MAXC];
#pragma unroll
  for (int c = 0; c < MAXC; ++c) o[c] = 0.f;
  for (int j0 = lo; j0 < hi; j0 += 32) {
    const int j = j0 + lane;
    float p = 0.f;
    if (j < hi) p = uniform ? pu : round_to<T>(expf(score(j) - m) * inv_l);
    const int cnt = min(32, hi - j0);
    for (int jj = 0; jj < cnt; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const T* vr = vbase + static_cast<long long>(j0 + jj) * a.ldv;
#pragma unroll
      for (int c = 0; c < MAXC; ++c) {
        const int col = lane + 32 * c;
        if (col < hd) o[c] = fmaf(pj, to_f32(vr[col]), o[c]);
      }
    }
  }
  T* orow = a.out + (static_cast<long long>(b) * a.Lq + i) * a.ldo + h * a.hso;
  const T* grow = a.gate ? a.gate + (static_cast<long long>(b) * a.Lq + i) * a.ldg + h * a.hsg : nullptr;
#pragma unroll
  for (int c = 0; c < MAXC; ++c) {
    const int col = lane + 32 * c;
    if (col < hd) {
      float val = round_to<T>(o[c]);
      if (grow) val = val * gate_factor<T>(to_f32(grow[col]), a.gate_presig);
      orow[col] = from_f32<T>(val);
    }
  }
}

// ---------------------------------------------------------------------------
// bf16 flash attention on mma.sync (m16n8k16), 4 warps x 16 query rows
// ---------------------------------------------------------------------------

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int D>
struct Fa2Shape {
  static constexpr int BQ = 64, BKV = 64, LDS = D + 8;
  static constexpr size_t SMEM = static_cast<size_t>(3 * 64 * LDS) * 2 + 64 * sizeof(float);
};

template <int D>
__global__ void __launch_bounds__(128, 2) attn_fa2_bf16_kernel(AttnArgs<__nv_bfloat16> a) {
  using Sh = Fa2Shape<D>;
  constexpr int BQ = Sh::BQ, BKV = Sh::BKV, LDS = Sh::LDS;
  extern __shared__ __align__(16) uint8_t fa_smem[];
  __nv_bfloat16* Qs = reinterpret_cast<__nv_bfloat16*>(fa_smem);
  __nv_bfloat16* Ks = Qs + BQ * LDS;
  __nv_bfloat16* Vs = Ks + BKV * LDS;
  float* kvalid = reinterpret_cast<float*>(Vs + BKV * LDS);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nqb = (a.Lq + BQ - 1) / BQ;
  const int qb = nqb - 1 - blockIdx.x;  // heaviest causal blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hk);
  const int q0 = qb * BQ;

  const __nv_bfloat16* qg = a.q + static_cast<long long>(b) * a.Lq * a.ldq + h * a.hsq;
  const __nv_bfloat16* kg = a.k + static_cast<long long>(b) * a.Lk * a.ldk + hk * a.hsk;
  const __nv_bfloat16* vg = a.v + static_cast<long long>(b) * a.Lk * a.ldv + hk * a.hsv;
  const uint8_t* mrow = a.key_mask ? a.key_mask + static_cast<long long>(b) * a.Lk : nullptr;

  constexpr int CPR = D / 8;  // 16-byte chunks per row
  auto load_tile = [&](__nv_bfloat16* dst, const __nv_bfloat16* src, long long ld, int row0, int rows_total) {
    for (int c = tid; c < 64 * CPR; c += 128) {
      const int r = c / CPR, cc = c % CPR;
      const bool ok = row0 + r < rows_total;
      const __nv_bfloat16* s = src + static_cast<long long>(ok ? row0 + r : 0) * ld + cc * 8;
      cp_async16(dst + r * LDS + cc * 8, s, ok);
    }
  };

  int kb_hi = (a.Lk + BKV - 1) / BKV;
  int kb_lo = 0;
  if (a.causal) {
    kb_hi = min(kb_hi, (min(q0 + BQ, a.Lq) - 1) / BKV + 1);
    if (a.window > 0) kb_lo = max(0, (q0 - a.window + 1)) / BKV;
  }

  load_tile(Qs, qg, a.ldq, q0, a.Lq);
  load_tile(Ks, kg, a.ldk, kb_lo * BKV, a.Lk);
  cp_async_commit();
  load_tile(Vs, vg, a.ldv, kb_lo * BKV, a.Lk);
  cp_async_commit();

  const float scale_log2 = rsqrtf(static_cast<float>(D)) * 1.4426950408889634f;
  const float fill_log2 = kMaskFill * 1.4426950408889634f;
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow_max[2] = {-INFINITY, -INFINITY};  // in log2 units
  float lsum[2] = {0.f, 0.f};

  const int r_lo = q0 + warp * 16 + (lane >> 2);  // this thread's rows: r_lo, r_lo + 8
  const uint32_t qs_base = smem_u32(Qs);
  const uint32_t ks_base = smem_u32(Ks);
  const uint32_t vs_base = smem_u32(Vs);

  for (int kb = kb_lo; kb < kb_hi; ++kb) {
    const int k0 = kb * BKV;
    cp_async_wait<1>();
    if (tid < 64) {
      const int key = k0 + tid;
      kvalid[tid] = (key < a.Lk && (!mrow || mrow[key])) ? 1.f : 0.f;
    }
    __syncthreads();

    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < D / 16; ++kc) {
      uint32_t a0, a1, a2, a3;
      {
        const int row = warp * 16 + (lane & 15);
        const int col = kc * 16 + (lane >> 4) * 8;
        ldsm_x4(qs_base + (row * LDS + col) * 2, a0, a1, a2, a3);
      }
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        const int mi = lane >> 3;
        const int row = np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int col = kc * 16 + (mi & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(ks_base + (row * LDS + col) * 2, b0, b1, b2, b3);
        mma_bf16_16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with Ks
    const bool more = kb + 1 < kb_hi;
    if (more) load_tile(Ks, kg, a.ldk, k0 + BKV, a.Lk);
    cp_async_commit();

    // scale, transform, mask; row max (log2 units)
    float bmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kl = j * 8 + 2 * (lane & 3) + (e & 1);
        const int key = k0 + kl;
        const int row = r_lo + (e >> 1) * 8;
        bool valid = kvalid[kl] != 0.f;
        if (a.causal) valid = valid && key <= row && (a.window <= 0 || row - key < a.window);
        float v;
        if (a.softcap > 0.f) {
          v = attn_score_transform(s[j][e] * rsqrtf(static_cast<float>(D)), a.softcap) * 1.4426950408889634f;
        } else {
          v = s[j][e] * scale_log2;
        }
        v = valid ? v : fill_log2;
        s[j][e] = v;
        bmax[e >> 1] = fmaxf(bmax[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      bmax[r] = fmaxf(bmax[r], __shfl_xor_sync(0xffffffffu, bmax[r], 1));
      bmax[r] = fmaxf(bmax[r], __shfl_xor_sync(0xffffffffu, bmax[r], 2));
      const float mn = fmaxf(mrow_max[r], bmax[r]);
      corr[r] = exp2f(mrow_max[r] - mn);
      mrow_max[r] = mn;
      lsum[r] *= corr[r];
    }
    uint32_t pa[4][4];  // P as A fragments, one per 16-key chunk
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        p[e] = exp2f(s[j][e] - mrow_max[e >> 1]);
        lsum[e >> 1] += p[e];
      }
      pa[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p[0], p[1]);
      pa[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p[2], p[3]);
    }
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }

    if (more) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncthreads();  // V tile visible
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      // pa[kc] = {a0 (row lo, keys 0-7 pair), a1 (row hi), a2 (row lo, keys 8-15), a3 (row hi)}
      const uint32_t a0 = pa[kc][0], a1 = pa[kc][1], a2 = pa[kc][2], a3 = pa[kc][3];
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        const int mi = lane >> 3;
        const int row = kc * 16 + (lane & 7) + (mi & 1) * 8;
        const int col = np * 16 + (mi >> 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vs_base + (row * LDS + col) * 2, b0, b1, b2, b3);
        mma_bf16_16816(o[2 * np], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with Vs
    if (more) load_tile(Vs, vg, a.ldv, k0 + BKV, a.Lk);
    cp_async_commit();
  }
  cp_async_wait<0>();

  // epilogue: normalise, round, gate, store
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 1);
    lsum[r] += __shfl_xor_sync(0xffffffffu, lsum[r], 2);
  }
  const float inv[2] = {1.f / lsum[0], 1.f / lsum[1]};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = r_lo + r * 8;
    if (row >= a.Lq) continue;
    __nv_bfloat16* orow = a.out + (static_cast<long long>(b) * a.Lq + row) * a.ldo + h * a.hso;
    const __nv_bfloat16* grow =
        a.gate ? a.gate + (static_cast<long long>(b) * a.Lq + row) * a.ldg + h * a.hsg : nullptr;
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      const int col = j * 8 + 2 * (lane & 3);
      float v0 = round_to<__nv_bfloat16>(o[j][2 * r] * inv[r]);
      float v1 = round_to<__nv_bfloat16>(o[j][2 * r + 1] * inv[r]);
      if (grow) {
        const __nv_bfloat162 g = *reinterpret_cast<const __nv_bfloat162*>(grow + col);
        v0 *= gate_factor<__nv_bfloat16>(__low2float(g), a.gate_presig);
        v1 *= gate_factor<__nv_bfloat16>(__high2float(g), a.gate_presig);
      }
      *reinterpret_cast<uint32_t*>(orow + col) = pack_bf16x2(v0, v1);
    }
  }
}

}  // namespace clef

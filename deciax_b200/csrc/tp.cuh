// Tensor-parallel reduction of the o-proj / down-proj partial products over
// NVLink peer memory: the FP32 sum across ranks, the cast, and the residual
// add of qwen3_5/pallas.py:66-69,121 (x = T(x + T(sum_k partial_k))), in one
// kernel per rank instead of an NCCL all-reduce followed by an add kernel.
//
// Every rank owns a contiguous 1/tp share of the rows.  For each element of
// its share it reads the tp FP32 partials (its own and, through CUDA IPC
// pointers, each peer's) and sums them in rank order -- so the result is the
// same bits on every rank -- adds its residual, casts, and stores the result
// into every rank's residual stream x (its own copy and each peer's).  The
// launch sits between two cross-rank barriers on the stream: before it every
// rank's partial is complete, after it every rank's x is.  Plain 16/8-byte
// peer loads and stores only; no multicast.  (Pushing the partials from the
// GEMM epilogue into their owners' memory instead was measured slower: the
// NVLink stores stall the epilogue.)
#pragma once

#include "common.cuh"

namespace clef {

constexpr int kTpMaxRanks = 8;

struct TpReduceArgs {
  const float* parts[kTpMaxRanks];  // rank k's FP32 partial [rows, dim]
  void* xs[kTpMaxRanks];            // rank k's residual stream x [rows, dim]
  int tp, rank;
  long long e0, e1;  // this rank's element range, multiples of 4 (of 8 with vec8)
  int vec8;          // bf16, e0 and e1 multiples of 8, 16-byte aligned rows: 8 elements per step
};

template <typename T>
__global__ void __launch_bounds__(256) tp_reduce_residual_kernel(TpReduceArgs a) {
  const T* own = static_cast<const T*>(a.xs[a.rank]);
  if constexpr (sizeof(T) == 2) {
    if (a.vec8) {
      // 8 elements per step: two 16-byte loads of every rank's partial in
      // flight, one 16-byte residual load, one 16-byte store per rank
      const long long stride8 = 8LL * gridDim.x * blockDim.x;
      for (long long i = a.e0 + 8LL * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x); i < a.e1;
           i += stride8) {
        float4 p0[kTpMaxRanks], p1[kTpMaxRanks];
#pragma unroll
        for (int k = 0; k < kTpMaxRanks; ++k)
          if (k < a.tp) {
            p0[k] = *reinterpret_cast<const float4*>(a.parts[k] + i);
            p1[k] = *reinterpret_cast<const float4*>(a.parts[k] + i + 4);
          }
        const uint4 rv = *reinterpret_cast<const uint4*>(own + i);
        float4 s0 = p0[0], s1 = p1[0];
#pragma unroll
        for (int k = 1; k < kTpMaxRanks; ++k)
          if (k < a.tp) {
            s0.x += p0[k].x;
            s0.y += p0[k].y;
            s0.z += p0[k].z;
            s0.w += p0[k].w;
            s1.x += p1[k].x;
            s1.y += p1[k].y;
            s1.z += p1[k].z;
            s1.w += p1[k].w;
          }
        const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
        const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
        uint32_t ow[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 r2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rw[e]));
          ow[e] = pack_bf16x2(r2.x + round_to<T>(sv[2 * e]), r2.y + round_to<T>(sv[2 * e + 1]));
        }
        const uint4 o = make_uint4(ow[0], ow[1], ow[2], ow[3]);
#pragma unroll
        for (int k = 0; k < kTpMaxRanks; ++k)
          if (k < a.tp) *reinterpret_cast<uint4*>(static_cast<T*>(a.xs[k]) + i) = o;
      }
      __threadfence_system();  // peer stores ordered before the barrier that follows
      return;
    }
  }
  const long long stride = 4LL * gridDim.x * blockDim.x;
  for (long long i = a.e0 + 4LL * (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x); i < a.e1;
       i += stride) {
    // every rank's partial in flight at once, then the sum in rank order
    float4 p[kTpMaxRanks];
#pragma unroll
    for (int k = 0; k < kTpMaxRanks; ++k)
      if (k < a.tp) p[k] = *reinterpret_cast<const float4*>(a.parts[k] + i);
    float4 s = p[0];
#pragma unroll
    for (int k = 1; k < kTpMaxRanks; ++k)
      if (k < a.tp) {
        s.x += p[k].x;
        s.y += p[k].y;
        s.z += p[k].z;
        s.w += p[k].w;
      }
    if constexpr (sizeof(T) == 2) {
      const uint2 rv = *reinterpret_cast<const uint2*>(own + i);
      const float2 r0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rv.x));
      const float2 r1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&rv.y));
      const uint2 o = make_uint2(pack_bf16x2(r0.x + round_to<T>(s.x), r0.y + round_to<T>(s.y)),
                                 pack_bf16x2(r1.x + round_to<T>(s.z), r1.y + round_to<T>(s.w)));
#pragma unroll
      for (int k = 0; k < kTpMaxRanks; ++k)
        if (k < a.tp) *reinterpret_cast<uint2*>(static_cast<T*>(a.xs[k]) + i) = o;
    } else {
      const float4 r = *reinterpret_cast<const float4*>(own + i);
      const float4 o = make_float4(r.x + s.x, r.y + s.y, r.z + s.z, r.w + s.w);
#pragma unroll
      for (int k = 0; k < kTpMaxRanks; ++k)
        if (k < a.tp) *reinterpret_cast<float4*>(static_cast<T*>(a.xs[k]) + i) = o;
    }
  }
  __threadfence_system();  // peer stores ordered before the barrier that follows
}

}  // namespace clef

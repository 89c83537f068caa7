// Causal GQA flash attention on CTA pairs (tcgen05 cta_group::2), sm_100a.
//
// A cluster of two CTAs on two SMs takes 256 query rows of one (batch row,
// query head); CTA r holds rows [q0 + 128 r, +128).  Keys go in 128-key tiles.
//
//   S_j = Q K_j^T   tcgen05.mma.cta_group::2, M = 256, N = 128, K = D: each
//                   CTA supplies its 128 query rows (A) and 64 of the tile's
//                   128 keys (B); each CTA's tensor memory receives its 128
//                   rows x all 128 keys.
//   O  += P_j V_j   M = 256, N = D, K = 128: A = P, which the softmax writes
//                   as bf16 pairs over the first 64 columns of its S buffer
//                   (the A operand read from tensor memory); B = V_j, each CTA
//                   holding all 128 keys x its D/2 head-dim columns.
//
// Why pairs: a one-CTA tile of 128 rows x 64 keys issues QK^T at N = 64,
// where each instruction reads 6 KB of operands from shared memory for 32
// cycles of math -- shared-memory bound at about half the tensor rate.  Here
// each CTA reads 6 KB per 64-cycle QK^T instruction and 8 KB per 128-cycle
// P.V instruction, both below the 128 B/clk shared-memory rate, and the K and
// V tiles cost each CTA half the shared memory, which leaves room for two
// stages of each at D = 256 (192 KB in all).
//
// Tensor memory per CTA (512 columns): O at [0, D), S buffers at D and
// D + 128.  Warps: 0 TMA producer (this CTA's halves; the leader's full
// barriers count both CTAs' bytes), 1 MMA issuer (leader CTA, one thread),
// 2..9 softmax of the CTA's 128 rows, two threads per row (64 keys of each
// tile each: one thread per row is bound by the latency of its ~1400
// dependent instructions per tile), then the epilogue (O / l times the
// sigmoid gate, staged in the Q buffer and stored by TMA).
//
// Ordering.  The MMA thread issues QK_0, QK_1, PV_0, QK_2, PV_1, ...;
// tcgen05.mma instructions of one thread execute in order, so QK_{j+2}
// (which overwrites S buffer j % 2, where P_j lives) runs after PV_j has read
// P_j.  The softmax of tile j waits for S_j (sfull, a commit after QK_j,
// which also covers PV_{j-2}); a rescale of O waits for PV_{j-1} (ofull).
// The running max moves only when it grows by more than 2^8 (log2 units);
// the final division by the row sum cancels the stale max exactly.
//
// Barriers: qfull, kfull[2], vfull[2] and pfull[2] live in the leader
// (pfull gets one arrive per softmax warp of both CTAs); kempty, vempty,
// sfull, ofull, ofinal and drain live in both CTAs and are signalled by the
// leader's commits multicast to the pair.  Every wait is bounded (common.cuh);
// no TMA multicast anywhere.
//
// Reference semantics: kernels/attention/blocked.py:9-32 (FP32 scores scaled
// by D^-1/2, MASK_FILL, FP32 softmax, probabilities rounded to bf16 before
// P.V, FP32 accumulation) and the output gate of qwen3_5/text.py:91.
#pragma once

#include "attention_sm100.cuh"
#include "common.cuh"
#include "gemm2_sm100.cuh"

namespace clef {

template <int D>
struct AttnPairShape {
  static constexpr int BQ = 128, BK = 128, ATOMS = D / 64;
  static constexpr uint32_t Q_BYTES = BQ * D * 2;            // ATOMS x [128 rows x 128 B]
  static constexpr uint32_t KH_BYTES = (BK / 2) * D * 2;     // this CTA's 64 keys: ATOMS x [64 rows x 128 B]
  static constexpr uint32_t VH_BYTES = BK * (D / 2) * 2;     // 128 keys x D/2 columns: ATOMS/2 x [128 rows x 128 B]
  static constexpr uint32_t O_COL = 0, S_COL = D;            // S buffers at D and D + BK
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int NBARS = 18;
  static constexpr int THREADS = 320;  // producer, MMA issuer, 8 softmax warps
  static constexpr size_t SMEM = 1024 + Q_BYTES + 2 * KH_BYTES + 2 * VH_BYTES + 256 + 6 * BQ * 4 + 16;
  static_assert(D + 2 * BK <= 512, "O and two S buffers must fit the 512 tensor-memory columns");
  static_assert(2 * KH_BYTES >= Q_BYTES, "the gate rows are staged in the two K stages");
};

// The pair MMA with A (P) in tensor memory: row i of this CTA's A in lane i,
// two bf16 per 32-bit column, K = 16 over 8 columns; both CTAs' tensor memory
// at the same address supply their 128 rows.
__device__ __forceinline__ void umma_bf16_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Wait on a barrier of this CTA that the peer CTA also arrives on: acquire at
// cluster scope, so the peer's tensor-memory stores before its arrive are
// visible to the MMAs issued after the wait.  Bounded like mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status, int code) {
  const uint32_t addr = smem_u32(bar);
  auto probe = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (probe()) return true;
  const long long t0 = clock64();
  while (!probe()) {
    if (clock64() - t0 > kWaitCycles) {
      record_status(status, code);
      return false;
    }
  }
  return true;
}

template <int D>
__global__ void __launch_bounds__(AttnPairShape<D>::THREADS, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_out,
                     AttnTcArgs a) {
  using Sh = AttnPairShape<D>;
  constexpr int BQ = Sh::BQ, BK = Sh::BK, ATOMS = Sh::ATOMS;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(2 * BQ, BK);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(2 * BQ, D) | (1u << 16);  // B (V) is MN-major
  constexpr float LOG2E = 1.4426950408889634f;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Sh::Q_BYTES;        // 2 stages of this CTA's 64 keys
  uint8_t* sV = sK + 2 * Sh::KH_BYTES;   // 2 stages of this CTA's D/2 columns
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * Sh::VH_BYTES);
  uint64_t* qfull = bars;        // leader
  uint64_t* kfull = bars + 1;    // leader, 2
  uint64_t* vfull = bars + 3;    // leader, 2
  uint64_t* pfull = bars + 5;    // leader, 2 (16 arrives: 8 softmax warps x 2 CTAs)
  uint64_t* kempty = bars + 7;   // both, 2
  uint64_t* vempty = bars + 9;   // both, 2
  uint64_t* sfull = bars + 11;   // both, 2
  uint64_t* ofull = bars + 13;   // both
  uint64_t* ofinal = bars + 14;  // both
  uint64_t* drain = bars + 15;   // both
  uint64_t* gfull = bars + 16;   // own gate load
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Sh::NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(bars + Sh::NBARS + 2);  // [2 tiles][2 halves][128 rows] row-max exchange
  float* xsum = xmax + 4 * BQ;                                    // [2 halves][128 rows] row-sum exchange
  volatile int* xfail = reinterpret_cast<volatile int*>(xsum + 2 * BQ);  // [2 tiles] a softmax warp's failed wait

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int npq = (a.S + 2 * BQ - 1) / (2 * BQ);
  const int pq = npq - 1 - static_cast<int>(blockIdx.x >> 1);  // heaviest (most keys) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hk);
  const int q0 = pq * 2 * BQ;              // the pair's first row
  const int qc = q0 + static_cast<int>(rank) * BQ;  // this CTA's first row
  const int kb_hi = (min(q0 + 2 * BQ, a.S) - 1) / BK + 1;
  const int kb_lo = a.window > 0 ? max(0, q0 - a.window + 1) / BK : 0;
  const int n = kb_hi - kb_lo;
  const int row_base = b * a.S;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < Sh::NBARS - 1; ++i) mbar_init(&bars[i], (i == 5 || i == 6) ? 16 : 1);
    *abort_flag = 0;
    xfail[0] = xfail[1] = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Sh::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: this CTA's halves ----------------
      const uint32_t lead = mapa_shared(smem_u32(bars), 0);  // the leader's barrier block
      const uint32_t qfull_l = lead, kfull_l = lead + 8, vfull_l = lead + 24;
      if (leader) mbar_arrive_expect_tx(qfull, 2 * Sh::Q_BYTES);
      for (int at = 0; at < ATOMS; ++at)
        for (int half = 0; half < 2; ++half)
          tma_load_2d_pair(sQ + at * (BQ * 128) + half * (64 * 128), &tmap, qfull_l, a.q_col + h * a.hsq + at * 64,
                           row_base + qc + half * 64);
      // K runs one tile ahead of V: a K stage frees when its QK^T is done, a
      // V stage only after the (later) P.V of the tile two back.
      int nk = 0, nv = 0;
      for (int i = 0; i <= n && !*abort_flag; ++i) {
        if (i < n) {
          const int s = i & 1;
          if (!mbar_wait(&kempty[s], ((i >> 1) & 1) ^ 1, a.status, kTimeoutAttention)) {
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&kfull[s], 2 * Sh::KH_BYTES);
          const int key0 = (kb_lo + i) * BK + static_cast<int>(rank) * (BK / 2);
          for (int at = 0; at < ATOMS; ++at)
            tma_load_2d_pair(sK + s * Sh::KH_BYTES + at * ((BK / 2) * 128), &tmap, kfull_l + s * 8,
                             a.k_col + hk * a.hsk + at * 64, row_base + key0);
          nk = i + 1;
        }
        if (i >= 1) {
          const int u = i - 1, s = u & 1;
          if (!mbar_wait(&vempty[s], ((u >> 1) & 1) ^ 1, a.status, kTimeoutAttention)) {
            *abort_flag = 1;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&vfull[s], 2 * Sh::VH_BYTES);
          for (int at = 0; at < ATOMS / 2; ++at)
            for (int half = 0; half < 2; ++half)
              tma_load_2d_pair(sV + s * Sh::VH_BYTES + at * (BK * 128) + half * (64 * 128), &tmap, vfull_l + s * 8,
                               a.v_col + hk * a.hsk + (static_cast<int>(rank) * (ATOMS / 2) + at) * 64,
                               row_base + (kb_lo + u) * BK + half * 64);
          nv = u + 1;
        }
      }
      // Gate prefetch: once the last QK^T has consumed both K stages, load
      // this CTA's gate rows (128 x D) into them for the epilogue.
      bool gate_issued = false;
      if (a.gate && !*abort_flag && nk == n) {
        bool free_ = true;
        for (int t = max(0, n - 2); t < n; ++t)
          free_ = free_ && mbar_wait(&kempty[t & 1], (t >> 1) & 1, a.status, kTimeoutAttention);
        if (free_) {
          mbar_arrive_expect_tx(gfull, Sh::Q_BYTES);
          for (int at = 0; at < ATOMS; ++at)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(sK + at * (BQ * 128) + half * (64 * 128), &tmap, gfull, a.g_col + h * a.hsq + at * 64,
                          row_base + qc + half * 64);
          gate_issued = true;
        } else {
          *abort_flag = 1;
        }
      }
      // Every load of this CTA lands before it may exit.  The leader's full
      // barriers count both CTAs' bytes, so the leader drains for the pair
      // (the final cluster barrier holds the peer until then); only the last
      // two stages per ring can still be in flight.
      if (leader) {
        mbar_wait(qfull, 0, a.status, kTimeoutDrain);
        for (int t = max(0, nk - 2); t < nk; ++t) mbar_wait(&kfull[t & 1], (t >> 1) & 1, a.status, kTimeoutDrain);
        for (int t = max(0, nv - 2); t < nv; ++t) mbar_wait(&vfull[t & 1], (t >> 1) & 1, a.status, kTimeoutDrain);
      }
      if (gate_issued) mbar_wait(gfull, 0, a.status, kTimeoutDrain);
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      // ---------------- MMA issuer (leader) ----------------
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int u) -> bool {
        const int s = u & 1;
        const uint32_t ph = (u >> 1) & 1;
        if (!mbar_wait_cluster(&pfull[s], ph, a.status, kTimeoutAttention) ||
            !mbar_wait(&vfull[s], ph, a.status, kTimeoutAttention))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + s * Sh::VH_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)  // 16 keys of P = 8 tensor-memory columns
          umma_bf16_pair_ts(tmem + Sh::O_COL, tmem + Sh::S_COL + s * BK + kk * 8,
                            smem_desc_mn128(v_addr + kk * 16 * 128, BK * 128), IDESC_PV, (u > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair(&vempty[s]);
        umma_commit_pair(ofull);
        return true;
      };
      bool ok = mbar_wait(qfull, 0, a.status, kTimeoutAttention);
      for (int t = 0; ok && t < n && !*abort_flag; ++t) {
        const int s = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&kfull[s], ph, a.status, kTimeoutAttention)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + s * Sh::KH_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int at = kk >> 2, w = kk & 3;
          umma_bf16_pair(tmem + Sh::S_COL + s * BK, smem_desc_k128(q_addr + at * (BQ * 128) + w * 32),
                         smem_desc_k128(k_addr + at * ((BK / 2) * 128) + w * 32), IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit_pair(&kempty[s]);
        umma_commit_pair(&sfull[s]);
        if (t >= 1 && !issue_pv(t - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && !*abort_flag) ok = issue_pv(n - 1);
      if (!ok) *abort_flag = 1;
      umma_commit_pair(ofinal);
      umma_commit_pair(drain);
      mbar_wait(drain, 0, a.status, kTimeoutDrain);
    }
  } else {
    // ---------------- softmax / epilogue warps ----------------
    // Two threads per query row: warp w (2..9) takes tensor-memory lane
    // quarter w % 4 and key half hf = (w - 2) / 4 of each 128-key tile (64
    // keys), and in the epilogue the same half of O's columns.  The two
    // threads of a row exchange their tile maxima through shared memory, so
    // both hold the same running max; each keeps the sum of its own half.
    const int q4 = warp & 3;
    const int hf = (warp - 2) >> 2;
    const int r = q4 * 32 + lane;
    const int row = qc + r;
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    const float scale = rsqrtf(static_cast<float>(D));
    const float scale_log2 = scale * LOG2E;
    const uint32_t pfull_l = mapa_shared(smem_u32(pfull), 0);
    float m = -INFINITY, l = 0.f;  // running max (log2 units, possibly stale by < 8); this half's sum
    const uint8_t* mrow = a.key_mask ? a.key_mask + static_cast<long long>(b) * a.S : nullptr;
    const bool flags = a.softcap > 0.f || a.window > 0;
    bool ok = true;
    constexpr int HK = BK / 2;  // keys per thread per tile
    uint4 mnext[4];  // key-mask bytes of this half of the next tile, in flight while the current one is processed
    auto load_mask = [&](int kk) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4)
        mnext[v4] = (mrow && a.mask_vec && kk + 16 * v4 < a.S) ? *reinterpret_cast<const uint4*>(mrow + kk + 16 * v4)
                                                                 : make_uint4(0, 0, 0, 0);
    };
    load_mask(kb_lo * BK + HK * hf);
    for (int t = 0; t < n; ++t) {
      const int s = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      const int k0 = (kb_lo + t) * BK + HK * hf;  // this thread's first key
      // after a failed wait, skip the remaining waits and pass the barrier below with the failure
      const bool ready = ok && mbar_wait(&sfull[s], ph, a.status, kTimeoutAttention);
      __syncwarp();
      if (!__all_sync(0xffffffffu, ready)) ok = false;
      tc_fence_after();
      uint32_t sr[HK];
      if (ok) {  // the loads run while the key mask below is examined
        tmem_ld32(tmem + t_lane + Sh::S_COL + s * BK + HK * hf, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tmem_ld32(tmem + t_lane + Sh::S_COL + s * BK + HK * hf + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      }
      // Key validity for this half tile (the same for every row): bit c = key k0 + c.
      uint32_t vbits[2] = {0xffffffffu, 0xffffffffu};
      if (k0 + HK > a.S) {
        const int nvk = a.S - k0;  // may be <= 0: no key of this half exists
        vbits[0] = nvk >= 32 ? 0xffffffffu : (nvk <= 0 ? 0u : ((1u << nvk) - 1u));
        vbits[1] = nvk >= 64 ? 0xffffffffu : (nvk <= 32 ? 0u : ((1u << (nvk - 32)) - 1u));
      }
      if (mrow) {
        if (a.mask_vec) {
          // this tile's mask bytes were loaded at the end of the previous tile
          uint32_t all = 0x01010101u;
          uint4 w[4];
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            w[v4] = mnext[v4];
            all &= w[v4].x & w[v4].y & w[v4].z & w[v4].w;
          }
          if (all != 0x01010101u) {  // some key masked: build the bits (0/1 bytes)
            uint32_t bits[2] = {0u, 0u};
#pragma unroll
            for (int v4 = 0; v4 < 4; ++v4) {
              const uint32_t ww[4] = {w[v4].x, w[v4].y, w[v4].z, w[v4].w};
#pragma unroll
              for (int e = 0; e < 16; ++e)
                bits[v4 >> 1] |= (((ww[e >> 2] >> (8 * (e & 3))) & 0xffu) != 0u ? 1u : 0u) << (16 * (v4 & 1) + e);
            }
            vbits[0] &= bits[0];
            vbits[1] &= bits[1];
          }
        } else {
          for (int c = 0; c < HK; ++c)
            if (k0 + c >= a.S || !mrow[k0 + c]) vbits[c >> 5] &= ~(1u << (c & 31));
        }
      }
      if (ok) tmem_wait_ld();
      // Raw scores x (= q.k); the softmax uses x * scale_log2.  Boundary tiles
      // (masked keys, the causal diagonal, beyond-reference flags) rewrite x
      // in place; a masked entry becomes -1e30 (MASK_FILL semantics: a row
      // with no valid key averages every key).
      const bool diag = k0 + HK - 1 > qc;
      if (ok && (diag || flags || (vbits[0] & vbits[1]) != 0xffffffffu)) {
        if (a.softcap > 0.f) {  // beyond-reference flag: kept out of the hot loop below
#pragma unroll
          for (int c = 0; c < HK; ++c)
            sr[c] = __float_as_uint(a.softcap * tanhf(__uint_as_float(sr[c]) * scale / a.softcap) / scale);
        }
        const int lim = row - k0;  // keys k0 + c with c <= lim are not in the future
        const int wlo = a.window > 0 ? row - a.window + 1 - k0 : -1;  // and c >= wlo inside the window
#pragma unroll
        for (int c = 0; c < HK; ++c) {
          const bool valid = ((vbits[c >> 5] >> (c & 31)) & 1u) && c <= lim && c >= wlo;
          sr[c] = valid ? sr[c] : __float_as_uint(kMaskFill);
        }
      }
      // This half's max with 8 independent partial maxima, then the row's
      // through the partner thread (every softmax warp passes the barrier,
      // also after a failed wait, so none is left waiting).
      float pm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pm[e] = ok ? __uint_as_float(sr[e]) : kMaskFill;
#pragma unroll
      for (int c = 8; c < HK; ++c) pm[c & 7] = fmaxf(pm[c & 7], ok ? __uint_as_float(sr[c]) : kMaskFill);
      const float mh = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      xmax[(s * 2 + hf) * BQ + r] = mh;
      if (!ok && lane == 0) xfail[s] = 1;  // tile t's failures reach every softmax warp through this barrier
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
      const float mt = fmaxf(mh, xmax[(s * 2 + (hf ^ 1)) * BQ + r]);
      if (xfail[s]) {  // the same decision in all eight warps: none is left waiting at the next barrier
        ok = false;
        break;
      }
      const float mn = fmaxf(m, mt * scale_log2);
      if (t == 0) {
        m = mn;
      } else {
        const bool need = mn > m + 8.f;
        if (__any_sync(0xffffffffu, need)) {
          // O must hold P_{t-1} V_{t-1} before it is rescaled (this thread's half of its columns).
          const bool done = mbar_wait(ofull, (t - 1) & 1, a.status, kTimeoutAttention);
          __syncwarp();
          if (!__all_sync(0xffffffffu, done)) {
            ok = false;  // reported at the next tile's barrier (or the epilogue's)
            continue;
          }
          tc_fence_after();
          const float corr = ex2_approx(m - mn);
          m = mn;
          l *= corr;
#pragma unroll 1
          for (int c = (D / 2) * hf; c < (D / 2) * (hf + 1); c += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + t_lane + Sh::O_COL + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * corr);
            tmem_st32(tmem + t_lane + Sh::O_COL + c, o);
          }
          tmem_wait_st();
        }
      }
      // P = exp2(x * scale_log2 - m) as bf16 pairs: keys [64 hf, +64) of the
      // tile -> packed columns [32 hf, +32) of this S buffer
      uint32_t pw[HK / 2];
      if (m < 0.5f * kMaskFill * scale_log2) {  // every key so far masked: P = 1 (MASK_FILL's uniform average)
        const uint32_t one = pack_bf16x2(1.f, 1.f);
#pragma unroll
        for (int e = 0; e < HK / 2; ++e) pw[e] = one;
        l += static_cast<float>(HK);
      } else {
        const float neg_m = -m;
        float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial sums
#pragma unroll
        for (int e = 0; e < HK / 2; ++e) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * e]), scale_log2, neg_m));
          const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * e + 1]), scale_log2, neg_m));
          ps[(2 * e) & 7] += p0;
          ps[(2 * e + 1) & 7] += p1;
          pw[e] = pack_bf16x2(p0, p1);
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
      }
      tmem_st32(tmem + t_lane + Sh::S_COL + s * BK + (HK / 2) * hf, pw);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(pfull_l + s * 8);
      // The next tile's mask bytes: loaded only now, so that no global load
      // is in flight at the release-ordered arrive above (which would wait
      // for it); they arrive while this thread waits for the next S tile.
      if (mrow && a.mask_vec) load_mask(k0 + BK);
    }
    if (!ok) *abort_flag = 1;
    // ---------------- epilogue ----------------
    // The row sum is the two halves' sums.  Phase 1: thread (r, hf) forms
    // out = T(T(O / l) * T(sigmoid(gate))) for columns [D/2 hf, +D/2) of row
    // r and writes them into the Q buffer (free: every MMA has completed once
    // ofinal fires) in the TMA layout [atom][128 rows][128 B] with the
    // 128-byte swizzle; the gate rows come from the same layout in the K
    // stages.
    xsum[hf * BQ + r] = l;
    const bool fin = ok && mbar_wait(ofinal, 0, a.status, kTimeoutAttention);
    const bool have_gate = fin && a.gate && mbar_wait(gfull, 0, a.status, kTimeoutAttention);
    asm volatile("bar.sync 1, 256;" ::: "memory");
    const float lsum = xsum[r] + xsum[BQ + r];
    __syncwarp();
    if (__all_sync(0xffffffffu, fin && (have_gate || !a.gate))) {
      tc_fence_after();
      const float inv = 1.f / lsum;
#pragma unroll 1
      for (int c = (D / 2) * hf; c < (D / 2) * (hf + 1); c += 32) {
        uint32_t o[32];
        tmem_ld32(tmem + t_lane + Sh::O_COL + c, o);
        tmem_wait_ld();
#pragma unroll
        for (int v4 = 0; v4 < 4; ++v4) {
          const int chunk = (c >> 3) + v4;
          const uint32_t off = (chunk >> 3) * (BQ * 128) + r * 128 + (((chunk & 7) ^ (r & 7)) << 4);
          uint32_t w[4];
          if (a.gate) {
            // T(T(O / l) * T(sigmoid(gate))) on bf16 pairs: the product of two
            // bf16 values is exact in FP32, so the packed multiply rounds once
            // exactly as the scalar form
            const uint4 gq = *reinterpret_cast<const uint4*>(sK + off);
            const uint32_t gw[4] = {gq.x, gq.y, gq.z, gq.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              __nv_bfloat162 g2 = *reinterpret_cast<const __nv_bfloat162*>(&gw[e]);
              if (!a.gate_presig) {
                const float2 g = __bfloat1622float2(g2);
                g2 = __floats2bfloat162_rn(sigmoid_fast(g.x), sigmoid_fast(g.y));
              }
              const __nv_bfloat162 x2 = __floats2bfloat162_rn(__uint_as_float(o[v4 * 8 + 2 * e]) * inv,
                                                              __uint_as_float(o[v4 * 8 + 2 * e + 1]) * inv);
              const __nv_bfloat162 r2 = __hmul2(x2, g2);
              w[e] = *reinterpret_cast<const uint32_t*>(&r2);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w[e] = pack_bf16x2(__uint_as_float(o[v4 * 8 + 2 * e]) * inv, __uint_as_float(o[v4 * 8 + 2 * e + 1]) * inv);
          }
          *reinterpret_cast<uint4*>(sQ + off) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_async_smem();  // generic-proxy writes -> visible to the TMA engine
    asm volatile("bar.sync 1, 256;" ::: "memory");  // the eight softmax warps
    // Phase 2: this CTA's rows leave through TMA bulk stores when its 128-row
    // tile lies inside one sequence; otherwise through coalesced 16-byte
    // stores of its valid rows.  A CTA whose rows all lie past the sequence
    // end (the second half of a last pair) stores nothing.
    const int tid = static_cast<int>(threadIdx.x) - 64;
    if (qc < a.S) {
      if (a.tma_store) {
        if (tid == 0) {
          for (int at = 0; at < ATOMS; ++at)
            for (int half = 0; half < 2; ++half)
              tma_store_2d(&tmap_out, sQ + at * (BQ * 128) + half * (64 * 128), h * static_cast<int>(a.hso) + at * 64,
                           row_base + qc + half * 64);
          tma_store_commit();
          tma_store_wait_read();  // the staging buffer must outlive the copy
        }
      } else {
        constexpr int CPR = D / 8;
#pragma unroll 4
        for (int idx = tid; idx < BQ * CPR; idx += 256) {
          const int rr = idx / CPR, ch = idx % CPR;
          if (qc + rr >= a.S) continue;
          const uint4 ov =
              *reinterpret_cast<const uint4*>(sQ + (ch >> 3) * (BQ * 128) + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4));
          *reinterpret_cast<uint4*>(a.out + (static_cast<long long>(row_base) + qc + rr) * a.ldo +
                                    static_cast<long long>(h) * a.hso + ch * 8) = ov;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA frees tensor memory while its pair may still use it
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, Sh::TMEM_COLS);
}

}  // namespace clef

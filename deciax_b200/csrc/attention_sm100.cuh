// Causal GQA flash attention on the 5th-generation tensor cores (sm_100a).
//
// One CTA = 128 query rows of one (batch row, query head), 192 threads
// (320 at head_dim 256, see below):
//   warp 0      TMA producer: the Q tile once, then K and V in 64-key tiles
//               through two-stage rings (128-byte swizzle, no multicast).
//   warp 1      one thread issues tcgen05.mma: S_j = Q K_j^T (M=128, N=64,
//               K=D) into one of two TMEM S buffers, then O += P_{j-1} V_{j-1}
//               (M=128, N=D, K=64) into the TMEM O accumulator.  V is the
//               MN-major B operand (it is stored [keys][d]).  For D = 128, P
//               is the A operand straight from tensor memory (see below).
//   warps 2..5  softmax: thread r owns query row r.  It reads its S row from
//               TMEM, masks (key mask, causal, optional window/softcap) with
//               MASK_FILL = -1e30, keeps a running max / sum, writes
//               P = exp(s - m) as bf16 into swizzled shared memory for the
//               P.V MMA, and at the end reads O from TMEM, divides by the sum,
//               applies the sigmoid output gate and stores.
// For D >= 128 the softmax writes P back into tensor memory over the first
// BK/2 columns of its own S buffer (bf16 pairs), and the P.V MMA reads A from
// there.  At D = 128, without the two shared-memory P buffers the CTA takes
// 97 KB, so two CTAs share an SM (256 TMEM columns each) and one CTA's softmax
// overlaps the other's MMAs.  At D = 256 one CTA fills the SM: keys come in
// 128-key tiles (QK^T at N = 128), and warps 2..9 run the softmax, two per
// row (warps w and w + 4 share a TMEM lane quarter, each taking 64 keys of
// the tile and half of O's columns), exchanging their tile maxima through
// shared memory.  The next QK^T into that S buffer is issued after the P.V
// that reads it, and one thread's tcgen05.mma instructions run in order.
// The running max is only moved (and O rescaled through TMEM) when it grows
// by more than 2^8 (log2 units): between moves P is computed against a stale
// max, which the final division cancels exactly.
//
// Reference semantics: kernels/attention/blocked.py:9-32 (FP32 scores scaled
// by D^-1/2, MASK_FILL, FP32 softmax, probabilities rounded to bf16 before
// P.V, FP32 accumulation) and the output gate of qwen3_5/text.py:91.  Every
// mbarrier wait is bounded (common.cuh).
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace clef {

struct AttnTcArgs {
  int B, S, H, Hk;
  int q_col, k_col, v_col;  // column offsets (elements) of head 0 of q / k / v in the packed rows
  int g_col;                 // column offset of head 0's gate (used when gate != nullptr)
  int hsq, hsk;              // head strides (elements) of q (and gate) / k and v
  const __nv_bfloat16* gate; // gate of head 0 (row stride ldg, head stride hsq), nullable
  long long ldg;
  __nv_bfloat16* out;
  long long ldo, hso;
  const uint8_t* key_mask;  // [B, S] or nullptr
  int mask_vec;             // key_mask rows are 16-byte aligned and S % 16 == 0
  int tma_store;            // S % 128 == 0: every 128-row tile lies inside one sequence (tmap_out valid)
  int gate_presig;          // gate slots hold T(sigmoid(T(gate))) already
  float softcap;
  int window;
  int* status;
};

template <int D>
struct AttnTcShape {
  // Key tile BK: 128 at head_dim 256 (QK^T at N = 128, full rate; two 128-column
  // S buffers and the 256-column O fill the 512 tensor-memory columns, and
  // Q + one K + one V stage fill shared memory), 64 otherwise.
  static constexpr int BQ = 128, BK = D == 256 ? 128 : 64, ATOMS = D / 64;
  static constexpr int KST = D == 256 ? 1 : 2;         // K and V stages each
  static constexpr bool P_TMEM = D >= 128;             // P over its S buffer in tensor memory
  // Softmax warps per tensor-memory lane quarter: at head_dim 256 two warps
  // share each row, one per half of the 128-key tile (one CTA per SM, so the
  // softmax, which is latency-bound with one warp per scheduler, gets twice
  // the warps).
  static constexpr int NP = D == 256 ? 2 : 1;
  static constexpr int THREADS = 64 + 128 * NP;
  static constexpr uint32_t XCH_BYTES = NP > 1 ? 3 * NP * 128 * 4 : 0;  // row maxima [2][NP][128], sums [NP][128]
  static constexpr uint32_t Q_BYTES = BQ * D * 2;      // ATOMS x [128 rows x 128 B]
  static constexpr uint32_t KV_BYTES = BK * D * 2;     // ATOMS x [BK rows x 128 B]
  static constexpr uint32_t P_BYTES = BQ * BK * 2;     // [128 rows x 2 BK B]
  static constexpr uint32_t TMEM_COLS = D + 2 * BK <= 256 ? 256 : 512;
  static constexpr uint32_t S_COL = 0, O_COL = 2 * BK;  // S buffers at 0 and BK, O after them
  static constexpr size_t SMEM = 1024 + Q_BYTES + 2 * KST * KV_BYTES + (P_TMEM ? 0 : 2 * P_BYTES) + 256 + XCH_BYTES;
  static_assert(D + 2 * BK <= 512, "tensor memory");
  static_assert(Q_BYTES <= KST * KV_BYTES, "the gate tile is prefetched into the K stages");
  static_assert(P_TMEM || BK == 64, "P through shared memory is laid out for 64-key tiles");
  static_assert(NP == 1 || (P_TMEM && (BK / NP) % 64 == 0), "each softmax part writes whole 32-column P chunks");
};

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// MN-major operand tile with the 128-byte swizzle: rows of 128 B along K,
// 64-element MN blocks `lbo` bytes apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_mn128(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Barrier `id` over `n` threads that also ORs `v` across them (bar.red.or).
__device__ __forceinline__ bool bar_red_or(int id, int n, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

template <int D>
__global__ void __launch_bounds__(AttnTcShape<D>::THREADS, D == 128 ? 2 : 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap tmap_out, AttnTcArgs a) {
  using Sh = AttnTcShape<D>;
  constexpr int BQ = Sh::BQ, BK = Sh::BK, ATOMS = Sh::ATOMS, KST = Sh::KST;
  constexpr uint32_t IDESC_QK = idesc_bf16_f32(BQ, BK);
  constexpr uint32_t IDESC_PV = idesc_bf16_f32(BQ, D) | (1u << 16);  // B (V) is MN-major
  constexpr float LOG2E = 1.4426950408889634f;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Sh::Q_BYTES;          // KST stages
  uint8_t* sV = sK + KST * Sh::KV_BYTES;   // KST stages
  uint8_t* sP = sV + KST * Sh::KV_BYTES;   // 2 buffers (none when P lives in tensor memory)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + (Sh::P_TMEM ? 0 : 2 * Sh::P_BYTES));
  uint64_t* qfull = bars;
  uint64_t* kfull = bars + 1;
  uint64_t* kempty = bars + 3;
  uint64_t* vfull = bars + 5;
  uint64_t* vempty = bars + 7;
  uint64_t* sfull = bars + 9;
  uint64_t* sfree = bars + 11;
  uint64_t* pfull = bars + 13;
  uint64_t* pempty = bars + 15;
  uint64_t* ofull = bars + 17;
  uint64_t* ofinal = bars + 18;
  uint64_t* drain = bars + 19;
  uint64_t* gfull = bars + 20;  // gate tile prefetched into the K stages
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xbuf = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);  // softmax parts' exchange

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqb = (a.S + BQ - 1) / BQ;
  const int qb = nqb - 1 - static_cast<int>(blockIdx.x);  // heaviest (most keys) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.H / a.Hk);
  const int q0 = qb * BQ;
  const int kb_hi = (min(q0 + BQ, a.S) - 1) / BK + 1;
  const int kb_lo = a.window > 0 ? max(0, q0 - a.window + 1) / BK : 0;
  const int n = kb_hi - kb_lo;
  const int row_base = b * a.S;

  if (threadIdx.x == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < 21; ++i) {
      const bool softmax_arrives = (i >= 11 && i < 15);  // sfree[2], pfull[2]: one arrive per softmax thread
      mbar_init(&bars[i], softmax_arrives ? 128 * Sh::NP : 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Sh::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      mbar_arrive_expect_tx(qfull, Sh::Q_BYTES);
      for (int at = 0; at < ATOMS; ++at)
        for (int half = 0; half < 2; ++half)
          tma_load_2d(sQ + at * (BQ * 128) + half * (64 * 128), &tmap, qfull, a.q_col + h * a.hsq + at * 64,
                      row_base + q0 + half * 64);
      // K runs one tile ahead of V: a K stage frees when its QK^T is done,
      // a V stage only after the (later) P.V that reads it.  Tile i uses
      // stage i % KST in phase (i / KST) & 1; each stage is BK / 64 boxes of
      // 64 rows per 64-column atom.
      int nk = 0, nv = 0;  // tiles whose K / V load has been issued
      for (int i = 0; i <= n && !*abort_flag; ++i) {
        if (i < n) {
          const int s = i % KST;
          if (!mbar_wait(&kempty[s], ((i / KST) & 1) ^ 1, a.status, kTimeoutAttention)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&kfull[s], Sh::KV_BYTES);
          for (int at = 0; at < ATOMS; ++at)
            for (int bx = 0; bx < BK / 64; ++bx)
              tma_load_2d(sK + s * Sh::KV_BYTES + at * (BK * 128) + bx * (64 * 128), &tmap, &kfull[s],
                          a.k_col + hk * a.hsk + at * 64, row_base + (kb_lo + i) * BK + bx * 64);
          nk = i + 1;
        }
        if (i >= 1) {
          const int u = i - 1, s = u % KST;
          if (!mbar_wait(&vempty[s], ((u / KST) & 1) ^ 1, a.status, kTimeoutAttention)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&vfull[s], Sh::KV_BYTES);
          for (int at = 0; at < ATOMS; ++at)
            for (int bx = 0; bx < BK / 64; ++bx)
              tma_load_2d(sV + s * Sh::KV_BYTES + at * (BK * 128) + bx * (64 * 128), &tmap, &vfull[s],
                          a.v_col + hk * a.hsk + at * 64, row_base + (kb_lo + u) * BK + bx * 64);
          nv = u + 1;
        }
      }
      // Gate prefetch: once the last QK^T has consumed every K stage, load
      // this tile's gate rows (128 x D) into them for the epilogue.
      bool gate_issued = false;
      if (a.gate && !*abort_flag && nk == n) {
        bool free_ = true;
        for (int t = max(0, n - KST); t < n; ++t)
          free_ = free_ && mbar_wait(&kempty[t % KST], (t / KST) & 1, a.status, kTimeoutAttention);
        if (free_) {
          mbar_arrive_expect_tx(gfull, Sh::Q_BYTES);
          for (int at = 0; at < ATOMS; ++at)
            for (int half = 0; half < 2; ++half)
              tma_load_2d(sK + at * (BQ * 128) + half * (64 * 128), &tmap, gfull, a.g_col + h * a.hsq + at * 64,
                          row_base + q0 + half * 64);
          gate_issued = true;
        } else {
          *abort_flag = 1;
        }
      }
      // Every issued load must land before the CTA may exit (only the last
      // KST per ring can still be in flight: earlier stages were re-awaited).
      mbar_wait(qfull, 0, a.status, kTimeoutDrain);
      if (gate_issued) mbar_wait(gfull, 0, a.status, kTimeoutDrain);
      for (int t = max(0, nk - KST); t < nk; ++t) mbar_wait(&kfull[t % KST], (t / KST) & 1, a.status, kTimeoutDrain);
      for (int t = max(0, nv - KST); t < nv; ++t) mbar_wait(&vfull[t % KST], (t / KST) & 1, a.status, kTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int u) -> bool {
        const int s = u & 1, vs = u % KST;  // S/P buffer, V stage
        const uint32_t ph = (u >> 1) & 1;
        if (!mbar_wait(&pfull[s], ph, a.status, kTimeoutAttention) ||
            !mbar_wait(&vfull[vs], (u / KST) & 1, a.status, kTimeoutAttention))
          return false;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + vs * Sh::KV_BYTES);
        if constexpr (Sh::P_TMEM) {
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)  // 16 keys of P = 8 TMEM columns
            umma_bf16_ts(tmem + Sh::O_COL, tmem + Sh::S_COL + s * BK + kk * 8,
                         smem_desc_mn128(v_addr + kk * 16 * 128, BK * 128), IDESC_PV, (u > 0 || kk > 0) ? 1u : 0u);
        } else {
          const uint32_t p_addr = smem_u32(sP + s * Sh::P_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16(tmem + Sh::O_COL, smem_desc_k128(p_addr + kk * 32),
                      smem_desc_mn128(v_addr + kk * 16 * 128, BK * 128), IDESC_PV, (u > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&vempty[vs]);
        umma_commit(&pempty[s]);
        umma_commit(ofull);
        return true;
      };
      bool ok = mbar_wait(qfull, 0, a.status, kTimeoutAttention);
      for (int t = 0; ok && t < n && !*abort_flag; ++t) {
        const int s = t & 1, ks = t % KST;  // S buffer, K stage
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&kfull[ks], (t / KST) & 1, a.status, kTimeoutAttention) ||
            !mbar_wait(&sfree[s], ph ^ 1, a.status, kTimeoutAttention)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + ks * Sh::KV_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int at = kk >> 2, w = kk & 3;
          umma_bf16(tmem + Sh::S_COL + s * BK, smem_desc_k128(q_addr + at * (BQ * 128) + w * 32),
                    smem_desc_k128(k_addr + at * (BK * 128) + w * 32), IDESC_QK, kk > 0 ? 1u : 0u);
        }
        umma_commit(&kempty[ks]);
        umma_commit(&sfull[s]);
        if (t >= 1 && !issue_pv(t - 1)) {
          ok = false;
          break;
        }
      }
      if (ok && !*abort_flag) ok = issue_pv(n - 1);
      if (!ok) *abort_flag = 1;
      umma_commit(ofinal);
      umma_commit(drain);
      mbar_wait(drain, 0, a.status, kTimeoutDrain);
    }
  } else {
    // ---------------- softmax / epilogue warps ----------------
    // NP warps per TMEM lane quarter: part p of row r takes keys
    // [p BKP, (p + 1) BKP) of every tile and O columns [p D/NP, (p + 1) D/NP).
    // The parts exchange their tile maxima through shared memory (one
    // barrier per tile); their row sums are added once, at the end.
    constexpr int NP = Sh::NP, BKP = BK / NP, NWP = BKP / 32, NT = 128 * NP, DP = D / NP;
    const int q4 = warp & 3;  // TMEM lane quarter
    const int part = (warp - 2) >> 2;
    const int c0 = part * BKP;  // this part's first key column within a tile
    const int r = q4 * 32 + lane;
    const int row = q0 + r;
    const uint32_t t_lane = static_cast<uint32_t>(q4 * 32) << 16;
    const float scale = rsqrtf(static_cast<float>(D));
    const float scale_log2 = scale * LOG2E;
    float m = -INFINITY, l = 0.f;  // running max (log2 units, possibly stale by < 8) and this part's sum
    const uint8_t* mrow = a.key_mask ? a.key_mask + static_cast<long long>(b) * a.S : nullptr;
    const bool flags = a.softcap > 0.f || a.window > 0;
    bool ok = true;
    // A failed wait sets `fail`.  With one part a warp leaves the loop at
    // once; with several, never alone: the next tile's exchange barrier ORs
    // the flags and every part leaves together.
    bool fail = false;
    uint4 mnext[BKP / 16];  // key-mask bytes of the next tile, in flight while the current one is processed
    auto load_mask = [&](int kk) {
#pragma unroll
      for (int v4 = 0; v4 < BKP / 16; ++v4)
        mnext[v4] = (mrow && a.mask_vec && kk + c0 + 16 * v4 < a.S)
                        ? *reinterpret_cast<const uint4*>(mrow + kk + c0 + 16 * v4)
                        : make_uint4(0, 0, 0, 0);
    };
    load_mask(kb_lo * BK);
    for (int t = 0; t < n; ++t) {
      const int s = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      const int k0 = (kb_lo + t) * BK;
      if (!fail) {
        const bool ready = mbar_wait(&sfull[s], ph, a.status, kTimeoutAttention);
        __syncwarp();
        fail = !__all_sync(0xffffffffu, ready);
      }
      if constexpr (NP == 1) {
        if (fail) {
          ok = false;
          break;
        }
      }
      tc_fence_after();
      uint32_t sr[BKP];  // the loads run while the key mask below is examined
      if (!fail) {
#pragma unroll
        for (int w = 0; w < NWP; ++w)
          tmem_ld32(tmem + t_lane + Sh::S_COL + s * BK + c0 + 32 * w, *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * w]));
      }
      // Key validity for this part of the tile (the same for every row): bit cc = key k0 + c0 + cc.
      uint32_t vbits[NWP];
#pragma unroll
      for (int w = 0; w < NWP; ++w) vbits[w] = 0xffffffffu;
      if (k0 + c0 + BKP > a.S) {
        const int nv = a.S - k0 - c0;  // keys of this part that exist (may be <= 0)
#pragma unroll
        for (int w = 0; w < NWP; ++w)
          vbits[w] = nv >= 32 * (w + 1) ? 0xffffffffu : (nv <= 32 * w ? 0u : ((1u << (nv - 32 * w)) - 1u));
      }
      if (mrow) {
        if (a.mask_vec) {
          // this tile's mask bytes were loaded at the end of the previous tile
          uint32_t all = 0x01010101u;
#pragma unroll
          for (int v4 = 0; v4 < BKP / 16; ++v4) all &= mnext[v4].x & mnext[v4].y & mnext[v4].z & mnext[v4].w;
          if (all != 0x01010101u) {  // some key masked: build the bits (0/1 bytes)
            uint32_t bits[NWP];
#pragma unroll
            for (int w = 0; w < NWP; ++w) bits[w] = 0u;
#pragma unroll
            for (int v4 = 0; v4 < BKP / 16; ++v4) {
              const uint32_t ww[4] = {mnext[v4].x, mnext[v4].y, mnext[v4].z, mnext[v4].w};
#pragma unroll
              for (int e = 0; e < 16; ++e)
                bits[v4 >> 1] |= (((ww[e >> 2] >> (8 * (e & 3))) & 0xffu) != 0u ? 1u : 0u) << (16 * (v4 & 1) + e);
            }
#pragma unroll
            for (int w = 0; w < NWP; ++w) vbits[w] &= bits[w];
          }
        } else {
#pragma unroll
          for (int w = 0; w < NWP; ++w) {  // word by word: vbits stays in registers
            uint32_t bw = vbits[w];
            for (int c = 0; c < 32; ++c) {
              const int key = k0 + c0 + 32 * w + c;
              if (key >= a.S || !mrow[key]) bw &= ~(1u << c);
            }
            vbits[w] = bw;
          }
        }
      }
      if (!fail) {
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&sfree[s]);
      }
      // Raw scores x (= q.k); the softmax uses x * scale_log2.  Boundary tiles
      // (masked keys, the causal diagonal, beyond-reference flags) rewrite x
      // in place; a masked entry becomes -1e30 (MASK_FILL semantics: a row
      // with no valid key averages every key).
      const bool diag = k0 + BK - 1 > q0;
      uint32_t vall = 0xffffffffu;
#pragma unroll
      for (int w = 0; w < NWP; ++w) vall &= vbits[w];
      if (diag || flags || vall != 0xffffffffu) {
        if (a.softcap > 0.f) {  // beyond-reference flag: kept out of the hot loop below
#pragma unroll
          for (int c = 0; c < BKP; ++c)
            sr[c] = __float_as_uint(a.softcap * tanhf(__uint_as_float(sr[c]) * scale / a.softcap) / scale);
        }
        const int lim = row - k0 - c0;  // keys k0 + c0 + c with c <= lim are not in the future
        const int wlo = a.window > 0 ? row - a.window + 1 - k0 - c0 : -BK;  // and c >= wlo inside the window
#pragma unroll
        for (int c = 0; c < BKP; ++c) {
          const bool valid = ((vbits[c >> 5] >> (c & 31)) & 1u) && c <= lim && c >= wlo;
          sr[c] = valid ? sr[c] : __float_as_uint(kMaskFill);
        }
      }
      // Row max with 8 independent partial maxima (short dependency chains).
      float pm[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) pm[e] = __uint_as_float(sr[e]);
#pragma unroll
      for (int c = 8; c < BKP; ++c) pm[c & 7] = fmaxf(pm[c & 7], __uint_as_float(sr[c]));
      float mt = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      if constexpr (NP > 1) {
        // both parts of a row end with the same maximum, bit for bit
        xbuf[(s * NP + part) * 128 + r] = mt;
        if (bar_red_or(1, NT, fail)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int p = 0; p < NP; ++p) mt = fmaxf(mt, xbuf[(s * NP + p) * 128 + r]);
      }
      const float mn = fmaxf(m, mt * scale_log2);
      if (t == 0) {
        m = mn;
      } else {
        // the parts of a row see the same m and mn, so they decide alike
        const bool need = mn > m + 8.f;
        if (__any_sync(0xffffffffu, need)) {
          // O must hold P_{t-1} V_{t-1} before it is rescaled.
          const bool done = mbar_wait(ofull, (t - 1) & 1, a.status, kTimeoutAttention);
          __syncwarp();
          if (!__all_sync(0xffffffffu, done)) {
            fail = true;
            if constexpr (NP == 1) {
              ok = false;
              break;
            } else {
              continue;
            }
          }
          tc_fence_after();
          const float corr = ex2_approx(m - mn);
          m = mn;
          l *= corr;
#pragma unroll 1
          for (int c = part * DP; c < (part + 1) * DP; c += 32) {
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
      // P = exp2(x * scale_log2 - m) as bf16
      const bool pe = mbar_wait(&pempty[s], ph ^ 1, a.status, kTimeoutAttention);
      __syncwarp();
      if (!__all_sync(0xffffffffu, pe)) {
        fail = true;
        if constexpr (NP == 1) {
          ok = false;
          break;
        } else {
          continue;
        }
      }
      if constexpr (Sh::P_TMEM) {
        // P packed as bf16 pairs over the first BK/2 columns of its S buffer
        // (key j in column j/2): this part's keys in columns [c0/2, (c0 + BKP)/2)
        const bool all_masked = m < 0.5f * kMaskFill * scale_log2;  // P = 1 (see below)
        const float neg_m = -m;
        float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int w = 0; w < NWP / 2; ++w) {
          uint32_t pw[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int c = 64 * w + 2 * e;
            const float p0 = all_masked ? 1.f : ex2_approx(fmaf(__uint_as_float(sr[c]), scale_log2, neg_m));
            const float p1 = all_masked ? 1.f : ex2_approx(fmaf(__uint_as_float(sr[c + 1]), scale_log2, neg_m));
            ps[c & 7] += p0;
            ps[(c + 1) & 7] += p1;
            pw[e] = pack_bf16x2(p0, p1);
          }
          tmem_st32(tmem + t_lane + Sh::S_COL + s * BK + c0 / 2 + 32 * w, pw);
        }
        l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&pfull[s]);
        // next tile's mask bytes: loaded after the (release-ordered) arrive, so it does not wait for them
        if (mrow && a.mask_vec) load_mask(k0 + BK);
        continue;
      } else {
        // row r of the swizzled [128 x 64] P tile in shared memory (one part)
        uint8_t* prow = sP + s * Sh::P_BYTES + r * 128;
        if (m < 0.5f * kMaskFill * scale_log2) {
          // Every key so far is masked (m is the fill): each entry equals m, so
          // P = 1 -- the uniform average MASK_FILL gives.  (The FFMA below would
          // turn the rounding error of the huge product into +-inf here.)
          const uint32_t one = pack_bf16x2(1.f, 1.f);
#pragma unroll
          for (int ch = 0; ch < 8; ++ch)
            *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(one, one, one, one);
          l += 64.f;
        } else {
          const float neg_m = -m;
          float ps[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial row sums
#pragma unroll
          for (int ch = 0; ch < 8; ++ch) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float p0 = ex2_approx(fmaf(__uint_as_float(sr[ch * 8 + 2 * e]), scale_log2, neg_m));
              const float p1 = ex2_approx(fmaf(__uint_as_float(sr[ch * 8 + 2 * e + 1]), scale_log2, neg_m));
              ps[2 * e] += p0;
              ps[2 * e + 1] += p1;
              w[e] = pack_bf16x2(p0, p1);
            }
            *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
          }
          l += ((ps[0] + ps[1]) + (ps[2] + ps[3])) + ((ps[4] + ps[5]) + (ps[6] + ps[7]));
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(&pfull[s]);
        if (mrow && a.mask_vec) load_mask(k0 + BK);  // after the release-ordered arrive (see above)
      }
    }
    ok = ok && !fail;
    if (!ok) *abort_flag = 1;
    if constexpr (NP > 1) {
      // the row sum: the parts' sums, added in part order
      float* lbuf = xbuf + 2 * NP * 128;
      lbuf[part * 128 + r] = l;
      asm volatile("bar.sync 1, %0;" ::"r"(NT) : "memory");
      l = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p) l += lbuf[p * 128 + r];
    }
    // ---------------- epilogue ----------------
    // Phase 1: thread r forms its row out = T(T(O / l) * T(sigmoid(gate))) (its
    // part's columns) and writes it into the Q buffer (free: every MMA has
    // completed once ofinal fires) in the TMA layout [atom][128 rows][128 B]
    // with the 128-byte swizzle; the gate rows come from the same layout in
    // the K stages.
    const bool fin = ok && mbar_wait(ofinal, 0, a.status, kTimeoutAttention);
    const bool have_gate = fin && a.gate && mbar_wait(gfull, 0, a.status, kTimeoutAttention);
    __syncwarp();
    if (__all_sync(0xffffffffu, fin && (have_gate || !a.gate))) {
      tc_fence_after();
      const float inv = 1.f / l;
#pragma unroll 1
      for (int c = part * DP; c < (part + 1) * DP; c += 32) {
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
    asm volatile("bar.sync 1, %0;" ::"r"(NT) : "memory");  // every softmax warp
    // Phase 2: the tile leaves through TMA bulk stores when it lies inside
    // one sequence; otherwise through coalesced 16-byte stores of its valid rows.
    const int tid = static_cast<int>(threadIdx.x) - 64;
    if (a.tma_store) {
      if (tid == 0) {
        for (int at = 0; at < ATOMS; ++at)
          for (int half = 0; half < 2; ++half)
            tma_store_2d(&tmap_out, sQ + at * (BQ * 128) + half * (64 * 128), h * static_cast<int>(a.hso) + at * 64,
                         row_base + q0 + half * 64);
        tma_store_commit();
        tma_store_wait_read();  // the staging buffer must outlive the copy
      }
    } else {
      constexpr int CPR = D / 8;
#pragma unroll 4
      for (int idx = tid; idx < BQ * CPR; idx += NT) {
        const int rr = idx / CPR, ch = idx % CPR;
        if (q0 + rr >= a.S) continue;
        const uint4 ov = *reinterpret_cast<const uint4*>(sQ + (ch >> 3) * (BQ * 128) + rr * 128 + (((ch & 7) ^ (rr & 7)) << 4));
        *reinterpret_cast<uint4*>(a.out + (static_cast<long long>(row_base) + q0 + rr) * a.ldo +
                                  static_cast<long long>(h) * a.hso + ch * 8) = ov;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, Sh::TMEM_COLS);
}

}  // namespace clef

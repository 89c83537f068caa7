// libclef_b200: the B200-native Clef prefill-and-score path behind a C ABI.
//
// Host side (this file): configuration checks, weight upload with
// tensor-parallel sharding and packing, the per-shape workspace, the forward
// orchestration (embedding -> decoder layers -> final norm -> lexical means
// -> joint head) on one CUDA stream, NCCL all-reduce for TP > 1, and the
// C-ABI entry points declared in include/clef_b200.h.
//
// Device side: gemm_sm100.cuh / gemm2_sm100.cuh (tcgen05 GEMMs),
// attention_sm100.cuh (tcgen05 attention), attention.cuh, gdn.cuh (Gated
// DeltaNet), simt.cuh, head.cuh.
//
// Reference: src/deciax/models/clef/model.py:30-102 (forward loop),
// models/qwen3_5/text.py:94-102 (layer), models/qwen3_5/pallas.py:62-129 (TP
// layout: FP32 partial sums reduced before the cast), models/clef/weights.py
// (names and shard specs), models/clef/head.py (head).

#include <cudaTypedefs.h>
#include <nccl.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "../../include/clef_b200.h"
#include "attention.cuh"
#include "attention_sm100.cuh"
#include "common.cuh"
#include "gemm_sm100.cuh"
#include "gemm2_sm100.cuh"
#include "gdn.cuh"
#include "gdn_tc.cuh"
#include "tp.cuh"
#include "head.cuh"
#include "simt.cuh"

using bf16 = __nv_bfloat16;

namespace clef {

// ===========================================================================
// errors
// ===========================================================================

struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CUDA_CHECK(expr)                                                                                 \
  do {                                                                                                   \
    cudaError_t e_ = (expr);                                                                             \
    if (e_ != cudaSuccess) throw ::clef::Error(CLEF_ECUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)
#define NCCL_CHECK(expr)                                                                                   \
  do {                                                                                                     \
    ncclResult_t r_ = (expr);                                                                              \
    if (r_ != ncclSuccess) throw ::clef::Error(CLEF_ENCCL, std::string(#expr) + ": " + ncclGetErrorString(r_)); \
  } while (0)
#define REQUIRE(cond, msg)                                  \
  do {                                                      \
    if (!(cond)) throw ::clef::Error(CLEF_EINVAL, (msg));   \
  } while (0)

static std::mutex g_error_mutex;
static std::string g_last_error;

static void set_global_error(const std::string& m) {
  std::lock_guard<std::mutex> lock(g_error_mutex);
  g_last_error = m;
}

// qk_norm_rope_kernel runs eight warps per block, each staging one head row
// of head_dim floats in dynamic shared memory: 8 * head_dim * 4 bytes must
// fit the default 48 KB.
constexpr int kQkRopeMaxHeadDim = 48 * 1024 / (8 * 4);

// ===========================================================================
// host bf16 helpers
// ===========================================================================

static inline uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40);  // NaN
  const uint32_t rounding = 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>((u + rounding) >> 16);
}
static inline float bf16_bits_to_f32(uint16_t h) {
  const uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ===========================================================================
// device properties, TMA descriptor encoding
// ===========================================================================

static int sm_count(int device) {
  static std::mutex mu;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(device);
  if (it != cache.end()) return it->second;
  int n = 0;
  CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  cache[device] = n;
  return n;
}

static int current_device() {
  int d = 0;
  CUDA_CHECK(cudaGetDevice(&d));
  return d;
}

static PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) throw Error(CLEF_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  return fn;
}

// Row-major bf16 [rows, cols] with row stride ld elements; box 64 columns x box_rows, 128-byte swizzle.
static CUtensorMap tmap_bf16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(CLEF_EINVAL, "cuTensorMapEncodeTiled rejected a GEMM operand");
  return m;
}

// bf16 rows of `states` sequences of `seq` tokens, row stride ld elements, as a
// [state][token][column] tensor: box 64 columns x box_rows tokens of one state,
// 128-byte swizzle; tokens past a sequence's end read zero.
static CUtensorMap tmap_bf16_states(const void* ptr, uint64_t states, uint64_t seq, uint64_t ld, uint32_t box_rows) {
  CUtensorMap m;
  cuuint64_t dims[3] = {ld, seq, states};
  cuuint64_t strides[2] = {ld * 2, seq * ld * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = tma_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box, es,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw Error(CLEF_EINVAL, "cuTensorMapEncodeTiled rejected the Gated DeltaNet conv rows");
  return m;
}

// ===========================================================================
// kernel launchers
// ===========================================================================

// Kernel categories for the per-kernel timing report (clef_timing_report).
enum Category : int {
  kCatEmbed = 0,
  kCatNorm = 1,
  kCatGemmQkv = 2,
  kCatQkRope = 3,
  kCatAttention = 4,
  kCatGemmO = 5,
  kCatGemmGateUp = 6,
  kCatGemmDown = 7,
  kCatAllReduce = 8,
  kCatResidual = 9,
  kCatHead = 10,
  kCatOther = 11,
  kCatGdn = 12,
  kNumCategories = 13,
};

// Optional CUDA-event timeline: one event after every launch on the stream,
// so launch i's device time is the gap between event i-1 and event i.
struct Timeline {
  bool enabled = false;
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<int> cats;
  cudaEvent_t next() {
    if (used == pool.size()) {
      cudaEvent_t e;
      CUDA_CHECK(cudaEventCreate(&e));
      pool.push_back(e);
    }
    return pool[used++];
  }
  ~Timeline() {
    for (auto e : pool) cudaEventDestroy(e);
  }
};

// NVTX range for profilers (Nsight Systems / Compute): forward, layer, mixer,
// MLP and head spans on the host timeline, around the kernels they launch.
// Without a profiler attached the push / pop are no-op calls.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

struct Launcher {
  cudaStream_t stream = nullptr;
  int* status = nullptr;
  int count = 0;        // kernels of this library launched
  int cat = kCatOther;  // category of the next launch
  Timeline* timeline = nullptr;
  void mark(int c) {
    if (timeline && timeline->enabled) {
      CUDA_CHECK(cudaEventRecord(timeline->next(), stream));
      timeline->cats.push_back(c);
    }
  }
  void tick() {
    ++count;
    mark(cat);
  }
};

template <int BN, int EPI>
static void launch_tc_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, cudaStream_t st) {
  using S = GemmShape<BN>;
  // The dynamic shared-memory limit is a per-device function attribute.
  static std::mutex mu;
  static std::set<int> done;
  const int dev = current_device();
  {
    std::lock_guard<std::mutex> lock(mu);
    if (!done.count(dev)) {
      CUDA_CHECK(cudaFuncSetAttribute(gemm_bf16_sm100<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(S::SMEM)));
      done.insert(dev);
    }
  }
  const int tiles = ((args.M + S::BM - 1) / S::BM) * ((args.N + BN - 1) / BN);
  const int grid = std::min(tiles, sm_count(dev));
  gemm_bf16_sm100<BN, EPI><<<grid, 192, S::SMEM, st>>>(ta, tb, args);
  CUDA_CHECK(cudaGetLastError());
}

// Launch the CTA-pair GEMM: clusters of 2, as many as can be resident at once
// (TPR: with the fused tensor-parallel reduction and its four extra warps).
template <int EPI, bool TPR = false>
static void launch_tc_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const GemmArgs& args, cudaStream_t st,
                                const TpFuse& tpf = TpFuse{}) {
  using S = Gemm2Shape;
  auto kern = gemm_bf16_sm100_pair<EPI, TPR>;
  static std::mutex mu;
  static std::map<int, int> max_clusters;
  const int dev = current_device();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(TPR ? 192 + 32 * kTpReduceWarps : 192);
  cfg.dynamicSmemBytes = S::SMEM;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = max_clusters.find(dev);
    if (it == max_clusters.end()) {
      CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(S::SMEM)));
      cfg.gridDim = dim3(2 * sm_count(dev) / 2);
      int n = 0;
      CUDA_CHECK(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      REQUIRE(n > 0, "no CTA-pair cluster fits on this device");
      it = max_clusters.emplace(dev, n).first;
    }
    clusters = it->second;
  }
  const int tiles = ((args.M + S::BM - 1) / S::BM) * ((args.N + S::BN - 1) / S::BN);
  cfg.gridDim = dim3(2 * std::min(tiles, clusters));
  CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, args, tpf));
}

// bf16 GEMM on tcgen05.  A [M, K] (lda), B [N, K] (ldb).  Large problems run
// on CTA pairs (256x256 tiles); small ones on single CTAs.
static void gemm_bf16(Launcher& L, int epi, const bf16* A, int lda, const bf16* B, int ldb, int M, int N, int K,
                      void* out, int ldo, const bf16* bias, const bf16* res, int ldr) {
  REQUIRE(M > 0 && N > 0 && K > 0, "GEMM dimensions must be positive");
  REQUIRE(K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0, "bf16 GEMM needs K and operand strides multiple of 8");
  REQUIRE(aligned16(A) && aligned16(B) && aligned16(out), "bf16 GEMM operands must be 16-byte aligned");
  REQUIRE(epi == kEpiF32 ? ldo % 4 == 0 : ldo % 8 == 0, "GEMM output stride must keep 16-byte rows");
  if (epi == kEpiResidual) REQUIRE(res && aligned16(res) && ldr % 8 == 0, "residual operand must be aligned");
  if (epi == kEpiSwiglu) REQUIRE(N % 256 == 0, "SwiGLU GEMM needs N = 2F with F a multiple of 128");
  GemmArgs args{M, N, K, out, ldo, bias, res, ldr, L.status};
  if (M >= 256 && N >= 256) {
    const CUtensorMap ta = tmap_bf16(A, M, K, lda, 128);
    const CUtensorMap tb = tmap_bf16(B, N, K, ldb, 128);
    switch (epi) {
      case kEpiStore: launch_tc_gemm_pair<kEpiStore>(ta, tb, args, L.stream); break;
      case kEpiSwiglu: launch_tc_gemm_pair<kEpiSwiglu>(ta, tb, args, L.stream); break;
      case kEpiResidual: launch_tc_gemm_pair<kEpiResidual>(ta, tb, args, L.stream); break;
      case kEpiF32: launch_tc_gemm_pair<kEpiF32>(ta, tb, args, L.stream); break;
      default: throw Error(CLEF_EINVAL, "bad GEMM epilogue");
    }
    L.tick();
    return;
  }
  const bool narrow = N <= 128 && epi != kEpiSwiglu;
  const int bn = narrow ? 128 : 256;
  const CUtensorMap ta = tmap_bf16(A, M, K, lda, 128);
  const CUtensorMap tb = tmap_bf16(B, N, K, ldb, bn);
  if (narrow) {
    switch (epi) {
      case kEpiStore: launch_tc_gemm<128, kEpiStore>(ta, tb, args, L.stream); break;
      case kEpiResidual: launch_tc_gemm<128, kEpiResidual>(ta, tb, args, L.stream); break;
      case kEpiF32: launch_tc_gemm<128, kEpiF32>(ta, tb, args, L.stream); break;
      default: throw Error(CLEF_EINVAL, "bad GEMM epilogue");
    }
  } else {
    switch (epi) {
      case kEpiStore: launch_tc_gemm<256, kEpiStore>(ta, tb, args, L.stream); break;
      case kEpiSwiglu: launch_tc_gemm<256, kEpiSwiglu>(ta, tb, args, L.stream); break;
      case kEpiResidual: launch_tc_gemm<256, kEpiResidual>(ta, tb, args, L.stream); break;
      case kEpiF32: launch_tc_gemm<256, kEpiF32>(ta, tb, args, L.stream); break;
      default: throw Error(CLEF_EINVAL, "bad GEMM epilogue");
    }
  }
  L.tick();
}

// Parameters of the fused QKV epilogue (q/k-norm + partial RoPE, sigmoid of the gate).
struct QkvFusion {
  const bf16* q_norm;
  const bf16* k_norm;
  const float* rope_cos;
  const float* rope_sin;
  int hq, hkv, head_dim, rot, seq;
  float eps;
};

// Whether the QKV projection can carry the fused epilogue: every 256-column
// tile must hold whole heads and the rotated half must be whole 32-column chunks.
static bool qkv_fusable(int head_dim, int rot) {
  return (head_dim == 64 || head_dim == 128 || head_dim == 256) && (rot % 64 == 0 || rot == 32);
}

static void gemm_bf16_qkv(Launcher& L, const bf16* A, int lda, const bf16* B, int ldb, int M, int N, int K, bf16* out,
                          int ldo, const QkvFusion& f) {
  REQUIRE(M > 0 && N > 0 && K > 0, "GEMM dimensions must be positive");
  REQUIRE(K % 8 == 0 && lda % 8 == 0 && ldb % 8 == 0 && ldo % 8 == 0, "bf16 GEMM needs strides multiple of 8");
  REQUIRE(aligned16(A) && aligned16(B) && aligned16(out), "bf16 GEMM operands must be 16-byte aligned");
  REQUIRE(qkv_fusable(f.head_dim, f.rot),
          "fused QKV epilogue needs head_dim in {64,128,256} and a rotary dimension of 32 or a multiple of 64");
  REQUIRE(N == f.hq * 2 * f.head_dim + 2 * f.hkv * f.head_dim, "fused QKV epilogue: N does not match the heads");
  GemmArgs args{M, N, K, out, ldo, nullptr, nullptr, 0, L.status, f.q_norm, f.k_norm, f.rope_cos, f.rope_sin,
                f.hq, f.hkv, f.head_dim, f.rot, f.seq, f.eps};
  const CUtensorMap ta = tmap_bf16(A, M, K, lda, 128);
  if (M >= 256 && N >= 256) {
    const CUtensorMap tb = tmap_bf16(B, N, K, ldb, 128);
    launch_tc_gemm_pair<kEpiQkv>(ta, tb, args, L.stream);
  } else {
    const CUtensorMap tb = tmap_bf16(B, N, K, ldb, 256);
    launch_tc_gemm<256, kEpiQkv>(ta, tb, args, L.stream);
  }
  L.tick();
}

template <typename T>
static void gemm_simt(Launcher& L, int epi, const T* A, int lda, const T* B, int ldb, int M, int N, int K, void* out,
                      int ldo, const T* bias, const T* res, int ldr) {
  REQUIRE(M > 0 && N > 0 && K > 0, "GEMM dimensions must be positive");
  SimtGemmArgs<T> a{A, lda, B, ldb, M, N, K, bias, res, ldr, out, ldo};
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  switch (epi) {
    case kSimtStore: simt_gemm<T, kSimtStore><<<grid, 256, 0, L.stream>>>(a); break;
    case kSimtGelu: simt_gemm<T, kSimtGelu><<<grid, 256, 0, L.stream>>>(a); break;
    case kSimtResidual: simt_gemm<T, kSimtResidual><<<grid, 256, 0, L.stream>>>(a); break;
    case kSimtF32: simt_gemm<T, kSimtF32><<<grid, 256, 0, L.stream>>>(a); break;
    default: throw Error(CLEF_EINVAL, "bad GEMM epilogue");
  }
  CUDA_CHECK(cudaGetLastError());
  L.tick();
}

template <typename T>
static void rmsnorm(Launcher& L, const T* x, int ldx, const T* w, T* out, int ldo, int rows, int dim, float eps,
                    const uint8_t* row_mask = nullptr) {
  if constexpr (sizeof(T) == 2) {
    if (dim % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0 && dim <= kRmsSmemMaxDim && aligned16(x) && aligned16(w) &&
        aligned16(out)) {
      const size_t smem = static_cast<size_t>(kRmsSmemRows) * dim * 2;  // one staged row per warp
      if (smem > 48 * 1024)
        CUDA_CHECK(cudaFuncSetAttribute(rmsnorm_bf16_smem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)));
      rmsnorm_bf16_smem_kernel<<<(rows + kRmsSmemRows - 1) / kRmsSmemRows, 32 * kRmsSmemRows, smem, L.stream>>>(
          x, ldx, w, out, ldo, rows, dim, eps, row_mask);
      CUDA_CHECK(cudaGetLastError());
      L.tick();
      return;
    }
  }
  const int warps = 8;
  rmsnorm_kernel<T><<<(rows + warps - 1) / warps, warps * 32, 0, L.stream>>>(x, ldx, w, out, ldo, rows, dim, eps,
                                                                            row_mask);
  CUDA_CHECK(cudaGetLastError());
  L.tick();
}

template <typename T, int DH>
static void launch_gdn_dh(Launcher& L, const GdnArgs& a) {
  const size_t smem = GdnShape<DH>::bytes;
  CUDA_CHECK(cudaFuncSetAttribute(gdn_chunk_kernel<T, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(smem)));
  gdn_chunk_kernel<T, DH><<<dim3(a.nv, a.B), kGdnThreads, smem, L.stream>>>(a);
  CUDA_CHECK(cudaGetLastError());
  L.tick();
}

// One CTA per (state, value head); the head dim is a template parameter.
template <typename T>
static void launch_gdn(Launcher& L, const GdnArgs& a, int dh) {
  REQUIRE(a.B > 0 && a.S > 0 && a.nh > 0 && a.nv > 0 && a.nv % a.nh == 0, "bad Gated DeltaNet shape");
  REQUIRE(a.width >= 1 && a.width <= 8, "linear_conv_kernel_dim must be 1..8");
  REQUIRE(a.B <= 65535, "too many states");
  switch (dh) {
    case 8: launch_gdn_dh<T, 8>(L, a); break;
    case 16: launch_gdn_dh<T, 16>(L, a); break;
    case 32: launch_gdn_dh<T, 32>(L, a); break;
    case 64: launch_gdn_dh<T, 64>(L, a); break;
    case 128:
      if constexpr (sizeof(T) == 2) {
        // bf16 activations at head dim 128: conv pass, prep pass, chain pass
        // (tensor cores: TF32 / BF16 products, FP32 state and solve)
        static std::mutex mu;
        static std::set<int> done;
        {
          std::lock_guard<std::mutex> lock(mu);
          if (!done.count(current_device())) {
            CUDA_CHECK(cudaFuncSetAttribute(gdn_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(GdnPrepShape::SMEM)));
            CUDA_CHECK(cudaFuncSetAttribute(gdn_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(GdnChainShape::SMEM)));
            done.insert(current_device());
          }
        }
        REQUIRE(a.qkv_conv != nullptr && a.prep != nullptr && a.a0_tiles != nullptr && a.v_tiles != nullptr &&
                    a.ldc >= 2LL * a.nh * 128,
                "the tensor-core Gated DeltaNet path needs its scratch (gdn_tc_bind_scratch)");
        REQUIRE(reinterpret_cast<uintptr_t>(a.qkv_conv) % 16 == 0 && reinterpret_cast<uintptr_t>(a.prep) % 16 == 0 &&
                    reinterpret_cast<uintptr_t>(a.a0_tiles) % 16 == 0 && reinterpret_cast<uintptr_t>(a.v_tiles) % 16 == 0,
                "Gated DeltaNet scratch must be 16-byte aligned");
        const int span = kGdnChunk * kGdnConvBlocks;
        const dim3 cgrid((a.S + span - 1) / span, 2 * a.nh + a.nv, a.B);
        if (a.width <= 4)
          gdn_conv_bf16_kernel<4><<<cgrid, kGdnThreads, 0, L.stream>>>(a);
        else
          gdn_conv_bf16_kernel<8><<<cgrid, kGdnThreads, 0, L.stream>>>(a);
        CUDA_CHECK(cudaGetLastError());
        L.tick();
        const int chunks = (a.S + kGdnChunk - 1) / kGdnChunk;
        const CUtensorMap qk_map = tmap_bf16_states(a.qkv_conv, a.B, a.S, a.ldc, kGdnChunk);
        gdn_prep_kernel<<<dim3(chunks, a.nh, a.B), kGdnThreads, GdnPrepShape::SMEM, L.stream>>>(qk_map, a);
        CUDA_CHECK(cudaGetLastError());
        L.tick();
        gdn_chain_kernel<<<dim3(a.nv, a.B), kGdnThreads, GdnChainShape::SMEM, L.stream>>>(a);
        CUDA_CHECK(cudaGetLastError());
        L.tick();
      } else {
        launch_gdn_dh<T, 128>(L, a);
      }
      break;
    default: throw Error(CLEF_EINVAL, "Gated DeltaNet head dim must be one of 8, 16, 32, 64, 128");
  }
}

template <typename T>
static void layernorm(Launcher& L, const T* x, const T* w, const T* b, T* out, int rows, int dim) {
  const int warps = 8;
  layernorm_kernel<T><<<(rows + warps - 1) / warps, warps * 32, 0, L.stream>>>(x, w, b, out, rows, dim, 1e-5f);
  CUDA_CHECK(cudaGetLastError());
  L.tick();
}

template <typename T>
static void attention(Launcher& L, const AttnArgs<T>& a) {
  REQUIRE(a.hd > 0 && a.hd <= 256, "attention head size must be in [1, 256]");
  REQUIRE(a.Hk > 0 && a.H % a.Hk == 0, "query heads must be a multiple of key/value heads");
  bool done = false;
  if constexpr (sizeof(T) == 2) {
    // tcgen05 flash attention over the packed QKV projection
    const long long kc = a.k - a.q, vc = a.v - a.q;
    const bool tc_ok = a.packed && a.causal && (a.hd == 64 || a.hd == 128 || a.hd == 256) && a.Lq == a.Lk &&
                       a.ldq == a.ldk && a.ldk == a.ldv && a.hsk == a.hsv && a.ldq % 8 == 0 && a.hsq % 64 == 0 &&
                       a.hsk % 64 == 0 && kc % 64 == 0 && vc % 64 == 0 && aligned16(a.q) && a.ldo % 8 == 0 &&
                       a.hso % 8 == 0 &&
                       (!a.gate || (a.ldg == a.ldq && a.hsg == a.hsq && (a.gate - a.q) % 64 == 0 && a.gate > a.q));
    if (tc_ok) {
      AttnTcArgs t{};
      t.B = a.B;
      t.S = a.Lq;
      t.H = a.H;
      t.Hk = a.Hk;
      t.q_col = 0;
      t.k_col = static_cast<int>(kc);
      t.v_col = static_cast<int>(vc);
      t.g_col = a.gate ? static_cast<int>(a.gate - a.q) : 0;
      t.hsq = static_cast<int>(a.hsq);
      t.hsk = static_cast<int>(a.hsk);
      t.gate = a.gate;
      t.ldg = a.ldg;
      t.out = a.out;
      t.ldo = a.ldo;
      t.hso = a.hso;
      t.key_mask = a.key_mask;
      t.mask_vec = a.key_mask && aligned16(a.key_mask) && a.Lk % 16 == 0;
      t.gate_presig = a.gate_presig;
      t.softcap = a.softcap;
      t.window = a.window;
      t.status = a.status;
      const CUtensorMap map = tmap_bf16(a.q, static_cast<uint64_t>(a.B) * a.Lq, a.ldq, a.ldq, 64);
      // Output through TMA bulk stores when every 128-row tile stays inside one sequence.
      t.tma_store = a.Lq % 128 == 0 && aligned16(a.out) && a.hso % 64 == 0;
      const CUtensorMap out_map =
          t.tma_store ? tmap_bf16(a.out, static_cast<uint64_t>(a.B) * a.Lq, a.ldo, a.ldo, 64) : map;
      dim3 grid((a.Lq + 127) / 128, a.H, a.B);
      static std::mutex mu_tc;
      static std::set<std::pair<int, int>> done_tc;
      const int dev = current_device();
      auto launch = [&](auto kern, size_t smem, int hd, int threads) {
        {
          std::lock_guard<std::mutex> lock(mu_tc);
          if (!done_tc.count({dev, hd})) {
            CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
            done_tc.insert({dev, hd});
          }
        }
        kern<<<grid, threads, smem, L.stream>>>(map, out_map, t);
      };
      if (a.hd == 64) {
        launch(attn_tc_kernel<64>, AttnTcShape<64>::SMEM, 64, AttnTcShape<64>::THREADS);
      } else if (a.hd == 128) {
        launch(attn_tc_kernel<128>, AttnTcShape<128>::SMEM, 128, AttnTcShape<128>::THREADS);
      } else {
        launch(attn_tc_kernel<256>, AttnTcShape<256>::SMEM, 256, AttnTcShape<256>::THREADS);
      }
      done = true;
    }
  }
  if constexpr (sizeof(T) == 2) {
    const bool vec_ok = a.ldq % 8 == 0 && a.ldk % 8 == 0 && a.ldv % 8 == 0 && a.hsq % 8 == 0 && a.hsk % 8 == 0 &&
                        a.hsv % 8 == 0 && aligned16(a.q) && aligned16(a.k) && aligned16(a.v) && a.ldo % 2 == 0 &&
                        a.hso % 2 == 0 && (!a.gate || (a.ldg % 2 == 0 && a.hsg % 2 == 0));
    if (!done && vec_ok && (a.hd == 64 || a.hd == 128 || a.hd == 256)) {
      dim3 grid((a.Lq + 63) / 64, a.H, a.B);
      static std::mutex mu;
      static std::set<std::pair<int, int>> done_attr;
      const int dev = current_device();
      auto set_attr = [&](auto kern, size_t smem, int hd) {
        std::lock_guard<std::mutex> lock(mu);
        if (!done_attr.count({dev, hd})) {
          CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
          done_attr.insert({dev, hd});
        }
      };
      if (a.hd == 64) {
        set_attr(attn_fa2_bf16_kernel<64>, Fa2Shape<64>::SMEM, 64);
        attn_fa2_bf16_kernel<64><<<grid, 128, Fa2Shape<64>::SMEM, L.stream>>>(a);
      } else if (a.hd == 128) {
        set_attr(attn_fa2_bf16_kernel<128>, Fa2Shape<128>::SMEM, 128);
        attn_fa2_bf16_kernel<128><<<grid, 128, Fa2Shape<128>::SMEM, L.stream>>>(a);
      } else {
        set_attr(attn_fa2_bf16_kernel<256>, Fa2Shape<256>::SMEM, 256);
        attn_fa2_bf16_kernel<256><<<grid, 128, Fa2Shape<256>::SMEM, L.stream>>>(a);
      }
      done = true;
    }
  }
  if (!done) {
    dim3 grid((a.Lq + 3) / 4, a.H, a.B);
    attn_simt_kernel<T><<<grid, 128, 4 * a.hd * sizeof(float), L.stream>>>(a);
  }
  CUDA_CHECK(cudaGetLastError());
  L.tick();
}

// RoPE tables [max_s, rot/2]: inv_freq = 1 / theta^(2i/rot) in float32 (nn.py:31-32),
// angle = float32(pos) * inv_freq in float32, then cos/sin of that float.
static void rope_tables(int max_s, int rot, float theta, std::vector<float>& cos_t, std::vector<float>& sin_t) {
  const int half = rot / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) {
    const float e = static_cast<float>(2 * i) / static_cast<float>(rot);
    inv[i] = 1.0f / powf(theta, e);
  }
  cos_t.resize(static_cast<size_t>(max_s) * half);
  sin_t.resize(static_cast<size_t>(max_s) * half);
  for (int p = 0; p < max_s; ++p)
    for (int i = 0; i < half; ++i) {
      const float f = static_cast<float>(p) * inv[i];
      cos_t[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(static_cast<double>(f)));
      sin_t[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(static_cast<double>(f)));
    }
}

// ===========================================================================
// device memory
// ===========================================================================

struct DBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  DBuf(DBuf&& o) noexcept : p(o.p), bytes(o.bytes) {
    o.p = nullptr;
    o.bytes = 0;
  }
  DBuf& operator=(DBuf&& o) noexcept {
    if (this != &o) {
      release();
      p = o.p;
      bytes = o.bytes;
      o.p = nullptr;
      o.bytes = 0;
    }
    return *this;
  }
  ~DBuf() { release(); }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  void alloc(size_t n) {
    release();
    if (n == 0) return;
    CUDA_CHECK(cudaMalloc(&p, n));
    bytes = n;
  }
  void ensure(size_t n) {
    if (n > bytes) alloc(n);
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(p);
  }
};

// A head / top-level tensor uploaded as-is (replicated).
struct Tensor {
  std::vector<int64_t> shape;
  DBuf buf;
  int64_t numel() const {
    int64_t n = 1;
    for (auto s : shape) n *= s;
    return n;
  }
};

struct Layer {
  DBuf w_in, w_post, q_norm, k_norm;
  DBuf w_qkv;   // [Nqkv_local, D]: q_proj (Hq_l x 2d, q|gate per head), k_proj, v_proj rows
  DBuf w_o;     // [D, Hq_l*d]
  DBuf w_gu;    // [2*Fp, D]: 256-row blocks of [128 gate rows | 128 up rows]
  DBuf w_down;  // [D, Fp]
  // linear_attention (Gated DeltaNet) layers
  DBuf g_proj;     // [Ng_pad, D]: q (nh_l*dh), k (nh_l*dh), v (nv_l*dh), z (nv_l*dh), a (nv_l), b (nv_l) rows, zero pad
  DBuf g_conv;     // [Cg, width]: q, k, v conv rows (projection column order)
  DBuf g_alog, g_dtb;  // [nv_l]
  DBuf g_norm;     // [dh]
  DBuf g_out;      // [D, nv_l*dh]
  std::set<std::string> have;
};

// ===========================================================================
// model
// ===========================================================================

struct Workspace {
  int b = 0, s = 0, lx = 0, o = 0, q = 0;
  DBuf ints, bytes;  // staged batch arrays (device)
  DBuf x, h, qkv, attn, gu, act, partial, gproj;
  DBuf gconv;  // Gated DeltaNet tensor-core scratch (bf16, head dim 128): conv rows [T, (2 nh_l + nv_l) dh], prep records
  DBuf tp_flags;  // TP: tile flags of the fused GEMM + reduction (peers write them)
  DBuf memory, mnorm, kv;
  DBuf gv, questions, contexts, lexical;
  DBuf small;  // head buffers of size b*max(o,q)*max(W,FF,4W)
  DBuf f32small;
  DBuf host_pinned;  // pinned staging for the host-buffer forward
  size_t pinned_bytes = 0;
};

struct Model {
  ClefConfig cfg{};
  std::vector<int32_t> layer_types, layer_window;
  int device = 0, rank = 0, tp = 1, dtype = CLEF_DTYPE_BF16;
  int esz = 2;
  int D = 0, F = 0, Hq = 0, Hkv = 0, d = 0, L = 0, V = 0;
  int Hq_l = 0, Hkv_l = 0, F_l = 0, Fp = 0, Nqkv = 0, rot = 0;
  int W = 0, HH = 0, RL = 0, HL = 0, FF = 0;
  // Gated DeltaNet dims (global / this rank) and packed projection layout
  int g_nh = 0, g_nv = 0, g_dh = 0, g_width = 0, g_nh_l = 0, g_nv_l = 0, Ng = 0, Ng_pad = 0, Cg = 0;
  bool any_linear = false;
  // BF16 Gated DeltaNet at head dim 128 runs the tensor-core kernel after a separate conv pass
  bool gdn_conv_pass() const { return dtype == CLEF_DTYPE_BF16 && g_dh == 128; }
  bool finalized = false;
  std::string last_error;
  cudaStream_t stream = nullptr;
  ncclComm_t comm = nullptr;
  int tp_timeout_ms = 0;  // longest host wait for the other TP ranks, 0 = no limit
  int debug_flags = 0;    // CLEF_DEBUG_*
  bool broken = false;    // a TP wait ran out: a collective may still wait on the stream
  DBuf status;  // int
  DBuf embedding, lm_head, final_norm, rope_cos, rope_sin;
  std::set<std::string> top_have;
  std::vector<Layer> layers;
  std::map<std::string, Tensor> head;
  Workspace ws;
  Timeline timeline;
  int last_launches = 0;
  int64_t ws_allocations = 0;  // workspace growths: device buffers, pinned staging, TP peer-handle exchanges
  bool src_on_device = false;  // clef_upload_device: the source pointer is device memory

  // Sum each category's device time over the recorded timeline, then reset it.
  void timing_report(int n, float* ms, int* launches) {
    for (int i = 0; i < n; ++i) {
      ms[i] = 0.f;
      launches[i] = 0;
    }
    if (timeline.used > 0) CUDA_CHECK(cudaEventSynchronize(timeline.pool[timeline.used - 1]));
    for (size_t i = 1; i < timeline.used; ++i) {
      const int c = timeline.cats[i];
      if (c < 0 || c >= n) continue;
      float t = 0.f;
      CUDA_CHECK(cudaEventElapsedTime(&t, timeline.pool[i - 1], timeline.pool[i]));
      ms[c] += t;
      launches[c] += 1;
    }
    timeline.used = 0;
    timeline.cats.clear();
  }

  // Peer pointers of the TP workspace (CUDA IPC): every rank's FP32 partial
  // and residual stream, refreshed whenever the local buffers move.
  void* ipc_part_src = nullptr;
  void* ipc_x_src = nullptr;
  void* ipc_flags_src = nullptr;
  std::vector<void*> peer_part, peer_x, peer_flags;
  unsigned tp_epoch = 0;  // launches of the fused GEMM + reduction so far (the same on every rank)
  DBuf ipc_scratch, barrier_buf;
  bool p2p = false;  // peer pointers valid: TP reduction through tp_reduce_residual_kernel

  void close_peers() {
    for (int k = 0; k < static_cast<int>(peer_part.size()); ++k) {
      if (k == rank) continue;
      if (peer_part[k]) cudaIpcCloseMemHandle(peer_part[k]);
      if (peer_x[k]) cudaIpcCloseMemHandle(peer_x[k]);
      if (k < static_cast<int>(peer_flags.size()) && peer_flags[k]) cudaIpcCloseMemHandle(peer_flags[k]);
    }
    peer_part.assign(tp, nullptr);
    peer_x.assign(tp, nullptr);
    peer_flags.assign(tp, nullptr);
    p2p = false;
  }

  // Milliseconds since t0.
  static double since_ms(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  }

  // The communicator is non-blocking, so that a rank that never joins cannot
  // hold this one forever: a call may return ncclInProgress while NCCL sets
  // up (or enqueues) in the background.  Poll until it is done, so that the
  // work enqueued after it stays ordered behind it, or until tp_timeout_ms.
  void nccl_done(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return;
    if (r != ncclInProgress) throw Error(CLEF_ENCCL, std::string(what) + ": " + ncclGetErrorString(r));
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      ncclResult_t st = ncclInProgress;
      const ncclResult_t q = ncclCommGetAsyncError(comm, &st);
      if (q != ncclSuccess) st = q;
      if (st == ncclSuccess) return;
      if (st != ncclInProgress) {
        broken = true;
        throw Error(CLEF_ENCCL, std::string(what) + ": " + ncclGetErrorString(st));
      }
      if (tp_timeout_ms > 0 && since_ms(t0) > tp_timeout_ms) {
        broken = true;
        throw Error(CLEF_ENCCL, std::string(what) + ": the other tensor-parallel ranks did not take part within " +
                                    std::to_string(tp_timeout_ms) + " ms");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
  }

  // Create the TP communicator (non-blocking).  If not every rank joins
  // within tp_timeout_ms the half-made communicator is aborted -- nothing of
  // it is on a stream yet -- and the call fails with CLEF_ENCCL.
  void create_comm(const ncclUniqueId& id) {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    const ncclResult_t r = ncclCommInitRankConfig(&comm, tp, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
      if (comm) ncclCommAbort(comm);
      comm = nullptr;
      throw Error(CLEF_ENCCL, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
    }
    try {
      nccl_done(r, "ncclCommInitRankConfig");
    } catch (const Error& e) {
      ncclCommAbort(comm);
      comm = nullptr;
      broken = false;
      throw Error(CLEF_ENCCL, std::string("tensor-parallel communicator of ") + std::to_string(tp) +
                                  " ranks not formed (rank " + std::to_string(rank) + "): " + e.what());
    }
  }

  // Host wait for the forward on `stream`.  With TP and a deadline, poll the
  // stream instead of blocking in it: a rank that skipped its forward leaves
  // this rank's collective waiting, and the caller gets CLEF_ENCCL instead of
  // a hang.  The handle is then unusable (the collective still waits on the
  // stream; only the end of the process releases it).
  void wait_stream() {
    if (tp <= 1 || tp_timeout_ms <= 0) {
      CUDA_CHECK(cudaStreamSynchronize(stream));
      return;
    }
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      const cudaError_t e = cudaStreamQuery(stream);
      if (e == cudaSuccess) return;
      if (e != cudaErrorNotReady) CUDA_CHECK(e);
      ncclResult_t st = ncclSuccess;
      if (ncclCommGetAsyncError(comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
        broken = true;
        throw Error(CLEF_ENCCL, std::string("tensor-parallel collective failed: ") + ncclGetErrorString(st));
      }
      if (since_ms(t0) > tp_timeout_ms) {
        broken = true;
        throw Error(CLEF_ENCCL, "tensor-parallel forward did not finish within " + std::to_string(tp_timeout_ms) +
                                    " ms: another rank did not take part in a collective; this handle is unusable");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }

  // Collective over the TP group: all ranks call it with the same buffer sizes.
  void exchange_ipc() {
    close_peers();
    cudaIpcMemHandle_t h[3];
    CUDA_CHECK(cudaIpcGetMemHandle(&h[0], ws.partial.p));
    CUDA_CHECK(cudaIpcGetMemHandle(&h[1], ws.x.p));
    CUDA_CHECK(cudaIpcGetMemHandle(&h[2], ws.tp_flags.p));
    const size_t hb = sizeof(h);
    ipc_scratch.ensure(static_cast<size_t>(tp) * hb);
    uint8_t* d = ipc_scratch.as<uint8_t>();
    CUDA_CHECK(cudaMemcpyAsync(d + rank * hb, h, hb, cudaMemcpyHostToDevice, stream));
    nccl_done(ncclAllGather(d + rank * hb, d, hb, ncclUint8, comm, stream), "ncclAllGather");
    std::vector<uint8_t> all(static_cast<size_t>(tp) * hb);
    CUDA_CHECK(cudaMemcpyAsync(all.data(), d, all.size(), cudaMemcpyDeviceToHost, stream));
    wait_stream();
    for (int k = 0; k < tp; ++k) {
      if (k == rank) {
        peer_part[k] = ws.partial.p;
        peer_x[k] = ws.x.p;
        peer_flags[k] = ws.tp_flags.p;
        continue;
      }
      cudaIpcMemHandle_t hk[3];
      std::memcpy(hk, all.data() + k * hb, hb);
      CUDA_CHECK(cudaIpcOpenMemHandle(&peer_part[k], hk[0], cudaIpcMemLazyEnablePeerAccess));
      CUDA_CHECK(cudaIpcOpenMemHandle(&peer_x[k], hk[1], cudaIpcMemLazyEnablePeerAccess));
      CUDA_CHECK(cudaIpcOpenMemHandle(&peer_flags[k], hk[2], cudaIpcMemLazyEnablePeerAccess));
    }
    ipc_part_src = ws.partial.p;
    ipc_x_src = ws.x.p;
    ipc_flags_src = ws.tp_flags.p;
    p2p = true;
  }

  // Every rank of the TP group has reached this point of its stream.
  void tp_barrier(Launcher& Lc) {
    nccl_done(ncclAllReduce(barrier_buf.p, barrier_buf.p, 1, ncclFloat32, ncclSum, comm, Lc.stream), "ncclAllReduce");
  }

  ~Model() {
    if (tp > 1) close_peers();
    if (comm) {
      // non-blocking communicator: flush, wait (bounded by tp_timeout_ms), free;
      // abort it instead if it does not quiesce in time
      const ncclResult_t r = ncclCommFinalize(comm);
      bool done = r == ncclSuccess;
      if (r == ncclInProgress) {
        const auto t0 = std::chrono::steady_clock::now();
        for (;;) {
          ncclResult_t st = ncclInProgress;
          if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) break;
          if (st != ncclInProgress) {
            done = st == ncclSuccess;
            break;
          }
          if (tp_timeout_ms > 0 && since_ms(t0) > tp_timeout_ms) break;
          std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
      }
      if (done)
        ncclCommDestroy(comm);
      else
        ncclCommAbort(comm);
    }
    if (stream) cudaStreamDestroy(stream);
  }

  size_t act_bytes(size_t n) const { return n * esz; }

  // -------------------------------------------------------------------------
  // creation
  // -------------------------------------------------------------------------

  void init(const ClefConfig& c, int dev, int tp_rank, int tp_size, const uint8_t* nccl_id, int dt) {
    REQUIRE(dt == CLEF_DTYPE_BF16 || dt == CLEF_DTYPE_F32, "dtype must be CLEF_DTYPE_BF16 or CLEF_DTYPE_F32");
    REQUIRE(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, "bad tensor-parallel rank/size");
    cfg = c;
    device = dev;
    rank = tp_rank;
    tp = tp_size;
    tp_timeout_ms = c.tp_timeout_ms > 0 ? c.tp_timeout_ms : 0;
    dtype = dt;
    esz = dt == CLEF_DTYPE_BF16 ? 2 : 4;
    D = c.hidden_size;
    F = c.intermediate_size;
    Hq = c.num_attention_heads;
    Hkv = c.num_key_value_heads;
    d = c.head_dim;
    L = c.num_layers;
    V = c.vocab_size;
    W = c.head_width;
    HH = c.head_heads;
    RL = c.head_routing_layers;
    HL = c.head_layers;
    FF = c.head_ffn;
    // TextConfig validation (models/qwen3_5/config.py:26-49)
    REQUIRE(D > 0 && F > 0 && Hq > 0 && Hkv > 0 && d > 0 && L > 0 && V > 0, "Qwen3.5 dimensions must be positive");
    REQUIRE(Hq % Hkv == 0, "Qwen3.5 query/value heads must divide into key head groups");
    rot = static_cast<int>(d * c.partial_rotary_factor);
    REQUIRE(rot > 0 && rot % 2 == 0 && rot <= d, "invalid partial rotary dimension");
    REQUIRE(c.max_seq_len > 0, "max_seq_len must be positive");
    REQUIRE(W > 0 && HH > 0 && W % HH == 0 && W / HH <= 256 && FF > 0 && RL >= 0 && HL >= 0, "invalid joint head config");
    layer_types.assign(L, CLEF_LAYER_FULL_ATTENTION);
    layer_window.assign(L, 0);
    for (int i = 0; i < L; ++i) {
      if (c.layer_types) layer_types[i] = c.layer_types[i];
      if (c.layer_window) layer_window[i] = c.layer_window[i];
      REQUIRE(layer_types[i] == CLEF_LAYER_FULL_ATTENTION || layer_types[i] == CLEF_LAYER_LINEAR_ATTENTION,
              "unsupported Qwen3.5 layer types");
      REQUIRE(layer_window[i] >= 0, "window must be >= 0");
    }
    cfg.layer_types = nullptr;
    cfg.layer_window = nullptr;
    // TP divisibility (the reference shards heads and MLP rows evenly, weights.py:60-67)
    REQUIRE(Hq % tp == 0 && Hkv % tp == 0 && F % tp == 0, "heads and intermediate size must divide by tp");
    REQUIRE(D % 8 == 0 && d % 8 == 0, "hidden size and head_dim must be multiples of 8");
    REQUIRE(d <= kQkRopeMaxHeadDim, "head_dim must be at most 1536");
    Hq_l = Hq / tp;
    Hkv_l = Hkv / tp;
    F_l = F / tp;
    Fp = (F_l + 127) / 128 * 128;
    Nqkv = Hq_l * 2 * d + 2 * Hkv_l * d;
    for (int i = 0; i < L; ++i) any_linear |= layer_types[i] == CLEF_LAYER_LINEAR_ATTENTION;
    if (any_linear) {
      g_nh = c.linear_num_key_heads;
      g_nv = c.linear_num_value_heads;
      g_dh = c.linear_key_head_dim;
      g_width = c.linear_conv_kernel_dim;
      REQUIRE(g_nh > 0 && g_nv > 0 && g_dh > 0 && c.linear_value_head_dim > 0 && g_width > 0,
              "Qwen3.5 dimensions must be positive");
      REQUIRE(g_nv % g_nh == 0, "Qwen3.5 query/value heads must divide into key head groups");
      REQUIRE(c.linear_value_head_dim == g_dh && (g_dh == 8 || g_dh == 16 || g_dh == 32 || g_dh == 64 || g_dh == 128),
              "Gated DeltaNet needs linear_key_head_dim == linear_value_head_dim in {8, 16, 32, 64, 128}");
      REQUIRE(g_width <= 8, "linear_conv_kernel_dim must be at most 8");
      // heads shard evenly across TP ranks (qwen3_5/pallas.py:84-90)
      REQUIRE(g_nh % tp == 0 && g_nv % tp == 0, "linear attention heads must divide by tp");
      g_nh_l = g_nh / tp;
      g_nv_l = g_nv / tp;
      Cg = 2 * g_nh_l * g_dh + g_nv_l * g_dh;
      Ng = Cg + g_nv_l * g_dh + 2 * g_nv_l;
      Ng_pad = (Ng + 15) / 16 * 16;
    }

    CUDA_CHECK(cudaSetDevice(device));
    CUDA_CHECK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
    status.alloc(sizeof(int));
    CUDA_CHECK(cudaMemset(status.p, 0, sizeof(int)));
    if (tp > 1) {
      REQUIRE(nccl_id != nullptr, "tp > 1 needs an NCCL unique id");
      ncclUniqueId id;
      std::memcpy(&id, nccl_id, sizeof(id));
      create_comm(id);
      barrier_buf.alloc(256);
      CUDA_CHECK(cudaMemset(barrier_buf.p, 0, 256));
    }
    embedding.alloc(static_cast<size_t>(V) * D * esz);
    lm_head.alloc(static_cast<size_t>(V) * D * esz);
    final_norm.alloc(static_cast<size_t>(D) * esz);
    layers.resize(L);
    for (int li = 0; li < L; ++li) {
      Layer& l = layers[li];
      l.w_in.alloc(static_cast<size_t>(D) * esz);
      l.w_post.alloc(static_cast<size_t>(D) * esz);
      if (layer_types[li] == CLEF_LAYER_LINEAR_ATTENTION) {
        l.g_proj.alloc(static_cast<size_t>(Ng_pad) * D * esz);
        CUDA_CHECK(cudaMemset(l.g_proj.p, 0, l.g_proj.bytes));
        l.g_conv.alloc(static_cast<size_t>(Cg) * g_width * esz);
        l.g_alog.alloc(static_cast<size_t>(g_nv_l) * esz);
        l.g_dtb.alloc(static_cast<size_t>(g_nv_l) * esz);
        l.g_norm.alloc(static_cast<size_t>(g_dh) * esz);
        l.g_out.alloc(static_cast<size_t>(D) * g_nv_l * g_dh * esz);
      } else {
        l.q_norm.alloc(static_cast<size_t>(d) * esz);
        l.k_norm.alloc(static_cast<size_t>(d) * esz);
        l.w_qkv.alloc(static_cast<size_t>(Nqkv) * D * esz);
        l.w_o.alloc(static_cast<size_t>(D) * Hq_l * d * esz);
      }
      l.w_gu.alloc(static_cast<size_t>(2) * Fp * D * esz);
      l.w_down.alloc(static_cast<size_t>(D) * Fp * esz);
      CUDA_CHECK(cudaMemset(l.w_gu.p, 0, l.w_gu.bytes));
      CUDA_CHECK(cudaMemset(l.w_down.p, 0, l.w_down.bytes));
    }
    std::vector<float> cs, sn;
    rope_tables(c.max_seq_len, rot, c.rope_theta, cs, sn);
    rope_cos.alloc(cs.size() * 4);
    rope_sin.alloc(sn.size() * 4);
    CUDA_CHECK(cudaMemcpy(rope_cos.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(rope_sin.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
  }

  // -------------------------------------------------------------------------
  // upload
  // -------------------------------------------------------------------------

  // Convert `count` host values to the compute dtype into `dst` (host bytes).
  void convert(const void* src, int src_dtype, size_t count, std::vector<uint8_t>& dst) const {
    dst.resize(count * esz);
    if (src_dtype == CLEF_DTYPE_F32) {
      const float* s = static_cast<const float*>(src);
      if (dtype == CLEF_DTYPE_F32) {
        std::memcpy(dst.data(), s, count * 4);
      } else {
        uint16_t* o = reinterpret_cast<uint16_t*>(dst.data());
        for (size_t i = 0; i < count; ++i) o[i] = f32_to_bf16_bits(s[i]);
      }
    } else {
      const uint16_t* s = static_cast<const uint16_t*>(src);
      if (dtype == CLEF_DTYPE_BF16) {
        std::memcpy(dst.data(), s, count * 2);
      } else {
        float* o = reinterpret_cast<float*>(dst.data());
        for (size_t i = 0; i < count; ++i) o[i] = bf16_bits_to_f32(s[i]);
      }
    }
  }

  // Copy rows [r0, r0+nrows) x cols [c0, c0+ncols) of a host [rows, cols] matrix
  // into device rows starting at dst_row of a [*, dst_ld] matrix, converting dtype.
  void put_block(const void* host, int host_dtype, int64_t cols, int64_t r0, int64_t nrows, int64_t c0, int64_t ncols,
                 void* dev, int64_t dst_row, int64_t dst_ld) {
    if (src_on_device) {
      REQUIRE(host_dtype == dtype, "a device-resident upload must already be in the compute dtype");
      CUDA_CHECK(cudaMemcpy2D(static_cast<uint8_t*>(dev) + static_cast<size_t>(dst_row) * dst_ld * esz, dst_ld * esz,
                              static_cast<const uint8_t*>(host) + (static_cast<size_t>(r0) * cols + c0) * esz, cols * esz,
                              ncols * esz, nrows, cudaMemcpyDeviceToDevice));
      return;
    }
    const size_t hsz = host_dtype == CLEF_DTYPE_F32 ? 4 : 2;
    std::vector<uint8_t> tmp;
    std::vector<uint8_t> rowbuf;
    if (c0 == 0 && ncols == cols && dst_ld == cols) {
      convert(static_cast<const uint8_t*>(host) + static_cast<size_t>(r0) * cols * hsz, host_dtype,
              static_cast<size_t>(nrows) * cols, tmp);
      CUDA_CHECK(cudaMemcpy(static_cast<uint8_t*>(dev) + static_cast<size_t>(dst_row) * dst_ld * esz, tmp.data(),
                            tmp.size(), cudaMemcpyHostToDevice));
      return;
    }
    for (int64_t r = 0; r < nrows; ++r) {
      convert(static_cast<const uint8_t*>(host) + (static_cast<size_t>(r0 + r) * cols + c0) * hsz, host_dtype,
              static_cast<size_t>(ncols), rowbuf);
      tmp.insert(tmp.end(), rowbuf.begin(), rowbuf.end());
    }
    CUDA_CHECK(cudaMemcpy2D(static_cast<uint8_t*>(dev) + static_cast<size_t>(dst_row) * dst_ld * esz, dst_ld * esz,
                            tmp.data(), ncols * esz, ncols * esz, nrows, cudaMemcpyHostToDevice));
  }

  static void expect_shape(const std::string& name, const int64_t* shape, int ndim, std::vector<int64_t> want) {
    bool ok = static_cast<int>(want.size()) == ndim;
    for (int i = 0; ok && i < ndim; ++i) ok = shape[i] == want[i];
    if (!ok) {
      std::string m = "shape mismatch for " + name + ": expected [";
      for (size_t i = 0; i < want.size(); ++i) m += (i ? "," : "") + std::to_string(want[i]);
      m += "], got [";
      for (int i = 0; i < ndim; ++i) m += (i ? "," : "") + std::to_string(shape[i]);
      throw Error(CLEF_EINVAL, m + "]");
    }
  }

  // Gated DeltaNet tensors of one layer, sharded by heads (models/clef/weights.py:43-67):
  // q/k rows by key heads, v/z/a/b rows and out_proj columns by value heads.
  // Accepts the split names of weights.py:43-57 and the checkpoint's fused
  // in_proj_qkv / conv1d tensors.
  void upload_gdn(const std::string& name, const std::string& key, Layer& l, const void* host, int host_dtype,
                  const int64_t* shape, int ndim) {
    const int64_t dh = g_dh, nk = static_cast<int64_t>(g_nh) * dh, nk_l = static_cast<int64_t>(g_nh_l) * dh;
    const int64_t nvd = static_cast<int64_t>(g_nv) * dh, nvd_l = static_cast<int64_t>(g_nv_l) * dh;
    const int64_t z0 = Cg, a0 = Cg + nvd_l, b0 = a0 + g_nv_l;
    // rows [src0 + rank*n, +n) of a [*, cols] host tensor into rows dst0.. of a packed device matrix
    auto rows = [&](int64_t cols, int64_t src0, int64_t n, DBuf& dst, int64_t dst0) {
      put_block(host, host_dtype, cols, src0 + rank * n, n, 0, cols, dst.p, dst0, cols);
    };
    if (key == "q.weight" || key == "k.weight") {
      expect_shape(name, shape, ndim, {nk, D});
      rows(D, 0, nk_l, l.g_proj, key[0] == 'q' ? 0 : nk_l);
    } else if (key == "v.weight" || key == "in_proj_z.weight") {
      expect_shape(name, shape, ndim, {nvd, D});
      rows(D, 0, nvd_l, l.g_proj, key[0] == 'v' ? 2 * nk_l : z0);
    } else if (key == "in_proj_a.weight" || key == "in_proj_b.weight") {
      expect_shape(name, shape, ndim, {g_nv, D});
      rows(D, 0, g_nv_l, l.g_proj, key[8] == 'a' ? a0 : b0);
    } else if (key == "in_proj_qkv.weight") {
      expect_shape(name, shape, ndim, {2 * nk + nvd, D});
      rows(D, 0, nk_l, l.g_proj, 0);
      rows(D, nk, nk_l, l.g_proj, nk_l);
      rows(D, 2 * nk, nvd_l, l.g_proj, 2 * nk_l);
      for (const char* k : {"q.weight", "k.weight", "v.weight"}) l.have.insert(std::string("mixer.") + k);
    } else if (key == "q.conv" || key == "k.conv") {
      expect_shape(name, shape, ndim, {nk, g_width});
      rows(g_width, 0, nk_l, l.g_conv, key[0] == 'q' ? 0 : nk_l);
    } else if (key == "v.conv") {
      expect_shape(name, shape, ndim, {nvd, g_width});
      rows(g_width, 0, nvd_l, l.g_conv, 2 * nk_l);
    } else if (key == "conv1d.weight") {
      expect_shape(name, shape, ndim, {2 * nk + nvd, 1, g_width});
      rows(g_width, 0, nk_l, l.g_conv, 0);
      rows(g_width, nk, nk_l, l.g_conv, nk_l);
      rows(g_width, 2 * nk, nvd_l, l.g_conv, 2 * nk_l);
      for (const char* k : {"q.conv", "k.conv", "v.conv"}) l.have.insert(std::string("mixer.") + k);
    } else if (key == "A_log" || key == "dt_bias") {
      expect_shape(name, shape, ndim, {g_nv});
      put_block(host, host_dtype, g_nv, 0, 1, static_cast<int64_t>(rank) * g_nv_l, g_nv_l,
                (key[0] == 'A' ? l.g_alog : l.g_dtb).p, 0, g_nv_l);
    } else if (key == "norm.weight") {
      expect_shape(name, shape, ndim, {dh});
      put_block(host, host_dtype, dh, 0, 1, 0, dh, l.g_norm.p, 0, dh);
    } else if (key == "out_proj.weight") {
      expect_shape(name, shape, ndim, {D, nvd});
      put_block(host, host_dtype, nvd, 0, D, rank * nvd_l, nvd_l, l.g_out.p, 0, nvd_l);
    } else {
      throw Error(CLEF_EINVAL, "unexpected backbone tensor: " + name);
    }
  }

  void upload(const std::string& name, const void* host, int host_dtype, const int64_t* shape, int ndim) {
    REQUIRE(!finalized, "clef_upload after clef_finalize");
    REQUIRE(host != nullptr, "null host pointer");
    REQUIRE(host_dtype == CLEF_DTYPE_F32 || host_dtype == CLEF_DTYPE_BF16, "host dtype must be F32 or BF16");
    CUDA_CHECK(cudaSetDevice(device));
    if (name == "embedding" || name == "lm_head") {
      expect_shape(name, shape, ndim, {V, D});
      put_block(host, host_dtype, D, 0, V, 0, D, (name == "embedding" ? embedding : lm_head).p, 0, D);
      top_have.insert(name);
      return;
    }
    if (name == "norm") {
      expect_shape(name, shape, ndim, {D});
      put_block(host, host_dtype, D, 0, 1, 0, D, final_norm.p, 0, D);
      top_have.insert(name);
      return;
    }
    if (name.rfind("head.", 0) == 0) {
      Tensor& t = head[name.substr(5)];
      t.shape.assign(shape, shape + ndim);
      const int64_t n = t.numel();
      if (src_on_device) {
        REQUIRE(host_dtype == dtype, "a device-resident upload must already be in the compute dtype");
        t.buf.alloc(std::max<size_t>(static_cast<size_t>(n) * esz, 16));
        CUDA_CHECK(cudaMemcpy(t.buf.p, host, static_cast<size_t>(n) * esz, cudaMemcpyDeviceToDevice));
        return;
      }
      std::vector<uint8_t> tmp;
      convert(host, host_dtype, static_cast<size_t>(n), tmp);
      t.buf.alloc(std::max<size_t>(tmp.size(), 16));
      CUDA_CHECK(cudaMemcpy(t.buf.p, tmp.data(), tmp.size(), cudaMemcpyHostToDevice));
      return;
    }
    if (name.rfind("layers.", 0) == 0) {
      const size_t dot = name.find('.', 7);
      REQUIRE(dot != std::string::npos, "bad layer tensor name: " + name);
      const int li = std::stoi(name.substr(7, dot - 7));
      REQUIRE(li >= 0 && li < L, "layer index out of range: " + name);
      const std::string key = name.substr(dot + 1);
      Layer& l = layers[li];
      const int64_t qrows = static_cast<int64_t>(Hq_l) * 2 * d, krows = static_cast<int64_t>(Hkv_l) * d;
      if (layer_types[li] == CLEF_LAYER_LINEAR_ATTENTION && key.rfind("mixer.", 0) == 0) {
        upload_gdn(name, key.substr(6), l, host, host_dtype, shape, ndim);
        l.have.insert(key);
        return;
      }
      if (key == "input_layernorm.weight" || key == "post_attention_layernorm.weight") {
        expect_shape(name, shape, ndim, {D});
        put_block(host, host_dtype, D, 0, 1, 0, D, (key[0] == 'i' ? l.w_in : l.w_post).p, 0, D);
      } else if (key == "mixer.q_norm.weight" || key == "mixer.k_norm.weight") {
        expect_shape(name, shape, ndim, {d});
        put_block(host, host_dtype, d, 0, 1, 0, d, (key[6] == 'q' ? l.q_norm : l.k_norm).p, 0, d);
      } else if (key == "mixer.q_proj.weight") {
        expect_shape(name, shape, ndim, {static_cast<int64_t>(Hq) * 2 * d, D});
        put_block(host, host_dtype, D, rank * qrows, qrows, 0, D, l.w_qkv.p, 0, D);
      } else if (key == "mixer.k_proj.weight") {
        expect_shape(name, shape, ndim, {static_cast<int64_t>(Hkv) * d, D});
        put_block(host, host_dtype, D, rank * krows, krows, 0, D, l.w_qkv.p, qrows, D);
      } else if (key == "mixer.v_proj.weight") {
        expect_shape(name, shape, ndim, {static_cast<int64_t>(Hkv) * d, D});
        put_block(host, host_dtype, D, rank * krows, krows, 0, D, l.w_qkv.p, qrows + krows, D);
      } else if (key == "mixer.o_proj.weight") {
        const int64_t in_l = static_cast<int64_t>(Hq_l) * d;
        expect_shape(name, shape, ndim, {D, static_cast<int64_t>(Hq) * d});
        put_block(host, host_dtype, static_cast<int64_t>(Hq) * d, 0, D, rank * in_l, in_l, l.w_o.p, 0, in_l);
      } else if (key == "mlp.gate_proj.weight" || key == "mlp.up_proj.weight") {
        expect_shape(name, shape, ndim, {F, D});
        const int64_t off = key[4] == 'g' ? 0 : 128;
        for (int64_t j0 = 0; j0 < F_l; j0 += 128) {
          const int64_t n = std::min<int64_t>(128, F_l - j0);
          put_block(host, host_dtype, D, rank * static_cast<int64_t>(F_l) + j0, n, 0, D, l.w_gu.p, (j0 / 128) * 256 + off,
                    D);
        }
      } else if (key == "mlp.down_proj.weight") {
        expect_shape(name, shape, ndim, {D, F});
        put_block(host, host_dtype, F, 0, D, static_cast<int64_t>(rank) * F_l, F_l, l.w_down.p, 0, Fp);
      } else {
        throw Error(CLEF_EINVAL, "unexpected backbone tensor: " + name);
      }
      l.have.insert(key);
      return;
    }
    throw Error(CLEF_EINVAL, "unexpected tensor name: " + name);
  }

  // -------------------------------------------------------------------------
  // finalize: every tensor present, head shapes consistent
  // -------------------------------------------------------------------------

  const Tensor& h(const std::string& k) const {
    auto it = head.find(k);
    if (it == head.end()) throw Error(CLEF_EINVAL, "missing joint head tensor: " + k);
    return it->second;
  }
  const Tensor* h_opt(const std::string& k) const {
    auto it = head.find(k);
    return it == head.end() ? nullptr : &it->second;
  }
  void head_shape(const std::string& k, std::vector<int64_t> want) const {
    const Tensor& t = h(k);
    expect_shape("head." + k, t.shape.data(), static_cast<int>(t.shape.size()), want);
  }

  void finalize() {
    for (const char* k : {"embedding", "lm_head", "norm"})
      REQUIRE(top_have.count(k), std::string("incomplete Clef text checkpoint: missing ") + k);
    const char* keys[] = {"input_layernorm.weight", "post_attention_layernorm.weight", "mixer.q_norm.weight",
                          "mixer.k_norm.weight",    "mixer.q_proj.weight",            "mixer.k_proj.weight",
                          "mixer.v_proj.weight",    "mixer.o_proj.weight",            "mlp.gate_proj.weight",
                          "mlp.up_proj.weight",     "mlp.down_proj.weight"};
    const char* gdn_keys[] = {"input_layernorm.weight", "post_attention_layernorm.weight", "mixer.q.weight",
                              "mixer.k.weight",         "mixer.v.weight",                  "mixer.in_proj_z.weight",
                              "mixer.in_proj_a.weight", "mixer.in_proj_b.weight",          "mixer.q.conv",
                              "mixer.k.conv",           "mixer.v.conv",                    "mixer.A_log",
                              "mixer.dt_bias",          "mixer.norm.weight",               "mixer.out_proj.weight",
                              "mlp.gate_proj.weight",   "mlp.up_proj.weight",              "mlp.down_proj.weight"};
    for (int i = 0; i < L; ++i) {
      if (layer_types[i] == CLEF_LAYER_LINEAR_ATTENTION) {
        for (const char* k : gdn_keys)
          REQUIRE(layers[i].have.count(k), "incomplete Clef text checkpoint: layers." + std::to_string(i) + "." + k);
      } else {
        for (const char* k : keys)
          REQUIRE(layers[i].have.count(k), "incomplete Clef text checkpoint: layers." + std::to_string(i) + "." + k);
      }
    }
    auto ln = [&](const std::string& n, int64_t dim) {
      head_shape(n + ".weight", {dim});
      head_shape(n + ".bias", {dim});
    };
    ln("hidden_norm", D);
    for (const char* n : {"memory_projection", "question_projection", "option_question_projection", "global_projection",
                          "option_context_projection", "option_lexical_projection"})
      head_shape(std::string(n) + ".weight", {W, D});
    REQUIRE(h("type_embedding.weight").shape.size() == 2 && h("type_embedding.weight").shape[1] == W,
            "head.type_embedding.weight must be [types, W]");
    auto mha = [&](const std::string& n) {
      head_shape(n + ".in_proj_weight", {3 * W, W});
      head_shape(n + ".in_proj_bias", {3 * W});
      head_shape(n + ".out_proj.weight", {W, W});
      head_shape(n + ".out_proj.bias", {W});
    };
    for (int i = 0; i < RL; ++i) {
      const std::string n = "evidence_layers." + std::to_string(i);
      ln(n + ".query_norm", W);
      ln(n + ".memory_norm", W);
      ln(n + ".feedforward_norm", W);
      mha(n + ".attention");
      head_shape(n + ".feedforward.0.weight", {FF, W});
      head_shape(n + ".feedforward.0.bias", {FF});
      head_shape(n + ".feedforward.3.weight", {W, FF});
      head_shape(n + ".feedforward.3.bias", {W});
    }
    ln("option_summary_norm", W);
    for (int i = 0; i < HL; ++i) {
      const std::string n = "layers." + std::to_string(i);
      mha(n + ".self_attn");
      mha(n + ".multihead_attn");
      ln(n + ".norm1", W);
      ln(n + ".norm2", W);
      ln(n + ".norm3", W);
      head_shape(n + ".linear1.weight", {FF, W});
      head_shape(n + ".linear1.bias", {FF});
      head_shape(n + ".linear2.weight", {W, FF});
      head_shape(n + ".linear2.bias", {W});
    }
    ln("field_norm", W);
    ln("option_norm", W);
    head_shape("residual_scorer.0.weight", {W, 4 * W});
    head_shape("residual_scorer.0.bias", {W});
    head_shape("residual_scorer.3.weight", {1, W});
    head_shape("residual_scorer.3.bias", {1});
    for (const char* n : {"prior_logit_scale", "joint_logit_scale", "residual_gate"})
      REQUIRE(h(n).numel() == 1, std::string("head.") + n + " must be a scalar");
    finalized = true;
  }

  // -------------------------------------------------------------------------
  // workspace
  // -------------------------------------------------------------------------

  size_t batch_int_count(int b, int s, int lx, int o, int q) const {
    return static_cast<size_t>(b) * s + static_cast<size_t>(b) * lx + static_cast<size_t>(b) * o * 2 +
           static_cast<size_t>(b) * q * 2 + static_cast<size_t>(b) * q + static_cast<size_t>(b) * o * 2 +
           static_cast<size_t>(b) * o;
  }
  size_t batch_byte_count(int b, int s, int o, int q) const {
    return static_cast<size_t>(b) * s + static_cast<size_t>(b) * q + static_cast<size_t>(b) * o;
  }

  // Grow a workspace buffer to at least n bytes, counting the allocation.
  void grow(DBuf& buf, size_t n) {
    if (n <= buf.bytes) return;
    buf.alloc(n);
    ++ws_allocations;
  }

  // Pinned host staging of a host forward: the batch arrays and the logits.
  void grow_pinned(size_t need) {
    Workspace& w = ws;
    if (w.pinned_bytes >= need) return;
    if (w.host_pinned.p) {
      cudaFreeHost(w.host_pinned.p);
      w.host_pinned.p = nullptr;
      w.pinned_bytes = 0;
    }
    CUDA_CHECK(cudaMallocHost(&w.host_pinned.p, need));
    w.pinned_bytes = need;
    ++ws_allocations;
  }

  size_t pinned_need(int b, int s, int lx, int o, int q) const {
    return batch_int_count(b, s, lx, o, q) * 4 + batch_byte_count(b, s, o, q) + static_cast<size_t>(b) * o * 4 + 64;
  }

  void reserve(int b, int s, int lx, int o, int q) {
    REQUIRE(b > 0 && s > 0 && lx > 0 && o > 0 && q > 0, "batch dimensions must be positive");
    REQUIRE(s <= cfg.max_seq_len, "sequence length exceeds max_seq_len");
    CUDA_CHECK(cudaSetDevice(device));
    Workspace& w = ws;
    const size_t T = static_cast<size_t>(b) * s;
    grow(w.ints, batch_int_count(b, s, lx, o, q) * 4 + 64);
    grow(w.bytes, batch_byte_count(b, s, o, q) + 64);
    grow(w.x, act_bytes(T * D));
    grow(w.h, act_bytes(T * D));
    grow(w.qkv, act_bytes(T * Nqkv));
    grow(w.attn, act_bytes(T * std::max(Hq_l * d, g_nv_l * g_dh)));
    if (any_linear) grow(w.gproj, act_bytes(T * Ng_pad));
    if (any_linear && gdn_conv_pass()) grow(w.gconv, gdn_tc_scratch_bytes(b, s, g_nh_l, g_nv_l));
    if (dtype == CLEF_DTYPE_F32) grow(w.gu, act_bytes(T * 2 * Fp));
    grow(w.act, act_bytes(T * Fp));
    if (tp > 1) {
      grow(w.partial, T * D * 4);
      // [tiles of 256 x 256][2 CTAs][4 warps][tp] flags of gemm_bf16_sm100_pair<kEpiF32, true>
      const size_t fb = ((T + 255) / 256) * ((static_cast<size_t>(D) + 255) / 256) * 8 * tp * 4;
      if (fb > w.tp_flags.bytes) {
        grow(w.tp_flags, fb);
        // on the stream, before the handle exchange that lets peers write here
        CUDA_CHECK(cudaMemsetAsync(w.tp_flags.p, 0, fb, stream));
      }
    }
    grow(w.memory, act_bytes(T * W));
    grow(w.mnorm, act_bytes(T * W));
    grow(w.kv, act_bytes(T * 2 * W));
    grow(w.gv, act_bytes(static_cast<size_t>(b) * D));
    grow(w.questions, act_bytes(static_cast<size_t>(b) * q * D));
    grow(w.contexts, act_bytes(static_cast<size_t>(b) * o * D));
    grow(w.lexical, act_bytes(static_cast<size_t>(b) * o * D));
    const size_t rows = static_cast<size_t>(b) * std::max(o, q);
    const size_t widest = std::max<size_t>({static_cast<size_t>(3 * W), static_cast<size_t>(FF), static_cast<size_t>(4 * W)});
    grow(w.small, act_bytes(rows * widest * 12 + static_cast<size_t>(b) * W * 2) + 16 * 64);
    grow(w.f32small, static_cast<size_t>(b) * o * 4 * 4 + 256);
    w.b = std::max(w.b, b);
    w.s = std::max(w.s, s);
    w.lx = std::max(w.lx, lx);
    w.o = std::max(w.o, o);
    w.q = std::max(w.q, q);
    if (tp > 1 && tp <= kTpMaxRanks &&
        (w.partial.p != ipc_part_src || w.x.p != ipc_x_src || w.tp_flags.p != ipc_flags_src)) {
      exchange_ipc();
      ++ws_allocations;
    }
  }

  // clef_reserve: the device workspace and the pinned host staging of a host
  // forward, for batches up to this shape.
  void reserve_all(int b, int s, int lx, int o, int q) {
    reserve(b, s, lx, o, q);
    grow_pinned(pinned_need(b, s, lx, o, q));
  }

  // -------------------------------------------------------------------------
  // forward
  // -------------------------------------------------------------------------

  template <typename T>
  void dense(Launcher& Lc, const T* x, int M, int K, const Tensor& w, const Tensor* bias, T* out, int ldo,
             bool gelu) {
    const int N = static_cast<int>(w.shape[0]);
    REQUIRE(static_cast<int>(w.shape[1]) == K, "dense(): inner dimension mismatch");
    const T* bp = bias ? bias->buf.as<T>() : nullptr;
    if constexpr (sizeof(T) == 2) {
      // tcgen05 at every M: per-row results then do not depend on how many
      // rows share the launch (answers are independent of batching).
      if (!gelu && K % 8 == 0 && N % 8 == 0 && ldo % 8 == 0 && aligned16(x) && aligned16(w.buf.p) && aligned16(out)) {
        gemm_bf16(Lc, kEpiStore, x, K, w.buf.as<bf16>(), K, M, N, K, out, ldo, bp, nullptr, 0);
        return;
      }
    }
    gemm_simt<T>(Lc, gelu ? kSimtGelu : kSimtStore, x, K, w.buf.as<T>(), K, M, N, K, out, ldo, bp, nullptr, 0);
  }

  // nn.MultiheadAttention with packed in-projection (head.py:37-47).
  template <typename T>
  void mha(Launcher& Lc, const T* query, int nq, const T* memory, int nk, const uint8_t* key_mask, int B,
           const std::string& name, T* qbuf, T* kvbuf, T* abuf, T* out) {
    const Tensor& win = h(name + ".in_proj_weight");
    const Tensor& bin = h(name + ".in_proj_bias");
    const T* wq = win.buf.as<T>();
    const T* wkv = wq + static_cast<size_t>(W) * W;
    const T* bq = bin.buf.as<T>();
    const T* bkv = bq + W;
    const int Mq = B * nq, Mk = B * nk;
    // q = T(query Wq^T + bq); [k|v] = T(memory [Wk;Wv]^T + [bk;bv])
    auto proj = [&](const T* x, int M, const T* w, int N, const T* b, T* o) {
      if constexpr (sizeof(T) == 2) {
        if (W % 8 == 0 && aligned16(x) && aligned16(w) && aligned16(o)) {
          gemm_bf16(Lc, kEpiStore, x, W, w, W, M, N, W, o, N, b, nullptr, 0);
          return;
        }
      }
      gemm_simt<T>(Lc, kSimtStore, x, W, w, W, M, N, W, o, N, b, nullptr, 0);
    };
    proj(query, Mq, wq, W, bq, qbuf);
    proj(memory, Mk, wkv, 2 * W, bkv, kvbuf);
    const int hd = W / HH;
    AttnArgs<T> a{};
    a.q = qbuf;
    a.ldq = W;
    a.hsq = hd;
    a.k = kvbuf;
    a.ldk = 2 * W;
    a.hsk = hd;
    a.v = kvbuf + W;
    a.ldv = 2 * W;
    a.hsv = hd;
    a.gate = nullptr;
    a.out = abuf;
    a.ldo = W;
    a.hso = hd;
    a.key_mask = key_mask;
    a.B = B;
    a.Lq = nq;
    a.Lk = nk;
    a.H = HH;
    a.Hk = HH;
    a.hd = hd;
    a.causal = 0;
    a.softcap = 0.f;
    a.window = 0;
    a.status = Lc.status;
    attention<T>(Lc, a);
    dense<T>(Lc, abuf, Mq, W, h(name + ".out_proj.weight"), h_opt(name + ".out_proj.bias"), out, W, false);
  }

  template <typename T>
  void add(Launcher& Lc, T* x, const T* y, long long n) {
    add_inplace_kernel<T><<<static_cast<int>(std::min<long long>((n + 255) / 256, 4096)), 256, 0, Lc.stream>>>(x, y, n);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
  }

  template <typename T>
  void ln(Launcher& Lc, const T* x, const std::string& name, T* out, int rows) {
    const Tensor& w = h(name + ".weight");
    layernorm<T>(Lc, x, w.buf.as<T>(), h(name + ".bias").buf.as<T>(), out, rows, static_cast<int>(w.shape[0]));
  }

  // Batch arrays in device memory.
  struct DevBatch {
    int b, s, lx, o, q;
    const int32_t *ids, *lex_ids, *lex_spans, *q_spans, *types, *o_spans, *owner;
    const uint8_t *mask, *q_mask, *o_mask;
  };

  // Full-attention mixer + residual: RMSNorm, QKV projection (fused q/k-norm,
  // RoPE and gate sigmoid where possible), causal GQA attention with the output
  // gate, o-proj with the residual (text.py:70-98).
  template <typename T>
  void attention_mixer(Launcher& Lc, Layer& l, int li, const DevBatch& bt, T* x, T* hbuf, T* qkv, T* attn_out, int Tt) {
    const int B = bt.b, S = bt.s;
    const float eps = cfg.rms_norm_eps;
    const int ldqkv = Nqkv;
    cudaStream_t st = Lc.stream;
    Lc.cat = kCatNorm;
    rmsnorm<T>(Lc, x, D, l.w_in.as<T>(), hbuf, D, Tt, D, eps);
    Lc.cat = kCatGemmQkv;
    bool fused_qkv = false;
    if constexpr (sizeof(T) == 2) {
      if (qkv_fusable(d, rot)) {
        const QkvFusion f{l.q_norm.as<bf16>(), l.k_norm.as<bf16>(), rope_cos.as<float>(), rope_sin.as<float>(),
                          Hq_l,           Hkv_l,  d,  rot, S, eps};
        gemm_bf16_qkv(Lc, hbuf, D, l.w_qkv.as<bf16>(), D, Tt, Nqkv, D, qkv, ldqkv, f);
        fused_qkv = true;
      } else {
        gemm_bf16(Lc, kEpiStore, hbuf, D, l.w_qkv.as<bf16>(), D, Tt, Nqkv, D, qkv, ldqkv, nullptr, nullptr, 0);
      }
    } else {
      gemm_simt<T>(Lc, kSimtStore, hbuf, D, l.w_qkv.as<T>(), D, Tt, Nqkv, D, qkv, ldqkv, nullptr, nullptr, 0);
    }
    if (!fused_qkv) {
      const int warps = 8;
      const long long items = static_cast<long long>(Tt) * (Hq_l + Hkv_l);
      qk_norm_rope_kernel<T><<<static_cast<int>((items + warps - 1) / warps), warps * 32, warps * d * 4, st>>>(
          qkv, ldqkv, Tt, S, Hq_l, Hkv_l, d, rot, l.q_norm.as<T>(), l.k_norm.as<T>(), rope_cos.as<float>(),
          rope_sin.as<float>(), eps);
      CUDA_CHECK(cudaGetLastError());
      Lc.cat = kCatQkRope;
      Lc.tick();
    }
    {
      AttnArgs<T> a{};
      a.q = qkv;
      a.ldq = ldqkv;
      a.hsq = 2 * d;
      a.k = qkv + static_cast<size_t>(Hq_l) * 2 * d;
      a.ldk = ldqkv;
      a.hsk = d;
      a.v = a.k + static_cast<size_t>(Hkv_l) * d;
      a.ldv = ldqkv;
      a.hsv = d;
      a.gate = qkv + d;
      a.ldg = ldqkv;
      a.hsg = 2 * d;
      a.out = attn_out;
      a.ldo = static_cast<long long>(Hq_l) * d;
      a.hso = d;
      a.key_mask = bt.mask;
      a.B = B;
      a.Lq = S;
      a.Lk = S;
      a.H = Hq_l;
      a.Hk = Hkv_l;
      a.hd = d;
      a.causal = 1;
      a.softcap = cfg.attn_softcap;
      a.window = layer_window[li];
      a.status = Lc.status;
      a.packed = 1;
      a.gate_presig = fused_qkv ? 1 : 0;
      Lc.cat = kCatAttention;
      attention<T>(Lc, a);
    }
    Lc.cat = kCatGemmO;
    project_residual<T>(Lc, attn_out, Hq_l * d, l.w_o.as<T>(), x, Tt);
  }

  // Gated DeltaNet mixer + residual (text.py:42-45,94-98): RMSNorm with padded
  // rows zeroed, one packed projection GEMM [q|k|v|z|a|b], the fused
  // conv/recurrence/gated-norm kernel, out_proj with the residual (FP32 TP sum
  // before the cast when tp > 1).
  template <typename T>
  void gdn_mixer(Launcher& Lc, Layer& l, const DevBatch& bt, T* x, T* hbuf, T* core, int Tt) {
    Lc.cat = kCatNorm;
    rmsnorm<T>(Lc, x, D, l.w_in.as<T>(), hbuf, D, Tt, D, cfg.rms_norm_eps, bt.mask);
    T* proj = ws.gproj.as<T>();
    Lc.cat = kCatGemmQkv;
    if constexpr (sizeof(T) == 2)
      gemm_bf16(Lc, kEpiStore, hbuf, D, l.g_proj.as<bf16>(), D, Tt, Ng_pad, D, proj, Ng_pad, nullptr, nullptr, 0);
    else
      gemm_simt<T>(Lc, kSimtStore, hbuf, D, l.g_proj.as<T>(), D, Tt, Ng_pad, D, proj, Ng_pad, nullptr, nullptr, 0);
    GdnArgs a{};
    a.proj = proj;
    a.ldp = Ng_pad;
    a.k_col = g_nh_l * g_dh;
    a.v_col = 2 * g_nh_l * g_dh;
    a.z_col = Cg;
    a.a_col = Cg + g_nv_l * g_dh;
    a.b_col = a.a_col + g_nv_l;
    a.conv = l.g_conv.p;
    a.width = g_width;
    a.A_log = l.g_alog.p;
    a.dt_bias = l.g_dtb.p;
    a.norm_w = l.g_norm.p;
    a.out = core;
    a.ldo = static_cast<long long>(g_nv_l) * g_dh;
    a.B = bt.b;
    a.S = bt.s;
    a.nh = g_nh_l;
    a.nv = g_nv_l;
    a.qscale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(g_dh)));
    a.eps = cfg.rms_norm_eps;
    a.status = Lc.status;
    if (gdn_conv_pass()) gdn_tc_bind_scratch(a, ws.gconv.p);
    Lc.cat = kCatGdn;
    launch_gdn<T>(Lc, a, g_dh);
    Lc.cat = kCatGemmO;
    project_residual<T>(Lc, core, g_nv_l * g_dh, l.g_out.as<T>(), x, Tt);
  }

  // CLEF_DEBUG_POISON: NaN bytes over every scratch buffer a forward writes
  // before it reads (not the staged batch, the flags or the status word).
  void poison_scratch(cudaStream_t st) {
    Workspace& w = ws;
    for (DBuf* b : {&w.x, &w.h, &w.qkv, &w.attn, &w.gu, &w.act, &w.partial, &w.gproj, &w.gconv, &w.memory, &w.mnorm, &w.kv,
                    &w.gv, &w.questions, &w.contexts, &w.lexical, &w.small, &w.f32small})
      if (b->p) CUDA_CHECK(cudaMemsetAsync(b->p, 0xFF, b->bytes, st));
  }

  template <typename T>
  void forward_impl(const DevBatch& bt, float* logits, cudaStream_t st) {
    REQUIRE(finalized, "clef_forward before clef_finalize");
    NvtxRange forward_range("clef forward");
    if (debug_flags & CLEF_DEBUG_POISON) poison_scratch(st);
    Launcher Lc{st, status.as<int>(), 0, kCatOther, &timeline};
    Lc.mark(-1);  // timeline start marker
    const int B = bt.b, S = bt.s;
    const int Tt = B * S;
    Workspace& w = ws;
    T* x = w.x.as<T>();
    T* hbuf = w.h.as<T>();
    T* qkv = w.qkv.as<T>();
    T* attn_out = w.attn.as<T>();
    T* act = w.act.as<T>();
    const float eps = cfg.rms_norm_eps;
    (void)S;

    // 1. embedding (model.py:95)
    {
      const int warps = 8;
      embed_kernel<T><<<(Tt + warps - 1) / warps, warps * 32, 0, st>>>(bt.ids, embedding.as<T>(), x, Tt, D, V,
                                                                      cfg.embed_scale, Lc.status);
      CUDA_CHECK(cudaGetLastError());
      Lc.cat = kCatEmbed;
      Lc.tick();
    }
    // 2. decoder layers (text.py:94-102; TP: pallas.py:62-129)
    for (int li = 0; li < L; ++li) {
      Layer& l = layers[li];
      const bool linear = layer_types[li] == CLEF_LAYER_LINEAR_ATTENTION;
      char name[48];
      std::snprintf(name, sizeof(name), "layer %d %s", li, linear ? "linear_attention" : "full_attention");
      NvtxRange layer_range(name);
      {
        NvtxRange mixer_range(linear ? "gated deltanet" : "attention");
        if (linear)
          gdn_mixer<T>(Lc, l, bt, x, hbuf, attn_out, Tt);
        else
          attention_mixer<T>(Lc, l, li, bt, x, hbuf, qkv, attn_out, Tt);
      }
      NvtxRange mlp_range("mlp");
      Lc.cat = kCatNorm;
      rmsnorm<T>(Lc, x, D, l.w_post.as<T>(), hbuf, D, Tt, D, eps);
      Lc.cat = kCatGemmGateUp;
      if constexpr (sizeof(T) == 2) {
        gemm_bf16(Lc, kEpiSwiglu, hbuf, D, l.w_gu.as<bf16>(), D, Tt, 2 * Fp, D, act, Fp, nullptr, nullptr, 0);
      } else {
        T* gu = w.gu.as<T>();
        gemm_simt<T>(Lc, kSimtStore, hbuf, D, l.w_gu.as<T>(), D, Tt, 2 * Fp, D, gu, 2 * Fp, nullptr, nullptr, 0);
        swiglu_packed_kernel<T><<<4096, 256, 0, st>>>(gu, act, Tt, Fp);
        CUDA_CHECK(cudaGetLastError());
        Lc.tick();
      }
      Lc.cat = kCatGemmDown;
      project_residual<T>(Lc, act, Fp, l.w_down.as<T>(), x, Tt);
    }
    // 3. final norm (model.py:99) -> hbuf
    Lc.cat = kCatNorm;
    rmsnorm<T>(Lc, x, D, final_norm.as<T>(), hbuf, D, Tt, D, eps);
    // 4-5. lexical means and the joint head
    Lc.cat = kCatHead;
    {
      NvtxRange head_range("lexical means + joint head");
      scoring<T>(Lc, bt, logits);
    }
    last_launches = Lc.count;
  }

  // Lexical option means over lm_head rows (model.py:100) and the joint head
  // (head.py:50-107) on the final-normed hidden states held in ws.h.
  template <typename T>
  void scoring(Launcher& Lc, const DevBatch& bt, float* logits) {
    T* lexical = ws.lexical.as<T>();
    span_means_kernel<T><<<dim3(bt.o, bt.b), 256, 0, Lc.stream>>>(lm_head.as<T>(), D, bt.lx, bt.lex_ids, V,
                                                                  bt.lex_spans, bt.o, D, lexical, Lc.status);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    head_forward<T>(Lc, bt, ws.h.as<T>(), ws.x.as<T>(), lexical, logits);
  }

  // Head only, from host hidden states [b, s, D] float32 (the joint-head fixture's input).
  void forward_head_host(const ClefBatch& b, const float* hidden, float* out_logits) {
    DevBatch d = stage_host_batch(b);
    const size_t nh = static_cast<size_t>(b.b) * b.s * D;
    std::vector<uint8_t> tmp;
    convert(hidden, CLEF_DTYPE_F32, nh, tmp);
    CUDA_CHECK(cudaMemcpyAsync(ws.h.p, tmp.data(), tmp.size(), cudaMemcpyHostToDevice, stream));
    const size_t nlog = static_cast<size_t>(b.b) * b.o;
    float* dlog = ws.f32small.as<float>() + nlog * 2;
    Launcher Lc{stream, status.as<int>(), 0, kCatHead, &timeline};
    if (dtype == CLEF_DTYPE_BF16)
      scoring<bf16>(Lc, d, dlog);
    else
      scoring<float>(Lc, d, dlog);
    std::vector<float> host(nlog);
    CUDA_CHECK(cudaMemcpyAsync(host.data(), dlog, nlog * 4, cudaMemcpyDeviceToHost, stream));
    CUDA_CHECK(cudaStreamSynchronize(stream));
    check_status();
    std::memcpy(out_logits, host.data(), nlog * 4);
  }

  // x = T(x + T(in W^T)), with an FP32 all-reduce across TP ranks before the
  // cast when tp > 1 (pallas.py:66-69,121).
  template <typename T>
  void project_residual(Launcher& Lc, const T* in, int K, const T* w, T* x, int Tt) {
    if (tp == 1) {
      if constexpr (sizeof(T) == 2)
        gemm_bf16(Lc, kEpiResidual, in, K, w, K, Tt, D, K, x, D, nullptr, x, D);
      else
        gemm_simt<T>(Lc, kSimtResidual, in, K, w, K, Tt, D, K, x, D, nullptr, x, D);
      return;
    }
    float* part = ws.partial.as<float>();
    if constexpr (sizeof(T) == 2) {
      // The fused kernel pays off while the GEMM is not much shorter than its
      // reduction: GEMM time ~ K, NVLink bytes per rank ~ 4 (tp-1)/tp per
      // output element, so K tp / (tp-1) >= 1536 (measured on cfg4: o-proj at
      // TP=8, K = 512, runs faster unfused; down-proj at every tp and o-proj
      // at TP=2 faster fused; o-proj at TP=4, K = 1024, the same either way).
      const bool fuse = static_cast<long long>(K) * tp >= 1536LL * (tp - 1);
      if (fuse && p2p && (tp == 2 || tp == 4 || tp == 8) && Tt >= 256 && D >= 256 && D % 8 == 0 && K % 8 == 0 &&
          aligned16(in) && aligned16(w) && static_cast<void*>(x) == ws.x.p) {
        // One kernel: the GEMM's FP32 partial tiles, flagged to their owners,
        // reduced by the owners while later tiles' MMAs run; after the barrier
        // every rank's x is complete.
        GemmArgs args{Tt, D, K, part, D, nullptr, nullptr, 0, Lc.status};
        TpFuse f{};
        for (int k = 0; k < tp; ++k) {
          f.parts[k] = static_cast<const float*>(peer_part[k]);
          f.xs[k] = static_cast<bf16*>(peer_x[k]);
          f.flags[k] = static_cast<unsigned*>(peer_flags[k]);
        }
        f.tp = tp;
        f.rank = rank;
        f.ldx = D;
        f.epoch = ++tp_epoch;
        const CUtensorMap ta = tmap_bf16(in, Tt, K, K, 128);
        const CUtensorMap tb = tmap_bf16(w, D, K, K, 128);
        launch_tc_gemm_pair<kEpiF32, true>(ta, tb, args, Lc.stream, f);
        Lc.tick();
        const int saved = Lc.cat;
        tp_barrier(Lc);
        Lc.mark(kCatAllReduce);
        Lc.cat = saved;
        return;
      }
      gemm_bf16(Lc, kEpiF32, in, K, w, K, Tt, D, K, part, D, nullptr, nullptr, 0);
    }
    else
      gemm_simt<T>(Lc, kSimtF32, in, K, w, K, Tt, D, K, part, D, nullptr, nullptr, 0);
    if (p2p) {
      // every rank's partial complete -> each rank reduces its rows from every
      // rank's partial and writes them into every x -> every x complete
      const int saved = Lc.cat;
      tp_barrier(Lc);
      Lc.mark(kCatAllReduce);  // barriers are timed as "allreduce", the reduction as "residual_add"
      Lc.cat = kCatResidual;
      TpReduceArgs a{};
      for (int k = 0; k < tp; ++k) {
        a.parts[k] = static_cast<const float*>(peer_part[k]);
        a.xs[k] = peer_x[k];
      }
      a.tp = tp;
      a.rank = rank;
      const long long rows_per = (Tt + tp - 1) / tp;
      const long long r0 = std::min<long long>(Tt, rows_per * rank), r1 = std::min<long long>(Tt, r0 + rows_per);
      a.e0 = r0 * D;
      a.e1 = r1 * D;
      a.vec8 = sizeof(T) == 2 && D % 8 == 0;  // rows of the cudaMalloc'd buffers are then 16-byte aligned
      const long long vecs = (a.e1 - a.e0) / (a.vec8 ? 8 : 4);
      const int grid = static_cast<int>(std::max<long long>(1, std::min<long long>((vecs + 255) / 256, 148LL * 8)));
      tp_reduce_residual_kernel<T><<<grid, 256, 0, Lc.stream>>>(a);
      CUDA_CHECK(cudaGetLastError());
      Lc.tick();
      tp_barrier(Lc);
      Lc.mark(kCatAllReduce);
      Lc.cat = saved;
      return;
    }
    nccl_done(ncclAllReduce(part, part, static_cast<size_t>(Tt) * D, ncclFloat32, ncclSum, comm, Lc.stream),
              "ncclAllReduce");
    Lc.mark(kCatAllReduce);
    const long long n = static_cast<long long>(Tt) * D;
    residual_add_f32_kernel<T><<<static_cast<int>(std::min<long long>((n + 255) / 256, 8192)), 256, 0, Lc.stream>>>(
        x, part, n);
    CUDA_CHECK(cudaGetLastError());
    const int saved = Lc.cat;
    Lc.cat = kCatResidual;
    Lc.tick();
    Lc.cat = saved;
  }

  template <typename T>
  void head_forward(Launcher& Lc, const DevBatch& bt, const T* hn, T* scratch_td, const T* lexical, float* logits) {
    const int B = bt.b, S = bt.s, O = bt.o, Q = bt.q, Tt = B * S;
    cudaStream_t st = Lc.stream;
    Workspace& w = ws;
    T* hl = scratch_td;  // hidden_norm(h): [Tt, D]
    T* memory = w.memory.as<T>();
    T* mn = w.mnorm.as<T>();
    T* kv = w.kv.as<T>();
    T* gv = w.gv.as<T>();
    T* questions = w.questions.as<T>();
    T* contexts = w.contexts.as<T>();
    // carve small buffers
    const size_t rows = static_cast<size_t>(B) * std::max(O, Q);
    const size_t widest = std::max<size_t>({static_cast<size_t>(3 * W), static_cast<size_t>(FF), static_cast<size_t>(4 * W)});
    T* base_ptr = w.small.as<T>();
    size_t off = 0;
    auto carve = [&](size_t n) {
      T* p = base_ptr + off;
      off += (n + 63) / 64 * 64;
      return p;
    };
    T* options = carve(rows * W);
    T* t1 = carve(rows * widest);
    T* t2 = carve(rows * widest);
    T* t3 = carve(rows * widest);
    T* t4 = carve(rows * widest);
    T* t5 = carve(rows * widest);
    T* base = carve(rows * W);
    T* fields = carve(rows * W);
    T* gp = carve(static_cast<size_t>(B) * W);
    float* prior = w.f32small.as<float>();
    float* cosv = prior + static_cast<size_t>(B) * O;

    ln<T>(Lc, hn, "hidden_norm", hl, Tt);
    dense<T>(Lc, hl, Tt, D, h("memory_projection.weight"), h_opt("memory_projection.bias"), memory, W, false);
    last_token_kernel<T><<<B, 256, 0, st>>>(hl, S, D, bt.mask, gv);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    span_means_kernel<T><<<dim3(Q, B), 256, 0, st>>>(hl, D, S, nullptr, 0, bt.q_spans, Q, D, questions, Lc.status);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    span_means_kernel<T><<<dim3(O, B), 256, 0, st>>>(hl, D, S, nullptr, 0, bt.o_spans, O, D, contexts, Lc.status);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    // options = ctx_proj + lex_proj + gather(q_proj, owners)   (head.py:62-63)
    dense<T>(Lc, contexts, B * O, D, h("option_context_projection.weight"), h_opt("option_context_projection.bias"), t1, W,
             false);
    dense<T>(Lc, lexical, B * O, D, h("option_lexical_projection.weight"), h_opt("option_lexical_projection.bias"), t2, W,
             false);
    dense<T>(Lc, questions, B * Q, D, h("option_question_projection.weight"), h_opt("option_question_projection.bias"),
             t3, W, false);
    options_init_kernel<T><<<dim3(O, B), 128, 0, st>>>(t1, t2, t3, bt.owner, O, Q, W, options);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    // evidence routing layers (head.py:65-70)
    for (int i = 0; i < RL; ++i) {
      const std::string n = "evidence_layers." + std::to_string(i);
      ln<T>(Lc, options, n + ".query_norm", t1, B * O);
      ln<T>(Lc, memory, n + ".memory_norm", mn, Tt);
      mha<T>(Lc, t1, O, mn, S, bt.mask, B, n + ".attention", t2, kv, t3, t4);
      add<T>(Lc, options, t4, static_cast<long long>(B) * O * W);
      ln<T>(Lc, options, n + ".feedforward_norm", t1, B * O);
      dense<T>(Lc, t1, B * O, W, h(n + ".feedforward.0.weight"), h_opt(n + ".feedforward.0.bias"), t2, FF, true);
      dense<T>(Lc, t2, B * O, FF, h(n + ".feedforward.3.weight"), h_opt(n + ".feedforward.3.bias"), t3, W, false);
      add<T>(Lc, options, t3, static_cast<long long>(B) * O * W);
    }
    // question base, routing softmax and summary (head.py:72-79)
    dense<T>(Lc, questions, B * Q, D, h("question_projection.weight"), h_opt("question_projection.bias"), base, W, false);
    route_summary_kernel<T><<<dim3(Q, B), 128, (O + 32) * sizeof(float), st>>>(options, base, bt.owner, bt.o_mask, O, Q,
                                                                              W, t1);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    ln<T>(Lc, t1, "option_summary_norm", t2, B * Q);
    dense<T>(Lc, gv, B, D, h("global_projection.weight"), h_opt("global_projection.bias"), gp, W, false);
    const Tensor& te = h("type_embedding.weight");
    fields_init_kernel<T><<<dim3(Q, B), 128, 0, st>>>(base, t2, gp, te.buf.as<T>(), static_cast<int>(te.shape[0]),
                                                      bt.types, Q, W, fields);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    // field transformer layers (head.py:84-90)
    for (int i = 0; i < HL; ++i) {
      const std::string n = "layers." + std::to_string(i);
      ln<T>(Lc, fields, n + ".norm1", t1, B * Q);
      mha<T>(Lc, t1, Q, t1, Q, bt.q_mask, B, n + ".self_attn", t2, t3, t4, t5);
      add<T>(Lc, fields, t5, static_cast<long long>(B) * Q * W);
      ln<T>(Lc, fields, n + ".norm2", t1, B * Q);
      mha<T>(Lc, t1, Q, memory, S, bt.mask, B, n + ".multihead_attn", t2, kv, t3, t4);
      add<T>(Lc, fields, t4, static_cast<long long>(B) * Q * W);
      ln<T>(Lc, fields, n + ".norm3", t1, B * Q);
      dense<T>(Lc, t1, B * Q, W, h(n + ".linear1.weight"), h_opt(n + ".linear1.bias"), t2, FF, true);
      dense<T>(Lc, t2, B * Q, FF, h(n + ".linear2.weight"), h_opt(n + ".linear2.bias"), t3, W, false);
      add<T>(Lc, fields, t3, static_cast<long long>(B) * Q * W);
    }
    // scoring (head.py:92-107)
    ln<T>(Lc, fields, "field_norm", t1, B * Q);
    ln<T>(Lc, options, "option_norm", t2, B * O);
    prior_cosine_kernel<T><<<dim3(O, B), 256, 0, st>>>(questions, gv, lexical, t1, t2, bt.owner, O, Q, D, W, t3, prior,
                                                       cosv);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
    dense<T>(Lc, t3, B * O, 4 * W, h("residual_scorer.0.weight"), h_opt("residual_scorer.0.bias"), t4, W, true);
    T* rs = t1;  // [B*O, 1]
    dense<T>(Lc, t4, B * O, W, h("residual_scorer.3.weight"), h_opt("residual_scorer.3.bias"), rs, 1, false);
    final_logits_kernel<T><<<(B * O + 127) / 128, 128, 0, st>>>(
        prior, cosv, rs, bt.o_mask, h("prior_logit_scale").buf.as<T>(), h("joint_logit_scale").buf.as<T>(),
        h("residual_gate").buf.as<T>(), B * O, static_cast<float>(std::log(100.0)), logits);
    CUDA_CHECK(cudaGetLastError());
    Lc.tick();
  }

  // -------------------------------------------------------------------------
  // entry points
  // -------------------------------------------------------------------------

  void check_batch(const ClefBatch& b) {
    REQUIRE(b.b > 0 && b.s > 0 && b.lx > 0 && b.o > 0 && b.q > 0, "batch dimensions must be positive");
    REQUIRE(b.s <= cfg.max_seq_len, "sequence length exceeds max_seq_len");
    REQUIRE(b.input_ids && b.mask && b.lexical_ids && b.lexical_spans && b.question_spans && b.question_mask &&
                b.types && b.option_spans && b.option_mask && b.option_field,
            "null batch array");
  }

  DevBatch carve_batch(const ClefBatch& b, int32_t* ibuf, uint8_t* bbuf) {
    DevBatch d{};
    d.b = b.b;
    d.s = b.s;
    d.lx = b.lx;
    d.o = b.o;
    d.q = b.q;
    size_t o = 0;
    auto ic = [&](size_t n) {
      int32_t* p = ibuf + o;
      o += n;
      return p;
    };
    const size_t B = b.b;
    d.ids = ic(B * b.s);
    d.lex_ids = ic(B * b.lx);
    d.lex_spans = ic(B * b.o * 2);
    d.q_spans = ic(B * b.q * 2);
    d.types = ic(B * b.q);
    d.o_spans = ic(B * b.o * 2);
    d.owner = ic(B * b.o);
    size_t ob = 0;
    auto bc = [&](size_t n) {
      uint8_t* p = bbuf + ob;
      ob += n;
      return p;
    };
    d.mask = bc(B * b.s);
    d.q_mask = bc(B * b.q);
    d.o_mask = bc(B * b.o);
    return d;
  }

  // Validate a host batch and copy it to the device through one pinned staging buffer.
  DevBatch stage_host_batch(const ClefBatch& b) {
    check_batch(b);
    CUDA_CHECK(cudaSetDevice(device));
    // Host-side validation the reference gets from JAX's checked gathers.
    for (size_t i = 0; i < static_cast<size_t>(b.b) * b.s; ++i)
      REQUIRE(b.input_ids[i] >= 0 && b.input_ids[i] < V, "input_ids out of vocabulary range");
    for (size_t i = 0; i < static_cast<size_t>(b.b) * b.lx; ++i)
      REQUIRE(b.lexical_ids[i] >= 0 && b.lexical_ids[i] < V, "lexical_ids out of vocabulary range");
    reserve(b.b, b.s, b.lx, b.o, b.q);
    Workspace& w = ws;
    const size_t ni = batch_int_count(b.b, b.s, b.lx, b.o, b.q), nb = batch_byte_count(b.b, b.s, b.o, b.q);
    grow_pinned(pinned_need(b.b, b.s, b.lx, b.o, b.q));
    uint8_t* hp = static_cast<uint8_t*>(w.host_pinned.p);
    int32_t* hi = reinterpret_cast<int32_t*>(hp);
    size_t o = 0;
    auto put = [&](const int32_t* src, size_t n) {
      std::memcpy(hi + o, src, n * 4);
      o += n;
    };
    const size_t B = b.b;
    put(b.input_ids, B * b.s);
    put(b.lexical_ids, B * b.lx);
    put(b.lexical_spans, B * b.o * 2);
    put(b.question_spans, B * b.q * 2);
    put(b.types, B * b.q);
    put(b.option_spans, B * b.o * 2);
    put(b.option_field, B * b.o);
    uint8_t* hb = hp + ni * 4;
    std::memcpy(hb, b.mask, B * b.s);
    std::memcpy(hb + B * b.s, b.question_mask, B * b.q);
    std::memcpy(hb + B * b.s + B * b.q, b.option_mask, B * b.o);
    CUDA_CHECK(cudaMemcpyAsync(w.ints.p, hi, ni * 4, cudaMemcpyHostToDevice, stream));
    CUDA_CHECK(cudaMemcpyAsync(w.bytes.p, hb, nb, cudaMemcpyHostToDevice, stream));
    return carve_batch(b, w.ints.as<int32_t>(), w.bytes.as<uint8_t>());
  }

  void forward_host(const ClefBatch& b, float* out_logits, float* out_hidden) {
    DevBatch d = stage_host_batch(b);
    Workspace& w = ws;
    const size_t nlog = static_cast<size_t>(b.b) * b.o;
    float* dlog = w.f32small.as<float>() + static_cast<size_t>(b.b) * b.o * 2;
    if (dtype == CLEF_DTYPE_BF16)
      forward_impl<bf16>(d, dlog, stream);
    else
      forward_impl<float>(d, dlog, stream);
    std::vector<float> tmp_logits(nlog);
    CUDA_CHECK(cudaMemcpyAsync(tmp_logits.data(), dlog, nlog * 4, cudaMemcpyDeviceToHost, stream));
    std::vector<uint8_t> hid;
    const size_t nh = static_cast<size_t>(b.b) * b.s * D;
    if (out_hidden) {
      hid.resize(nh * esz);
      CUDA_CHECK(cudaMemcpyAsync(hid.data(), w.h.p, nh * esz, cudaMemcpyDeviceToHost, stream));
    }
    wait_stream();
    check_status();
    std::memcpy(out_logits, tmp_logits.data(), nlog * 4);
    if (out_hidden) {
      if (dtype == CLEF_DTYPE_F32) {
        std::memcpy(out_hidden, hid.data(), nh * 4);
      } else {
        const uint16_t* hb16 = reinterpret_cast<const uint16_t*>(hid.data());
        for (size_t i = 0; i < nh; ++i) out_hidden[i] = bf16_bits_to_f32(hb16[i]);
      }
    }
  }

  void forward_device(const ClefBatch& b, float* out_logits, cudaStream_t st) {
    check_batch(b);
    CUDA_CHECK(cudaSetDevice(device));
    reserve(b.b, b.s, b.lx, b.o, b.q);
    DevBatch d{};
    d.b = b.b;
    d.s = b.s;
    d.lx = b.lx;
    d.o = b.o;
    d.q = b.q;
    d.ids = b.input_ids;
    d.lex_ids = b.lexical_ids;
    d.lex_spans = b.lexical_spans;
    d.q_spans = b.question_spans;
    d.types = b.types;
    d.o_spans = b.option_spans;
    d.owner = b.option_field;
    d.mask = b.mask;
    d.q_mask = b.question_mask;
    d.o_mask = b.option_mask;
    if (dtype == CLEF_DTYPE_BF16)
      forward_impl<bf16>(d, out_logits, st ? st : stream);
    else
      forward_impl<float>(d, out_logits, st ? st : stream);
  }

  void check_status() {
    int s = 0;
    CUDA_CHECK(cudaMemcpy(&s, status.p, sizeof(int), cudaMemcpyDeviceToHost));
    if (s != 0) {
      CUDA_CHECK(cudaMemset(status.p, 0, sizeof(int)));
      const char* what = s == kBadIndex         ? "token id out of range"
                         : s == kTimeoutTpFlag  ? "a tensor-parallel peer's tile did not arrive in time"
                         : s == kBadTpRanks     ? "fused tensor-parallel reduction launched for an unsupported rank count"
                                                : "pipeline wait timed out";
      char buf[160];
      std::snprintf(buf, sizeof(buf), "device status 0x%x (%s)", s, what);
      throw Error(CLEF_EDEVICE, buf);
    }
  }
};

}  // namespace clef

// ===========================================================================
// C ABI
// ===========================================================================

using clef::Error;
using clef::Model;

template <typename F>
static int guarded(Model* m, F&& f) {
  if (m && m->broken) {
    m->last_error = "handle unusable after a tensor-parallel timeout or NCCL failure; destroy it and end the process";
    clef::set_global_error(m->last_error);
    return CLEF_ESTATE;
  }
  try {
    f();
    return CLEF_OK;
  } catch (const Error& e) {
    if (m) m->last_error = e.what();
    clef::set_global_error(e.what());
    return e.code;
  } catch (const std::exception& e) {
    if (m) m->last_error = e.what();
    clef::set_global_error(e.what());
    return CLEF_EINVAL;
  }
}

extern "C" {

int clef_nccl_unique_id(uint8_t out[CLEF_NCCL_ID_BYTES]) {
  return guarded(nullptr, [&] {
    REQUIRE(out != nullptr, "null output");
    static_assert(sizeof(ncclUniqueId) == CLEF_NCCL_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    NCCL_CHECK(ncclGetUniqueId(&id));
    std::memcpy(out, &id, sizeof(id));
  });
}

int clef_create(const ClefConfig* config, int device, int tp_rank, int tp_size, const uint8_t* nccl_id, int dtype,
                void** handle) {
  return guarded(nullptr, [&] {
    REQUIRE(config && handle, "null argument");
    auto m = std::make_unique<Model>();
    m->init(*config, device, tp_rank, tp_size, nccl_id, dtype);
    *handle = m.release();
  });
}

int clef_upload(void* handle, const char* name, const void* host, int host_dtype, const int64_t* shape, int ndim) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && name && (ndim == 0 || shape) && ndim >= 0 && ndim <= 4, "bad clef_upload arguments");
    m->upload(name, host, host_dtype, shape, ndim);
  });
}

int clef_upload_device(void* handle, const char* name, const void* device_ptr, int dtype, const int64_t* shape,
                       int ndim) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && name && (ndim == 0 || shape) && ndim >= 0 && ndim <= 4, "bad clef_upload_device arguments");
    m->src_on_device = true;
    try {
      m->upload(name, device_ptr, dtype, shape, ndim);
    } catch (...) {
      m->src_on_device = false;
      throw;
    }
    m->src_on_device = false;
  });
}

int clef_set_timing(void* handle, int enable) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m, "null handle");
    m->timeline.enabled = enable != 0;
    m->timeline.used = 0;
    m->timeline.cats.clear();
  });
}

int clef_timing_report(void* handle, int n, float* ms, int* launches) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && ms && launches && n > 0, "bad clef_timing_report arguments");
    CUDA_CHECK(cudaSetDevice(m->device));
    m->timing_report(n, ms, launches);
  });
}

int clef_finalize(void* handle) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m, "null handle");
    m->finalize();
  });
}

int clef_forward(void* handle, const ClefBatch* batch, float* out_logits, float* out_hidden) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && batch && out_logits, "null argument");
    if (!m->finalized) throw Error(CLEF_ESTATE, "clef_forward before clef_finalize");
    m->forward_host(*batch, out_logits, out_hidden);
  });
}

int clef_forward_head(void* handle, const ClefBatch* batch, const float* hidden, float* out_logits) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && batch && hidden && out_logits, "null argument");
    if (!m->finalized) throw Error(CLEF_ESTATE, "clef_forward_head before clef_finalize");
    m->forward_head_host(*batch, hidden, out_logits);
  });
}

int clef_forward_device(void* handle, const ClefBatch* batch, float* out_logits, void* stream) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && batch && out_logits, "null argument");
    if (!m->finalized) throw Error(CLEF_ESTATE, "clef_forward_device before clef_finalize");
    m->forward_device(*batch, out_logits, static_cast<cudaStream_t>(stream));
  });
}

int clef_reserve(void* handle, int b, int s, int lx, int o, int q) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m, "null handle");
    m->reserve_all(b, s, lx, o, q);
  });
}

int clef_workspace_allocations(void* handle, int64_t* count) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m && count, "null handle or output");
    *count = m->ws_allocations;
  });
}

int clef_check_status(void* handle) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m, "null handle");
    CUDA_CHECK(cudaSetDevice(m->device));
    CUDA_CHECK(cudaDeviceSynchronize());
    m->check_status();
  });
}

int clef_set_debug(void* handle, int flags) {
  Model* m = static_cast<Model*>(handle);
  return guarded(m, [&] {
    REQUIRE(m, "null handle");
    REQUIRE((flags & ~CLEF_DEBUG_POISON) == 0, "unknown debug flag");
    m->debug_flags = flags;
  });
}

int clef_last_launch_count(void* handle) {
  Model* m = static_cast<Model*>(handle);
  return m ? m->last_launches : -1;
}

int clef_destroy(void* handle) {
  Model* m = static_cast<Model*>(handle);
  return guarded(nullptr, [&] {
    // After a TP timeout a collective may still wait on the stream: freeing
    // its buffers or destroying its communicator would block behind it (or
    // pull memory from under it), so the model is left for the process exit.
    if (m && m->broken) return;
    if (m) {
      cudaSetDevice(m->device);
      if (m->ws.host_pinned.p) {
        cudaFreeHost(m->ws.host_pinned.p);
        m->ws.host_pinned.p = nullptr;
      }
      delete m;
    }
  });
}

const char* clef_last_error(void* handle) {
  Model* m = static_cast<Model*>(handle);
  if (m) return m->last_error.c_str();
  std::lock_guard<std::mutex> lock(clef::g_error_mutex);
  static thread_local std::string copy;
  copy = clef::g_last_error;
  return copy.c_str();
}

// ---- kernel-level entry points ----

int clef_op_gemm(int dtype, int epi, int M, int N, int K, const void* A, const void* B, void* out, int ldo,
                 const void* bias, const void* residual, int ldr, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(A && B && out, "null operand");
    REQUIRE(epi >= 0 && epi <= 3, "epilogue must be 0..3");
    clef::Launcher L{static_cast<cudaStream_t>(stream), nullptr, 0};
    if (dtype == CLEF_DTYPE_BF16) {
      clef::gemm_bf16(L, epi, static_cast<const bf16*>(A), K, static_cast<const bf16*>(B), K, M, N, K, out, ldo,
                      static_cast<const bf16*>(bias), static_cast<const bf16*>(residual), ldr);
    } else if (dtype == CLEF_DTYPE_F32) {
      REQUIRE(epi != clef::kEpiSwiglu, "the F32 GEMM has no fused SwiGLU epilogue");
      const int simt_epi = epi == clef::kEpiStore ? clef::kSimtStore
                                                  : (epi == clef::kEpiResidual ? clef::kSimtResidual : clef::kSimtF32);
      clef::gemm_simt<float>(L, simt_epi, static_cast<const float*>(A), K, static_cast<const float*>(B), K, M, N, K, out,
                             ldo, static_cast<const float*>(bias), static_cast<const float*>(residual), ldr);
    } else {
      throw Error(CLEF_EINVAL, "bad dtype");
    }
  });
}

int clef_op_gemm_qkv(const void* A, const void* B, void* out, int M, int K, int hq, int hkv, int d,
                     float partial_rotary_factor, float rope_theta, int seq, const void* q_norm, const void* k_norm,
                     float eps, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(A && B && out && q_norm && k_norm && M > 0 && K > 0 && hq > 0 && hkv > 0 && d > 0 && seq > 0,
            "bad fused QKV GEMM arguments");
    const int rot = static_cast<int>(d * partial_rotary_factor);
    REQUIRE(rot > 0 && rot % 2 == 0 && rot <= d, "invalid partial rotary dimension");
    REQUIRE(M % seq == 0, "rows must be whole sequences of length seq");
    std::vector<float> cs, sn;
    clef::rope_tables(seq, rot, rope_theta, cs, sn);
    clef::DBuf dc, ds;
    dc.alloc(cs.size() * 4);
    ds.alloc(sn.size() * 4);
    CUDA_CHECK(cudaMemcpy(dc.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(ds.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    const int N = hq * 2 * d + 2 * hkv * d;
    clef::Launcher L{static_cast<cudaStream_t>(stream), nullptr, 0};
    const clef::QkvFusion f{static_cast<const bf16*>(q_norm), static_cast<const bf16*>(k_norm), dc.as<float>(),
                            ds.as<float>(), hq, hkv, d, rot, seq, eps};
    clef::gemm_bf16_qkv(L, static_cast<const bf16*>(A), K, static_cast<const bf16*>(B), K, M, N, K,
                        static_cast<bf16*>(out), N, f);
    CUDA_CHECK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));  // the tables are freed on return
  });
}

int clef_op_rmsnorm(int dtype, const void* x, const void* w, void* out, int rows, int dim, float eps, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(x && w && out && rows > 0 && dim > 0, "bad rmsnorm arguments");
    clef::Launcher L{static_cast<cudaStream_t>(stream), nullptr, 0};
    if (dtype == CLEF_DTYPE_BF16)
      clef::rmsnorm<bf16>(L, static_cast<const bf16*>(x), dim, static_cast<const bf16*>(w), static_cast<bf16*>(out), dim,
                          rows, dim, eps);
    else
      clef::rmsnorm<float>(L, static_cast<const float*>(x), dim, static_cast<const float*>(w), static_cast<float*>(out),
                           dim, rows, dim, eps);
  });
}

int clef_op_qk_norm_rope(int dtype, void* qkv, int b, int s, int hq, int hkv, int d, float partial_rotary_factor,
                         float rope_theta, const void* q_norm, const void* k_norm, float eps, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(qkv && q_norm && k_norm && b > 0 && s > 0 && hq > 0 && hkv > 0 && d > 0, "bad qk_norm_rope arguments");
    const int rot = static_cast<int>(d * partial_rotary_factor);
    REQUIRE(rot > 0 && rot % 2 == 0 && rot <= d, "invalid partial rotary dimension");
    // eight warps, one d-float row each, in the default 48 KB of dynamic shared memory
    REQUIRE(d <= clef::kQkRopeMaxHeadDim, "clef_op_qk_norm_rope supports head_dim <= 1536");
    std::vector<float> cs, sn;
    clef::rope_tables(s, rot, rope_theta, cs, sn);
    clef::DBuf dc, ds;
    dc.alloc(cs.size() * 4);
    ds.alloc(sn.size() * 4);
    CUDA_CHECK(cudaMemcpy(dc.p, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(ds.p, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice));
    const int ld = hq * 2 * d + 2 * hkv * d;
    const int Tt = b * s, warps = 8;
    const long long items = static_cast<long long>(Tt) * (hq + hkv);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == CLEF_DTYPE_BF16)
      clef::qk_norm_rope_kernel<bf16><<<static_cast<int>((items + warps - 1) / warps), warps * 32, warps * d * 4, st>>>(
          static_cast<bf16*>(qkv), ld, Tt, s, hq, hkv, d, rot, static_cast<const bf16*>(q_norm),
          static_cast<const bf16*>(k_norm), dc.as<float>(), ds.as<float>(), eps);
    else
      clef::qk_norm_rope_kernel<float><<<static_cast<int>((items + warps - 1) / warps), warps * 32, warps * d * 4, st>>>(
          static_cast<float*>(qkv), ld, Tt, s, hq, hkv, d, rot, static_cast<const float*>(q_norm),
          static_cast<const float*>(k_norm), dc.as<float>(), ds.as<float>(), eps);
    CUDA_CHECK(cudaGetLastError());
    CUDA_CHECK(cudaStreamSynchronize(st));  // the tables are freed on return
  });
}

int clef_op_attention(int dtype, const void* qkv, const uint8_t* mask, void* out, int b, int s, int hq, int hkv, int d,
                      float softcap, int window, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(qkv && out && b > 0 && s > 0 && hq > 0 && hkv > 0 && d > 0, "bad attention arguments");
    clef::Launcher L{static_cast<cudaStream_t>(stream), nullptr, 0};
    const long long ld = static_cast<long long>(hq) * 2 * d + 2LL * hkv * d;
    auto run = [&](auto* base) {
      using T = std::remove_const_t<std::remove_pointer_t<decltype(base)>>;
      clef::AttnArgs<T> a{};
      a.q = base;
      a.ldq = ld;
      a.hsq = 2 * d;
      a.k = base + static_cast<size_t>(hq) * 2 * d;
      a.ldk = ld;
      a.hsk = d;
      a.v = a.k + static_cast<size_t>(hkv) * d;
      a.ldv = ld;
      a.hsv = d;
      a.gate = base + d;
      a.ldg = ld;
      a.hsg = 2 * d;
      a.out = static_cast<T*>(out);
      a.ldo = static_cast<long long>(hq) * d;
      a.hso = d;
      a.key_mask = mask;
      a.B = b;
      a.Lq = s;
      a.Lk = s;
      a.H = hq;
      a.Hk = hkv;
      a.hd = d;
      a.causal = 1;
      a.softcap = softcap;
      a.window = window;
      a.status = nullptr;
      a.packed = 1;
      clef::attention<T>(L, a);
    };
    if (dtype == CLEF_DTYPE_BF16)
      run(static_cast<const bf16*>(qkv));
    else
      run(static_cast<const float*>(qkv));
  });
}

}  // extern "C"

namespace clef {
// A stream-ordered memory pool of this library per device, for the scratch of
// single-op entry points: it keeps its memory between calls (an allocation
// after a synchronize does not map the memory again), and other users of the
// device's default pool are not affected.  A device whose context was reset
// and rebuilt gets a new pool (detected by its default pool's handle).
static cudaMemPool_t op_scratch_pool(int device) {
  static std::mutex mu;
  static std::map<int, std::pair<cudaMemPool_t, cudaMemPool_t>> pools;  // device -> (default pool seen, ours)
  std::lock_guard<std::mutex> lock(mu);
  cudaMemPool_t def = nullptr;
  CUDA_CHECK(cudaDeviceGetDefaultMemPool(&def, device));
  auto it = pools.find(device);
  if (it != pools.end() && it->second.first == def) return it->second.second;
  cudaMemPoolProps props{};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = device;
  cudaMemPool_t pool = nullptr;
  CUDA_CHECK(cudaMemPoolCreate(&pool, &props));
  uint64_t keep = ~0ull;
  CUDA_CHECK(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
  pools[device] = {def, pool};
  return pool;
}
}  // namespace clef

extern "C" {

int clef_op_gdn_core(int dtype, const void* proj, int ldp, const void* conv, int width, const void* A_log,
                     const void* dt_bias, const void* norm_w, void* out, int b, int s, int nh, int nv, int dh, float eps,
                     void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(proj && conv && A_log && dt_bias && norm_w && out, "null Gated DeltaNet argument");
    REQUIRE(dtype == CLEF_DTYPE_BF16 || dtype == CLEF_DTYPE_F32, "dtype must be CLEF_DTYPE_BF16 or CLEF_DTYPE_F32");
    REQUIRE(nh > 0 && nv > 0 && dh > 0 && nv % nh == 0, "Gated DeltaNet value heads must divide into key head groups");
    const long long need = 2LL * nh * dh + 2LL * nv * dh + 2LL * nv;
    REQUIRE(ldp >= need, "ldp is smaller than the packed projection width");
    const int vec = dtype == CLEF_DTYPE_BF16 ? 8 : 4;
    REQUIRE(ldp % vec == 0 && (reinterpret_cast<uintptr_t>(proj) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0,
            "Gated DeltaNet rows must be 16-byte aligned (ldp a multiple of 16 bytes)");
    clef::Launcher L{static_cast<cudaStream_t>(stream), nullptr, 0};
    clef::GdnArgs a{};
    a.proj = proj;
    a.ldp = ldp;
    a.k_col = nh * dh;
    a.v_col = 2 * nh * dh;
    a.z_col = a.v_col + nv * dh;
    a.a_col = a.z_col + nv * dh;
    a.b_col = a.a_col + nv;
    a.conv = conv;
    a.width = width;
    a.A_log = A_log;
    a.dt_bias = dt_bias;
    a.norm_w = norm_w;
    a.out = out;
    a.ldo = static_cast<long long>(nv) * dh;
    a.B = b;
    a.S = s;
    a.nh = nh;
    a.nv = nv;
    a.qscale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(dh)));
    a.eps = eps;
    if (dtype == CLEF_DTYPE_BF16 && dh == 128) {
      // the tensor-core passes' scratch, stream-ordered: allocated and freed on the caller's stream
      void* scratch = nullptr;
      const size_t bytes = clef::gdn_tc_scratch_bytes(b, s, nh, nv);
      CUDA_CHECK(cudaMallocFromPoolAsync(&scratch, bytes, clef::op_scratch_pool(clef::current_device()), L.stream));
      clef::gdn_tc_bind_scratch(a, scratch);
      try {
        clef::launch_gdn<bf16>(L, a, dh);
      } catch (...) {
        cudaFreeAsync(scratch, L.stream);
        throw;
      }
      CUDA_CHECK(cudaFreeAsync(scratch, L.stream));
    } else if (dtype == CLEF_DTYPE_BF16) {
      clef::launch_gdn<bf16>(L, a, dh);
    } else {
      clef::launch_gdn<float>(L, a, dh);
    }
  });
}

}  // extern "C"

// ===========================================================================
// Allocation-free variant of clef_op_qk_norm_rope
// ===========================================================================
//
// clef_op_qk_norm_rope builds its cos/sin tables in freshly allocated device
// memory on every call.  Some callers cannot allocate device memory: a host
// framework that owns every device buffer (an XLA/JAX FFI custom call gets
// its inputs, outputs and workspace from XLA), or a serving loop that must not
// run cudaMalloc/cudaFree because they can synchronise the whole device.  For
// them, clef_op_qk_norm_rope_noalloc keeps the tables in a fixed array in the
// library's own device memory instead.

namespace clef {

// cos table followed by sin table, each up to kNoAllocRopeEntries floats
// (positions x rot/2): 2 x 4 MiB, resident on every GPU that loads the library.
constexpr int kNoAllocRopeEntries = 1 << 20;
static __device__ __align__(256) float g_noalloc_rope[2 * kNoAllocRopeEntries];

struct RopeFreqs {
  float inv[128];  // inverse frequencies, rot/2 <= 128 (head_dim <= 256)
};

// Fill cos/sin [s, half] from float32 angles pos * inv_freq, evaluated in
// double precision like the host tables of clef_op_qk_norm_rope.
__global__ void noalloc_rope_table_kernel(float* __restrict__ cos_t, float* __restrict__ sin_t, int s, int half,
                                          RopeFreqs f) {
  const long long n = static_cast<long long>(s) * half;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int p = static_cast<int>(i / half), j = static_cast<int>(i % half);
    const float ang = static_cast<float>(p) * f.inv[j];
    cos_t[i] = static_cast<float>(cos(static_cast<double>(ang)));
    sin_t[i] = static_cast<float>(sin(static_cast<double>(ang)));
  }
}

// Device address of g_noalloc_rope on the current device.  The array's
// host-side name is not a device address; cudaGetSymbolAddress, called with
// the device current, gives it (the first call on a device loads the module
// there).  Outside stream capture the address is looked up afresh on every
// call, so a context that was reset and rebuilt (cudaDeviceReset) yields its
// new address; while `st` is being captured the address last looked up on
// this device is used, since loading a module is not allowed during capture.
static float* noalloc_rope_scratch(int device, cudaStream_t st) {
  static std::mutex mu;
  static std::map<int, float*> addr;
  std::lock_guard<std::mutex> lock(mu);
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cap) != cudaSuccess) {
    (void)cudaGetLastError();  // a legacy-stream query during another stream's capture: treat as capturing
    cap = cudaStreamCaptureStatusActive;
  }
  if (cap != cudaStreamCaptureStatusNone) {
    auto it = addr.find(device);
    REQUIRE(it != addr.end(),
            "clef_op_qk_norm_rope_noalloc: make one call on this device outside stream capture first");
    return it->second;
  }
  float* p = nullptr;
  CUDA_CHECK(cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_noalloc_rope));
  addr[device] = p;
  return p;
}

}  // namespace clef

extern "C" int clef_op_qk_norm_rope_noalloc(int dtype, void* qkv, int b, int s, int hq, int hkv, int d,
                                            float partial_rotary_factor, float rope_theta, const void* q_norm,
                                            const void* k_norm, float eps, void* stream) {
  return guarded(nullptr, [&] {
    REQUIRE(qkv && q_norm && k_norm && b > 0 && s > 0 && hq > 0 && hkv > 0 && d > 0, "bad qk_norm_rope arguments");
    REQUIRE(dtype == CLEF_DTYPE_BF16 || dtype == CLEF_DTYPE_F32, "bad dtype");
    const int rot = static_cast<int>(d * partial_rotary_factor);
    REQUIRE(rot > 0 && rot % 2 == 0 && rot <= d, "invalid partial rotary dimension");
    const int half = rot / 2;
    REQUIRE(half <= 128, "clef_op_qk_norm_rope_noalloc supports rot/2 <= 128 (head_dim <= 256)");
    REQUIRE(d <= clef::kQkRopeMaxHeadDim, "clef_op_qk_norm_rope_noalloc supports head_dim <= 1536");
    REQUIRE(static_cast<long long>(s) * half <= clef::kNoAllocRopeEntries,
            "clef_op_qk_norm_rope_noalloc: seq_len * rot/2 exceeds its fixed table of 1048576 entries");
    const int device = clef::current_device();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* cos_t = clef::noalloc_rope_scratch(device, st);
    float* sin_t = cos_t + clef::kNoAllocRopeEntries;
    clef::RopeFreqs f{};
    for (int i = 0; i < half; ++i)
      f.inv[i] = 1.0f / powf(rope_theta, static_cast<float>(2 * i) / static_cast<float>(rot));
    const long long n = static_cast<long long>(s) * half;
    clef::noalloc_rope_table_kernel<<<static_cast<int>(std::min<long long>((n + 255) / 256, 1024)), 256, 0, st>>>(
        cos_t, sin_t, s, half, f);
    CUDA_CHECK(cudaGetLastError());
    const int ld = hq * 2 * d + 2 * hkv * d;
    const int Tt = b * s, warps = 8;
    const long long items = static_cast<long long>(Tt) * (hq + hkv);
    const int grid = static_cast<int>((items + warps - 1) / warps);
    if (dtype == CLEF_DTYPE_BF16)
      clef::qk_norm_rope_kernel<bf16><<<grid, warps * 32, warps * d * 4, st>>>(
          static_cast<bf16*>(qkv), ld, Tt, s, hq, hkv, d, rot, static_cast<const bf16*>(q_norm),
          static_cast<const bf16*>(k_norm), cos_t, sin_t, eps);
    else
      clef::qk_norm_rope_kernel<float><<<grid, warps * 32, warps * d * 4, st>>>(
          static_cast<float*>(qkv), ld, Tt, s, hq, hkv, d, rot, static_cast<const float*>(q_norm),
          static_cast<const float*>(k_norm), cos_t, sin_t, eps);
    CUDA_CHECK(cudaGetLastError());
  });
}

/*
 * clef_b200.h -- C ABI of libclef_b200.so, the B200 (sm_100a) implementation of
 * deciax's Clef prefill-and-score path.
 *
 * The library replaces the device side of `ClefModel` in the reference
 * (src/deciax/models/clef/model.py:30-102): weight placement
 * (models/clef/weights.py:70-101), the per-layer forward (models/qwen3_5/text.py:94-102
 * and its Pallas TP form models/qwen3_5/pallas.py:132-150), the final norm,
 * the lexical option means and the joint schema head (models/clef/head.py:50-107).
 * Host code keeps tokenisation, collate and decode (models/clef/input.py).
 *
 * Conventions
 *  - Every function returns 0 on success or a CLEF_E* status; clef_last_error()
 *    gives a message.  CLEF_EINVAL marks bad shapes/config/names (the reference
 *    raises ValueError there -> HTTP 422); CLEF_ECUDA / CLEF_ENCCL / CLEF_EDEVICE
 *    mark device failures (RuntimeError -> HTTP 500).
 *  - Plain pointers and sizes only.  Host buffers are caller-owned.
 *  - One handle drives one GPU (one tensor-parallel rank).  Calls on one handle
 *    must be serialised by the caller (the reference's ClefEngine holds a lock,
 *    runtime/clef.py:21,36); distinct handles are independent.
 */
#ifndef CLEF_B200_H
#define CLEF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CLEF_OK 0
#define CLEF_EINVAL 1   /* bad argument, shape, name or configuration */
#define CLEF_ECUDA 2    /* CUDA runtime error */
#define CLEF_ENCCL 3    /* NCCL error */
#define CLEF_EDEVICE 4  /* a kernel reported a device-side status (timeout, bad index) */
#define CLEF_ESTATE 5   /* call out of order (e.g. forward before finalize) */

#define CLEF_DTYPE_F32 0
#define CLEF_DTYPE_BF16 1

#define CLEF_LAYER_FULL_ATTENTION 0
#define CLEF_LAYER_LINEAR_ATTENTION 1

/* Model configuration: the reference TextConfig (models/qwen3_5/config.py:10-75)
 * plus joint_head_config.json (models/clef/model.py:80-83).  The three
 * beyond-reference fields default to 0 = off = reference semantics. */
typedef struct ClefConfig {
  int32_t hidden_size;           /* D */
  int32_t intermediate_size;     /* F */
  int32_t num_attention_heads;   /* Hq */
  int32_t num_key_value_heads;   /* Hkv */
  int32_t head_dim;              /* d */
  int32_t num_layers;
  const int32_t* layer_types;    /* [num_layers] CLEF_LAYER_*; NULL = all full attention */
  int32_t vocab_size;
  float rms_norm_eps;
  float rope_theta;
  float partial_rotary_factor;
  int32_t max_seq_len;           /* longest sequence a forward may use (RoPE table) */
  /* joint schema head */
  int32_t head_width;            /* W */
  int32_t head_heads;
  int32_t head_routing_layers;
  int32_t head_layers;
  int32_t head_ffn;              /* rows of feedforward.0 / linear1 */
  /* beyond-reference options (not in deciax; 0 = off) */
  float attn_softcap;            /* softcap * tanh(score / softcap) on attention scores */
  const int32_t* layer_window;   /* [num_layers] causal window per layer, 0 = global; NULL = all global */
  float embed_scale;             /* multiply embeddings by this in the activation dtype */
  /* Gated DeltaNet, the mixer of linear_attention layers (models/qwen3_5/text.py:42-67,
   * config.py:15-19); read only when some layer is linear. */
  int32_t linear_num_key_heads;
  int32_t linear_num_value_heads;
  int32_t linear_key_head_dim;   /* must equal linear_value_head_dim, one of 8, 16, 32, 64, 128 */
  int32_t linear_value_head_dim;
  int32_t linear_conv_kernel_dim; /* depthwise causal conv width, 1..8 */
  /* Tensor parallelism only: the longest host wait, in milliseconds, for the
   * other ranks -- communicator creation and each clef_forward.  0 = no limit.
   * A rank that never joins makes clef_create fail with CLEF_ENCCL (the
   * communicator is aborted); a forward that does not finish in time returns
   * CLEF_ENCCL and leaves the handle unusable (CLEF_ESTATE on every later
   * call; clef_destroy then releases nothing on the device, since a collective
   * may still be waiting on the stream -- end the process). */
  int32_t tp_timeout_ms;
} ClefConfig;

/* One collated batch: the dict returned by the reference collate()
 * (models/clef/input.py:140-182).  Shapes: b rows, s sequence bucket,
 * lx lexical length, o option bucket, q question bucket. */
typedef struct ClefBatch {
  int32_t b, s, lx, o, q;
  const int32_t* input_ids;       /* [b, s] */
  const uint8_t* mask;            /* [b, s] 0/1 */
  const int32_t* lexical_ids;     /* [b, lx] */
  const int32_t* lexical_spans;   /* [b, o, 2] */
  const int32_t* question_spans;  /* [b, q, 2] */
  const uint8_t* question_mask;   /* [b, q] */
  const int32_t* types;           /* [b, q] */
  const int32_t* option_spans;    /* [b, o, 2] */
  const uint8_t* option_mask;     /* [b, o] */
  const int32_t* option_field;    /* [b, o] */
} ClefBatch;

/* ---- model lifecycle: replaces ClefModel.__init__ (models/clef/model.py:34-85) ---- */

/* Size of an NCCL unique id; rank 0 makes one, every rank passes the same bytes. */
#define CLEF_NCCL_ID_BYTES 128
int clef_nccl_unique_id(uint8_t out[CLEF_NCCL_ID_BYTES]);

/* Create a model on `device` as tensor-parallel rank tp_rank of tp_size
 * (mesh of models/clef/model.py:59-63; heads and MLP columns sharded as
 * models/clef/weights.py:60-67).  nccl_id may be NULL when tp_size == 1.
 * dtype: CLEF_DTYPE_BF16 (serving) or CLEF_DTYPE_F32 (parity). */
int clef_create(const ClefConfig* config, int device, int tp_rank, int tp_size, const uint8_t* nccl_id, int dtype,
                void** handle);

/* Upload one tensor from host memory (models/clef/weights.py:70-101).  The
 * library converts to the compute dtype, keeps this rank's shard and packs it.
 * Names: "embedding", "lm_head", "norm",
 *   "layers.{i}.{input_layernorm,post_attention_layernorm}.weight",
 *   "layers.{i}.mixer.{q_proj,k_proj,v_proj,o_proj,q_norm,k_norm}.weight" (full_attention),
 *   "layers.{i}.mixer.{q,k,v,in_proj_z,in_proj_a,in_proj_b,out_proj,norm}.weight",
 *   "layers.{i}.mixer.{q,k,v}.conv", "layers.{i}.mixer.{A_log,dt_bias}" (linear_attention:
 *   the names after the in_proj_qkv / conv1d split of models/clef/weights.py:43-57),
 *   "layers.{i}.mlp.{gate_proj,up_proj,down_proj}.weight",
 *   "head.<joint_head.safetensors key>".
 * host_dtype: CLEF_DTYPE_F32 or CLEF_DTYPE_BF16 (raw bfloat16 bits). */
int clef_upload(void* handle, const char* name, const void* host, int host_dtype, const int64_t* shape, int ndim);

/* As clef_upload, with the source already in device memory of this handle's
 * GPU and in the compute dtype (weights created or loaded on the device). */
int clef_upload_device(void* handle, const char* name, const void* device_ptr, int dtype, const int64_t* shape,
                       int ndim);

/* Check every tensor is present and build the packed layouts. */
int clef_finalize(void* handle);

/* ClefModel.forward (models/clef/model.py:92-102): host batch in, option
 * logits [b, o] float32 out (host).  out_hidden, if not NULL, receives the
 * final-normed hidden states [b, s, hidden] as float32.  All ranks of a TP
 * group must call it with the same batch. */
int clef_forward(void* handle, const ClefBatch* batch, float* out_logits, float* out_hidden);

/* Lexical means + joint head only (models/clef/model.py:100-102,
 * models/clef/head.py:50-107) on caller-supplied final-normed hidden states
 * [b, s, hidden] float32 (host) -- the input of the reference's joint-head
 * fixture test (tests/clef/test_head.py:11-29). */
int clef_forward_head(void* handle, const ClefBatch* batch, const float* hidden, float* out_logits);

/* Same computation with every ClefBatch pointer and out_logits in device
 * memory of this handle's GPU, enqueued on `stream` (a cudaStream_t; NULL =
 * the library's stream).  No host synchronisation and no allocation once the
 * workspace for this shape exists (see clef_reserve). */
int clef_forward_device(void* handle, const ClefBatch* batch, float* out_logits, void* stream);

/* Allocate the workspace for batches up to (b, s, lx, o, q) ahead of time:
 * the device buffers of a forward and the pinned host staging of
 * clef_forward (under TP, also the exchange of the ranks' peer-memory
 * handles, so every rank must call it with the same shape).  Sizes only grow;
 * a later forward within every reserved maximum allocates nothing.  A
 * serving warm-up calls it for the largest batch it admits -- the
 * counterpart of the reference server's warm-up request
 * (serve/app.py:385-406), which the library turns into one reservation of
 * the whole admitted range instead of one small shape. */
int clef_reserve(void* handle, int b, int s, int lx, int o, int q);

/* Number of workspace allocations since clef_create: device buffers grown,
 * pinned staging grown, and TP peer-handle exchanges (each follows a move of
 * the buffers peers write into).  Lets a caller check that its warm-up
 * reserved enough.  No counterpart in the reference (XLA allocates inside
 * each jitted call). */
int clef_workspace_allocations(void* handle, int64_t* count);

/* Synchronise the device and report (then clear) any device-side status a
 * kernel recorded since the last check (CLEF_EDEVICE: wait timeout or an
 * out-of-range token id).  clef_forward does this itself. */
int clef_check_status(void* handle);

/* Per-kernel device timing.  While enabled, every forward records a CUDA
 * event after each launch on its stream; clef_timing_report synchronises and
 * returns, per category, the summed milliseconds and launch count since the
 * last report (then resets).  Categories: 0 embedding, 1 RMSNorm, 2 QKV GEMM,
 * 3 q/k-norm+RoPE, 4 attention, 5 o-proj GEMM, 6 gate/up GEMM, 7 down GEMM,
 * 8 NCCL all-reduce, 9 TP residual add, 10 lexical means + joint head,
 * 11 other, 12 Gated DeltaNet core (linear_attention layers; their input
 * projection counts as 2 and their output projection as 5). */
#define CLEF_TIMING_CATEGORIES 13
int clef_set_timing(void* handle, int enable);
int clef_timing_report(void* handle, int n, float* ms, int* launches);

/* Number of kernels the last forward launched (for launch accounting). */
int clef_last_launch_count(void* handle);

/* Debug switches (bit flags, 0 = off).  CLEF_DEBUG_POISON: before every
 * forward, fill the forward's scratch buffers (activations, projections,
 * head buffers, FP32 partials) with 0xFF bytes -- NaN in bf16 and fp32 -- so
 * that a kernel reading memory it has not written first shows up as NaN or
 * changed logits.  A sanitizer substitute for testing; it costs one memset
 * per buffer per forward.  The reference has no counterpart. */
#define CLEF_DEBUG_POISON 1
int clef_set_debug(void* handle, int flags);

int clef_destroy(void* handle);

/* Message of the last failure on this handle (or of the last global failure when NULL). */
const char* clef_last_error(void* handle);

/* ---- kernel-level entry points (device pointers; used by the parity tests) ----
 * All run on `stream` (cudaStream_t, NULL = default stream) on the current device
 * and return CLEF_E* status after checking arguments. */

/* C[M,N] = A[M,K] B[N,K]^T with a fused epilogue (nn.py:11-19, text.py:21-22):
 * epi 0 store T(acc+bias) | 1 SwiGLU of packed [128 gate|128 up] blocks
 * (kernels/swiglu.py:100-101) | 2 residual T(res + T(acc)) | 3 float acc.
 * dtype BF16 runs the tcgen05 kernel, F32 the CUDA-core kernel. */
int clef_op_gemm(int dtype, int epi, int M, int N, int K, const void* A, const void* B, void* out, int ldo,
                 const void* bias, const void* residual, int ldr, void* stream);

/* The QKV projection with its fused epilogue, bf16 (tcgen05): out[M, N] with
 * N = hq*2d + 2*hkv*d = A[M,K] B[N,K]^T where each query head's q and each
 * key head leave RMSNorm(1+w)-normalised with partial RoPE at positions
 * row % seq (models/qwen3_5/text.py:79-88), each gate leaves as
 * T(sigmoid(T(gate))) (text.py:91) and v is unchanged.  Needs d in
 * {64, 128, 256} and d * partial_rotary_factor equal to 32 or a multiple of 64. */
int clef_op_gemm_qkv(const void* A, const void* B, void* out, int M, int K, int hq, int hkv, int d,
                     float partial_rotary_factor, float rope_theta, int seq, const void* q_norm, const void* k_norm,
                     float eps, void* stream);

/* RMSNorm scaling by (1 + w) (models/qwen3_5/text.py:25-28). */
int clef_op_rmsnorm(int dtype, const void* x, const void* w, void* out, int rows, int dim, float eps, void* stream);

/* In-place per-head q/k RMSNorm + partial RoPE on a packed projection
 * [b*s, Hq*2d + 2*Hkv*d] (models/qwen3_5/text.py:79-88, nn.py:31-44).
 * head_dim <= 1536. */
int clef_op_qk_norm_rope(int dtype, void* qkv, int b, int s, int hq, int hkv, int d, float partial_rotary_factor,
                         float rope_theta, const void* q_norm, const void* k_norm, float eps, void* stream);

/* Allocation-free form of clef_op_qk_norm_rope (no counterpart in the reference).
 * For callers that cannot allocate device memory themselves or through us: a
 * host framework that owns every device buffer (e.g. an XLA FFI custom call,
 * which receives all its memory from XLA), or a serving loop that must avoid
 * cudaMalloc/cudaFree because they may synchronise the device.  Same
 * arguments and result as clef_op_qk_norm_rope; the cos/sin tables live in a
 * fixed 8 MiB array inside the library (held on every GPU that loads it until
 * exit) instead of memory allocated per call.
 *  - Limit: s * rot/2 <= 1048576 table entries, rot/2 <= 128 and
 *    head_dim <= 1536 (rot = head_dim * partial_rotary_factor); larger sizes
 *    return CLEF_EINVAL before any device work.
 *  - Each call outside stream capture looks up the array's device address
 *    (cudaGetSymbolAddress) with the device current, so a context that was
 *    reset and rebuilt gets its new address; the first such lookup on a
 *    device loads the module there.  Make one call on each device before any
 *    stream capture: during capture the last address looked up is used.
 *  - Every call rewrites the table entries it reads, so no state carries over
 *    between calls, but all calls on a device share the one array: calls whose
 *    kernels overlap on the GPU (e.g. on two streams) race. */
int clef_op_qk_norm_rope_noalloc(int dtype, void* qkv, int b, int s, int hq, int hkv, int d,
                                 float partial_rotary_factor, float rope_theta, const void* q_norm, const void* k_norm,
                                 float eps, void* stream);

/* Causal GQA attention with the sigmoid output gate over a packed projection
 * (kernels/attention/blocked.py:9-32, text.py:90-91): out [b*s, Hq*d]. */
int clef_op_attention(int dtype, const void* qkv, const uint8_t* mask, void* out, int b, int s, int hq, int hkv, int d,
                      float softcap, int window, void* stream);

/* Gated DeltaNet core, delta_net_core of models/qwen3_5/text.py:48-67 with the
 * chunked rule of kernels/gdn/reference.py:40-92: from the projections
 * proj [b*s, ldp] = [q (nh*dh) | k (nh*dh) | v (nv*dh) | z (nv*dh) | a (nv) | b (nv)]
 * (the outputs of the q, k, v, in_proj_z, in_proj_a, in_proj_b dense layers, in
 * that column order) to the gated, normalised output out [b*s, nv*dh] that
 * feeds out_proj.  conv [2*nh*dh + nv*dh, width] holds the q, k and v conv
 * rows; A_log, dt_bias [nv]; norm_w [dh].  dh = key = value head dim, one of
 * 8, 16, 32, 64, 128; nv % nh == 0; width 1..8; proj and out 16-byte aligned
 * and ldp * element size a multiple of 16 bytes. */
int clef_op_gdn_core(int dtype, const void* proj, int ldp, const void* conv, int width, const void* A_log,
                     const void* dt_bias, const void* norm_w, void* out, int b, int s, int nh, int nv, int dh, float eps,
                     void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CLEF_B200_H */

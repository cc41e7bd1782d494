/*
 * libjitcast_b200 — the C ABI of the B200 forward-pass GEMM engine.
 *
 * Plain C types only (pointers, sizes, enums, POD structs), so that Java 22+ can bind every
 * entry point with the Panama FFM API (Linker.nativeLinker().downcallHandle) and Python with
 * ctypes. No exception or abort crosses the ABI: every entry point returns a jc_status, and
 * jc_last_error() holds the calling thread's last message.
 *
 * Reference interfaces replaced (paths in the jitCast source tree, src/main/java/ai/beestream/jitcast/):
 *   - cpu/Ops.java:33-51            Ops.linear (y = x·Wᵀ + b)                → jc_linear
 *   - tornado/Kernels.java:50-102   Kernels.gemm and its flags             → jc_linear, jc_linear_device
 *   - tornado/GemmMode.java:40-77   GemmMode (FP32 / TF32 / FP16 cuBLAS)   → jc_precision
 *   - timestral/BlockForward.java:20-24 and timestral/tornado/TimestralForward.java:187-642
 *       BlockForward.predictBlock's device forward (TimestralForward)   → jc_engine_create_timestral,
 *                                                                          jc_forward_timestral
 *   - timestral/BlockPrep.java:40-101 BlockPrep.of / BlockPrep.finish   → jc_forecast_timestral (the
 *       host ends on the GPU around the same forward)
 *   - chronos2/ModelForward.java and chronos2/tornado/Chronos2Forward.java:148-494
 *       ModelForward.forward's device forward (Chronos2Forward)         → jc_engine_create_chronos2,
 *                                                                          jc_forward_chronos2
 *   - chronos2/ModelPrep.java:29-137 ModelPrep.of / ModelPrep.finish    → jc_forecast_chronos2 (the
 *       host ends on the GPU around the same forward)
 *   - tirex2/ForwardPass.java and tirex2/tornado/TornadoForward.java:353-827
 *       ForwardPass.forward's device forward (TornadoForward)           → jc_engine_create_tirex2,
 *                                                                          jc_forward_tirex2
 *   - tornado/PlanCache.java:40-162  per-shape plans, CUDA-graph replay → engine plans, jc_engine_set_option
 */
#ifndef JITCAST_B200_H
#define JITCAST_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The reference fails fast with IllegalArgumentException / IllegalStateException
 * (docs/CONFIGURATION.md, PlanCache.java:70-100); a Java binding maps INVALID_ARG and
 * UNSUPPORTED_SHAPE to IllegalArgumentException and the rest to IllegalStateException. */
typedef enum jc_status {
  JC_OK = 0,
  JC_ERR_INVALID_ARG = 1,
  JC_ERR_UNSUPPORTED_SHAPE = 2,
  JC_ERR_OOM = 3,
  JC_ERR_CUDA = 4,
  JC_ERR_TIMEOUT = 5,
  JC_ERR_INTERNAL = 6,
  JC_ERR_NO_DEVICE = 7
} jc_status;

/* Arithmetic of the tensor-core GEMMs (replaces tornado/GemmMode.java:40-41).
 *   JC_FP32  FP32 operands as TF32 hi/lo pairs, four TF32 MMAs per product (≈ FP32 accuracy)
 *   JC_TF32  TF32 operands, FP32 accumulation (the reference's CUBLAS_TF32)
 *   JC_BF16  BF16 operands, FP32 accumulation and FP32 residual stream
 *   JC_FP16  FP16 operands (stores saturate at ±65504, as Kernels.HALF_MAX), FP32 accumulation and
 *            FP32 residual stream (the reference's CUBLAS_FP16 / gemmHalf, fused) */
typedef enum jc_precision { JC_FP32 = 0, JC_TF32 = 1, JC_BF16 = 2, JC_FP16 = 3 } jc_precision;

/* GEMM epilogue flags: the values of tornado/Kernels.java:50-56, plus GELU.
 * Order as Kernels.gemm (Kernels.java:86-100): bias, then SiLU and/or ReLU (or GELU), then += C. */
#define JC_BIAS 1
#define JC_ACCUMULATE 2
#define JC_SILU 4
#define JC_TWIN_ONLY 8 /* FP16-twin-only output of gemmHalf; not meaningful for FP32 C: rejected */
#define JC_RELU 16
#define JC_GELU 32

/* Library version string, e.g. "jitcast_b200 0.1.0 (sm_100a)". */
const char* jc_version(void);

/* The calling thread's last error message ("" if none). Valid until the thread's next call. */
const char* jc_last_error(void);

/* Number of CUDA devices visible to the library (0 without a GPU). */
int jc_device_count(void);

/*
 * C[m, n] (+)= act(A[m, :] · W[n, :] + b[n]) on HOST buffers, with the flags of Kernels.gemm
 * (tornado/Kernels.java:59-102) and the operator of Ops.linear (cpu/Ops.java:33-51):
 *   a    [m, k] row-major FP32          w [n, k] row-major FP32 (PyTorch [out, in])
 *   bias [n] FP32, read when flags has JC_BIAS (may be NULL otherwise)
 *   c    [m, n] row-major FP32, read when flags has JC_ACCUMULATE, always written.
 * The call uploads, runs one tcgen05 GEMM on `device` with the epilogue fused, downloads
 * C and returns when C is written. Thread-safe; calls on one device are serialised.
 * Ragged m, n, k are fine (inputs are zero-padded on the device).
 */
jc_status jc_linear(int device, jc_precision precision, const float* a, const float* w, const float* bias, float* c,
                    int m, int n, int k, int flags);

/*
 * The same operation on DEVICE buffers that stay resident in HBM, enqueued on `stream`
 * (a cudaStream_t, NULL = the legacy default stream) without synchronising:
 *   a [m, k] FP32 (row pitch lda), w [n, k] FP32 (row pitch ldw), bias [n] FP32, c [m, n] FP32 (row pitch ldc).
 * A and W are converted to the precision's operand format in library-owned scratch memory
 * (grown on demand and reused; the call synchronises `stream` before it grows), then one
 * GEMM runs with the epilogue fused. Kernel-side errors (a bounded wait that gave up) are
 * reported by the next jc_device_sync on the device.
 */
jc_status jc_linear_device(int device, jc_precision precision, const float* a, long long lda, const float* w,
                           long long ldw, const float* bias, float* c, long long ldc, int m, int n, int k, int flags,
                           void* stream);

/*
 * jc_linear_device for callers that cannot allocate GPU memory once they are running: code that has
 * handed the GPU to a fixed arena or memory budget (where a cudaMalloc could fail or stall between
 * steps), or that must not call cudaMalloc / cudaFree because those can synchronise the device.
 * This entry point has no counterpart in the reference.
 *
 * Same arguments and result as jc_linear_device, but the converted operands go into a fixed scratch
 * array compiled into the library (16 MiB on every GPU that loads the library, held until the
 * process exits) instead of memory allocated on demand, and nothing in the call allocates.
 *   - (m + n) x round_up(k, 64) operands must fit: 2 bytes per element for JC_BF16 and JC_FP16, 4
 *     for JC_TF32, 8 for JC_FP32 (hi and lo). Larger shapes fail with JC_ERR_UNSUPPORTED_SHAPE.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 *     that device current. Under CUDA's lazy module loading (the default since CUDA 12.2) that first
 *     use of the library on a device is also what loads its module there and reserves the 16 MiB.
 *     So make one call on each device at start-up: before any stream capture, and before the caller
 *     sizes its arena from the free memory.
 *   - Calls on one device are serialised (they share that device's array); calls on different
 *     devices run side by side.
 *   - Every call on a device shares that device's array and it keeps the last call's contents; the
 *     operands are fully rewritten by each call. Calls that overlapped on the GPU would race on it,
 *     so each call waits for its own kernels on `stream` before it returns.
 *   - Returns JC_ERR_TIMEOUT if a bounded wait inside the GEMM gave up.
 */
jc_status jc_linear_device_noalloc(int device, jc_precision precision, const float* a, long long lda, const float* w,
                                   long long ldw, const float* bias, float* c, long long ldc, int m, int n, int k,
                                   int flags, void* stream);

/*
 * The GEMM on DEVICE operands already in the precision's storage format, with no conversion and
 * no scratch memory (the form the engine's own layers use):
 *   JC_BF16  a_hi [m, k] and w_hi [n, k] bfloat16; a_lo and w_lo unused (NULL)
 *   JC_TF32  a_hi, w_hi FP32 holding TF32 values; a_lo, w_lo unused
 *   JC_FP32  a_hi, w_hi TF32 parts and a_lo, w_lo FP32 remainders (x = hi + lo)
 * lda and ldw are row pitches in elements (pitch × element size a multiple of 16 bytes, base
 * addresses 16-byte aligned). bias, c and flags as jc_linear_device. Enqueued on `stream`.
 * Replaces the reference's per-mode GEMM dispatch (timestral/tornado/TimestralForward.java:404-499).
 */
jc_status jc_gemm_device(int device, jc_precision precision, const void* a_hi, const void* a_lo, long long lda,
                         const void* w_hi, const void* w_lo, long long ldw, const float* bias, float* c,
                         long long ldc, int m, int n, int k, int flags, void* stream);

/* One GEMM of a group (jc_gemm_group_device): the arguments of jc_gemm_device after the precision. */
typedef struct jc_gemm_problem {
  const void* a_hi;
  const void* a_lo;
  long long lda;
  const void* w_hi;
  const void* w_lo;
  long long ldw;
  const float* bias;
  float* c;
  long long ldc;
  int m, n, k;
  int flags;
} jc_gemm_problem;

/*
 * 1 to 4 independent GEMMs of one precision as ONE persistent launch on DEVICE operands (each problem as
 * jc_gemm_device: operands in the precision's storage format, its own shape, bias, flags and C), enqueued
 * on `stream`. Every problem's tiles run in one walk over the SMs; the results equal one jc_gemm_device call
 * per problem bit for bit. No problem may write what another reads. Replaces the reference's per-head gate
 * GEMMs of the sLSTM (tirex2/tornado/TornadoForward.java:730, one launch over the dense block-diagonal
 * packing of tirex2/tornado/PackedWeights.java:242-254) and runs independent projections of one input
 * together (timestral/tornado/TimestralForward.java:327, the patch embedding's hidden and residual).
 */
jc_status jc_gemm_group_device(int device, jc_precision precision, const jc_gemm_problem* problems, int count,
                               void* stream);

/*
 * Time attention of one layer on DEVICE buffers, the companion kernel of the Timestral and Chronos-2
 * forwards (timestral/tornado/TimestralKernels.java:114 timeAttention, chronos2/tornado/Chronos2Kernels.java:130
 * timeAttention), enqueued on `stream`:
 *   qkv  [rows·n, ld_qkv]: q | k | v at columns 0, d, 2d, heads-major (head h at h·head_dim in each part)
 *   gate [rows·n, ld_gate] multiplied into the output (NULL: none), out [rows·n, ld_out]
 * in the precision's storage type (bfloat16 for JC_BF16, IEEE half for JC_FP16, FP32 otherwise).
 * out = softmax(scale · q·kᵀ over the allowed keys) · v (· gate), per row, head and query (zeros for a query
 * with no allowed key), with
 *   mask_mode 0: BlockLayout.timeAllowed (timestral/BlockLayout.java:209-221): encoder queries (< enc) see
 *                themselves and valid encoder keys up to themselves, or all valid encoder keys when the row
 *                is a known covariate; decoder queries see valid encoder keys < ll and decoder keys up to
 *                themselves. key_valid [rows·enc], known [rows] (0/1).
 *   mask_mode 1: every live key in both directions (Chronos-2's ModelLayout.live), live [rows·n] (0/1).
 * 16-bit operands of 64-wide heads and n ≤ 256 run on the tcgen05 tensor cores; flags JC_ATTN_CUDA_CORES
 * forces the FP32-math CUDA-core kernel (a reference for comparisons).
 */
#define JC_ATTN_CUDA_CORES 1
jc_status jc_time_attention_device(int device, jc_precision precision, const void* qkv, long long ld_qkv,
                                   const void* gate, long long ld_gate, void* out, long long ld_out, int rows, int n,
                                   int heads, int head_dim, int d, float scale, int mask_mode, int enc, int ll,
                                   const int32_t* key_valid, const int32_t* known, const int32_t* live, int flags,
                                   void* stream);

/* Waits for all work on `device`, then returns and clears the device's kernel error word:
 * JC_ERR_TIMEOUT if a kernel's bounded wait gave up since the last call. */
jc_status jc_device_sync(int device);

/* ===================================================================================== */
/* Engines: a model's weights resident on one or more GPUs, and its forward pass.          */
/* ===================================================================================== */

/* One checkpoint tensor from the caller (the reference maps model.safetensors with FFM,
 * io/SafeTensors.java:49-70, and hands out MemorySegment views): FP32, row-major, contiguous. */
typedef struct jc_tensor_view {
  const char* name; /* checkpoint name, e.g. "transformer.layers.0.mlp.w3.weight" */
  const float* data;
  int ndim;
  int64_t shape[4];
} jc_tensor_view;

typedef struct jc_engine jc_engine;

/* Timestral layer kinds (block_schedule of timestral/TimestralConfig.java:173-182). */
#define JC_LAYER_TIME 0
#define JC_LAYER_VARIATE 1
#define JC_LAYER_TIME_VARIATE 2
#define JC_LAYER_VARIATE_TIME 3

/* The TimestralConfig fields the forward pass uses (timestral/TimestralConfig.java:53-71). */
typedef struct jc_timestral_desc {
  int patch_size;
  int d_model;
  int num_heads;
  int mlp_hidden_dim;
  int num_layers;
  const int32_t* layer_kinds; /* [num_layers] JC_LAYER_* */
  int num_quantiles;
  float rope_theta;
  float rope_partial_factor;
  float norm_eps;
  int time_attn_gate;
  int variate_attn_gate;
} jc_timestral_desc;

/*
 * Creates a Timestral engine: binds `weights` by the checkpoint's names and shapes (every tensor
 * exactly once, as timestral/TimestralWeights.java:83-115 does; an unknown, missing or misshapen
 * tensor fails with JC_ERR_INVALID_ARG), rearranges and converts them to `precision` on each of
 * the `n_devices` GPUs in `devices` (a full replica per GPU). The weights are copied; the
 * caller's buffers may be released when the call returns. Head widths other than 32 or 64 fail
 * with JC_ERR_UNSUPPORTED_SHAPE, as TimestralForward.java:163-166 rejects unsupported widths.
 */
jc_status jc_engine_create_timestral(const jc_timestral_desc* desc, const jc_tensor_view* weights, int n_weights,
                                     const int* devices, int n_devices, jc_precision precision, jc_engine** out);

/* One decode block's device-forward inputs: what TimestralForward.Plan.run uploads
 * (timestral/tornado/TimestralForward.java:594-632), as BlockLayout and BlockPrep compute them. */
typedef struct jc_timestral_block {
  int rows;
  int encoder;         /* encoder tokens per row (BlockLayout.encoderTokens) */
  int horizon;         /* decoder tokens per row (BlockLayout.horizonPatches) */
  int context_patches; /* BlockLayout.contextPatches */
  int covariates;      /* BlockLayout.covariates */
  const float* tokens;         /* [rows · encoder · 2P] BlockPrep.tokens */
  const int32_t* positions;    /* [rows · (encoder + horizon)] BlockLayout.position */
  const int32_t* key_valid;    /* [rows · encoder] BlockLayout.keyValid, 0/1 */
  const int32_t* known;        /* [rows] BlockLayout.known, 0/1 */
  const int32_t* role;         /* [rows] BlockLayout.role */
  const int32_t* group_start;  /* [rows] first row of the row's series */
  const int32_t* group_end;    /* [rows] one past its last row */
} jc_timestral_block;

/*
 * The Timestral forward of one block on HOST buffers: raw_out [rows · horizon · P · Q] receives
 * the quantile head's raw outputs (what TimestralForward.Plan.run downloads; the caller then runs
 * BlockPrep.finish). Rows are sharded across the engine's GPUs in contiguous ranges that keep
 * each series on one GPU; every GPU runs its shard as a CUDA graph and the results are gathered
 * into raw_out. Rows of one series must be contiguous (JC_ERR_INVALID_ARG otherwise, as
 * TimestralForward.java:616-619). Thread-safe; calls on one engine are serialised.
 */
jc_status jc_forward_timestral(jc_engine* engine, const jc_timestral_block* block, float* raw_out);

/*
 * The same forward on inputs already in HBM of the engine's GPU number `slot` (0-based index
 * into the devices given at creation): every pointer of `block` and `raw_out` is a device
 * pointer on that GPU. Enqueued on `stream` (cudaStream_t; NULL = the legacy default stream),
 * returns without synchronising. Device-side errors surface on the next jc_engine_sync.
 */
jc_status jc_forward_timestral_device(jc_engine* engine, int slot, const jc_timestral_block* block, float* raw_out,
                                      void* stream);

/*
 * One decode block with BlockPrep's host ends moved onto the GPU (timestral/BlockPrep.java:40-101):
 * the layout fields of `layout` as for jc_forward_timestral (its `tokens` is not read and may be
 * NULL), and the raw window they are computed from instead of the tokens. The GPU runs the scaler
 * (Scaler.causalPatchLocScale, Scaler.instanceNorm on known-covariate rows), assembles the
 * tokens, runs the forward, then BlockPrep.finish (Quantiles.apply, Scaler.invert,
 * Scaler.clampNonFinite) with the reference's arithmetic: statistics in double, each float
 * product and sum rounded on its own.
 */
typedef struct jc_timestral_window {
  jc_timestral_block layout;
  const float* window;         /* [rows · encoder · P] BlockLayout.window */
  const uint8_t* observed;     /* [rows · encoder · P] BlockLayout.observed, 0/1 */
  float minimum_scale;         /* TimestralConfig.minimumScale */
  int use_asinh;               /* TimestralConfig.useAsinh */
  int median;                  /* Quantiles.median() */
  const float* quantile_scale; /* [Q] Quantiles.scale(); a HOST array in both calls below, Q <= 64 */
} jc_timestral_window;

/*
 * BlockForward.predictBlock after the layout, on HOST buffers: quantiles_out [rows · horizon · P · Q]
 * receives BlockPrep.finish's raw-space quantiles ([rows][H·P][Q]). Sharded, graphed and
 * validated as jc_forward_timestral; the window crosses to the GPU instead of the tokens
 * (5 bytes per step instead of 8) and nothing is left for the host to finish.
 */
jc_status jc_forecast_timestral(jc_engine* engine, const jc_timestral_window* block, float* quantiles_out);

/* The same on device buffers of the engine's GPU number `slot` (every pointer of `block` except
 * quantile_scale, and quantiles_out), enqueued on `stream` as jc_forward_timestral_device. */
jc_status jc_forecast_timestral_device(jc_engine* engine, int slot, const jc_timestral_window* block,
                                       float* quantiles_out, void* stream);

/* The Chronos2Config fields the forward pass uses (chronos2/Chronos2Config.java:45-60). */
typedef struct jc_chronos2_desc {
  int d_model;
  int d_kv;
  int d_ff;
  int num_layers;
  int num_heads;
  int patch_size;
  int num_quantiles;
  int use_reg_token;
  float layer_norm_eps;
  float rope_theta;
} jc_chronos2_desc;

/*
 * Creates a Chronos-2 engine: binds `weights` by the checkpoint's names and shapes (every tensor once,
 * as chronos2/Chronos2Weights.java:80-100; unknown, missing or misshapen tensors fail with
 * JC_ERR_INVALID_ARG) and converts them to `precision` on every GPU in `devices`. Head widths other
 * than 64 fail with JC_ERR_UNSUPPORTED_SHAPE (as Chronos2Forward.java:126-128 rejects widths).
 */
jc_status jc_engine_create_chronos2(const jc_chronos2_desc* desc, const jc_tensor_view* weights, int n_weights,
                                    const int* devices, int n_devices, jc_precision precision, jc_engine** out);

/* One forward pass's device inputs: what Chronos2Forward.Plan.run uploads
 * (chronos2/tornado/Chronos2Forward.java:463-489), as ModelLayout and ModelPrep compute them. */
typedef struct jc_chronos2_block {
  int rows;
  int context_patches; /* ModelLayout.contextPatches (nc) */
  int output_patches;  /* ModelLayout.outputPatches (h) */
  const float* tokens;        /* [rows · (nc + h) · 3P] ModelPrep.tokens */
  const int32_t* live;        /* [rows · (nc + reg + h)] ModelLayout.live, 0/1 */
  const int32_t* group_start; /* [rows] first row of the row's group */
  const int32_t* group_end;   /* [rows] one past its last row */
} jc_chronos2_block;

/*
 * The Chronos-2 encoder on HOST buffers: raw_out [rows · h · Q · P] receives the output patch
 * embedding's raw values, each token's quantiles level-major (the caller then runs
 * ModelPrep.finish). Rows are sharded across the engine's GPUs in contiguous ranges that keep each
 * group on one GPU; rows of one group must be contiguous (JC_ERR_INVALID_ARG otherwise).
 */
jc_status jc_forward_chronos2(jc_engine* engine, const jc_chronos2_block* block, float* raw_out);

/* The same on inputs already in HBM of the engine's GPU number `slot`, enqueued on `stream`. */
jc_status jc_forward_chronos2_device(jc_engine* engine, int slot, const jc_chronos2_block* block, float* raw_out,
                                     void* stream);

/*
 * One forward with ModelPrep's host ends moved onto the GPU (chronos2/ModelPrep.java:29-137): the
 * layout fields of `layout` as for jc_forward_chronos2 (its `tokens` is not read and may be NULL), and
 * the window and future covariates the tokens are made from. The GPU runs InstanceNorm (statistics in
 * double, in the reference's order), assembles the tokens, runs the encoder, then ModelPrep.finish.
 */
typedef struct jc_chronos2_window {
  jc_chronos2_block layout;
  const float* window;       /* [rows · nc · P] ModelLayout.window, NaN = missing */
  const float* future;       /* [rows · h · P] ModelLayout.future, NaN = missing */
  float time_encoding_scale; /* Chronos2Config.timeEncodingScale */
  int use_arcsinh;           /* Chronos2Config.useArcsinh */
} jc_chronos2_window;

/* ModelForward.forward after the layout, on HOST buffers: quantiles_out [rows · Q · h·P] receives
 * ModelPrep.finish's quantiles in each row's own scale. Sharded and validated as jc_forward_chronos2. */
jc_status jc_forecast_chronos2(jc_engine* engine, const jc_chronos2_window* block, float* quantiles_out);

/* The same on device buffers of the engine's GPU number `slot`, enqueued on `stream`. */
jc_status jc_forecast_chronos2_device(jc_engine* engine, int slot, const jc_chronos2_window* block,
                                      float* quantiles_out, void* stream);

/* TiRex-2 time-mixer kinds (the stack recipe's "bi-mlstm" / "bi-slstm", tirex2/TiRex2Config.java:161-175). */
#define JC_TIREX_MLSTM 0
#define JC_TIREX_SLSTM 1

/* The TiRex2Config fields the forward pass uses (tirex2/TiRex2Config.java:48-66). */
typedef struct jc_tirex2_desc {
  int embedding_dim;
  int num_blocks;
  int patch_size;
  int input_ff_dim;
  int output_ff_dim;
  int context_len;
  int future_len;
  int num_quantiles;
  const int32_t* block_types; /* [num_blocks] JC_TIREX_MLSTM / JC_TIREX_SLSTM */
  int time_mixer_heads;
  int slstm_heads;
  int variate_heads;
  int use_arcsinh;
  int binary_aware;
  int use_qk_norm;
  float stack_out_norm_eps;
} jc_tirex2_desc;

/*
 * Creates a TiRex-2 engine: binds `weights` by the checkpoint's names and shapes (every tensor once, as
 * tirex2/TiRex2Weights.java:128-247; unknown, missing or misshapen tensors fail with JC_ERR_INVALID_ARG)
 * and converts them to `precision` on every GPU in `devices`. The cells and the variate attention take
 * 128-wide heads (64-wide mLSTM q/k), as the reference's device forward does
 * (tirex2/tornado/TornadoForward.java:261-264, :708-710); other widths fail with JC_ERR_UNSUPPORTED_SHAPE.
 */
jc_status jc_engine_create_tirex2(const jc_tirex2_desc* desc, const jc_tensor_view* weights, int n_weights,
                                  const int* devices, int n_devices, jc_precision precision, jc_engine** out);

/* One forward pass's device inputs: what TornadoForward.Plan.run uploads
 * (tirex2/tornado/TornadoForward.java:799-815), with the structure lists of TornadoForward.structure
 * (:406-449). len = context_len + future_len. */
typedef struct jc_tirex2_batch {
  int rows;
  const float* x;            /* [rows · len] values, 0 where there is no observation */
  const float* present;      /* [rows · len] 1 where x holds an observation, else 0 */
  int n_known;               /* covariate rows with a value in the future window (reverse pass) */
  const int32_t* known;      /* [n_known] increasing row indices */
  int n_kept;                /* rows of multi-row groups (variate mixer) */
  const int32_t* kept;       /* [n_kept] increasing row indices; a group's rows are contiguous */
  const int32_t* group_start; /* [n_kept] first kept index of the row's group */
  const int32_t* group_end;   /* [n_kept] one past the group's last kept index */
  const int32_t* kept_target; /* [n_kept] 1 for target rows, 0 for covariates */
} jc_tirex2_batch;

/*
 * The TiRex-2 forward (TiRex2.forward as ForwardPass.forward, tirex2/ForwardPass.java) on HOST buffers:
 * out [rows · Q · len] receives the rescaled quantile outputs over the whole padded length, in data units.
 * Rows are sharded across the engine's GPUs in contiguous ranges that keep each group on one GPU.
 */
jc_status jc_forward_tirex2(jc_engine* engine, const jc_tirex2_batch* batch, float* out);

/* The same on inputs already in HBM of the engine's GPU number `slot` (every pointer of `batch`, and `out`,
 * a device pointer on that GPU), enqueued on `stream`. The lists are not checked on the host here. */
jc_status jc_forward_tirex2_device(jc_engine* engine, int slot, const jc_tirex2_batch* batch, float* out,
                                   void* stream);

/*
 * BlockPrep.of's GPU half alone (timestral/BlockPrep.java:40-73, the kernels jc_forecast_timestral runs
 * before its forward): on DEVICE buffers of `device`, window [rows · encoder · patch] FP32 and observed
 * (0/1 bytes) as BlockLayout.window / observed, known [rows] as BlockLayout.known, write
 * tokens_out [rows · encoder · 2·patch] as BlockPrep.tokens (each patch's scaled values, then its missing
 * flags). For callers that build their own device inputs for jc_forward_timestral_device. Enqueued on
 * `stream`; the call's scratch is stream-ordered memory freed on the same stream.
 */
jc_status jc_timestral_prep_device(int device, int rows, int encoder, int patch, const float* window,
                                   const uint8_t* observed, const int32_t* known, float minimum_scale, int use_asinh,
                                   float* tokens_out, void* stream);

/*
 * ModelPrep.of's GPU half alone (chronos2/ModelPrep.java:29-70, the kernels jc_forecast_chronos2 runs before
 * its encoder): on DEVICE buffers of `device`, window [rows · context_patches · patch] and future
 * [rows · output_patches · patch] FP32 (NaN = missing) as ModelLayout.window / future, write
 * tokens_out [rows · (context_patches + output_patches) · 3·patch] as ModelPrep.tokens. Enqueued on `stream`.
 */
jc_status jc_chronos2_prep_device(int device, int rows, int context_patches, int output_patches, int patch,
                                  const float* window, const float* future, float time_encoding_scale,
                                  int use_arcsinh, float* tokens_out, void* stream);

/*
 * BlockPrep.finish on the GPU alone (timestral/BlockPrep.java:81-101): in place on raw [rows · steps · Q]
 * (steps = horizon · P, the head's raw outputs), Quantiles.apply with `quantile_scale` [Q] (Quantiles.scale(),
 * a HOST array, Q <= 64) and `median`, then Scaler.invert with each row's (loc, scale) of its last context
 * patch (loc_scale [rows · 2], device, 8-byte aligned) and Scaler.clampNonFinite. Enqueued on `stream`.
 */
jc_status jc_timestral_finish_device(int device, int rows, int steps, int quantiles, int median,
                                     const float* quantile_scale, int use_asinh, const float* loc_scale, float* raw,
                                     void* stream);

/*
 * ModelPrep.finish on the GPU alone (chronos2/ModelPrep.java:116-137): out [rows · Q · h·P] =
 * sinh(raw)·scale + loc from raw [rows · h · Q · P] (each output token's quantiles level-major) and each
 * row's (loc, scale) (loc_scale [rows · 2], device, 8-byte aligned). Enqueued on `stream`.
 */
jc_status jc_chronos2_finish_device(int device, int rows, int output_patches, int patch, int quantiles,
                                    int use_arcsinh, const float* loc_scale, const float* raw, float* out,
                                    void* stream);

/*
 * Self-test of the bounded waits every kernel of the library uses (no counterpart in the reference): one
 * thread waits `limit_us` microseconds (1 .. 1,000,000), with the same mbarrier wait, for a barrier phase
 * that nothing completes, gives up, records it in the device's error word and returns. The call then reports
 * it as jc_device_sync would — JC_ERR_TIMEOUT, the error word cleared — and the device stays usable.
 */
jc_status jc_device_wait_selftest(int device, int limit_us);

/* Waits for every GPU of the engine; JC_ERR_TIMEOUT if a kernel's bounded wait gave up. */
jc_status jc_engine_sync(jc_engine* engine);

/*
 * The rule every multi-GPU forward shards rows by (host arithmetic only, no device): cuts_out[0 .. parts]
 * receives the first row of each of `parts` contiguous ranges and cuts_out[parts] = rows. Each cut starts
 * at rows·p/parts and moves forward to the next series boundary, so no series (group_start/group_end,
 * as the blocks carry them) spans two GPUs; a range may be empty. JC_ERR_INVALID_ARG for rows < 0,
 * parts < 1, null arrays or series ranges that are not contiguous.
 */
jc_status jc_shard_rows(int rows, const int32_t* group_start, const int32_t* group_end, int parts, int32_t* cuts_out);

/*
 * Engine options (the reference's -D properties, e.g. timestral.tornado.cudaGraph and
 * timestral.tornado.plans in TimestralForward.java:146-160):
 *   "cuda_graph"  1 (default) replay each shape as a captured CUDA graph, 0 run eagerly
 *   "max_plans"   shape plans kept per GPU (default 8; least recently used evicted)
 *   "buckets"     1 (default) shards run on plans built for a bucketed row count (the
 *                 count itself up to 8, then the next multiple of a quarter of its power of two: at most 25 %
 *                 padding, TimestralForward.bucket, TimestralForward.java:88-99); 0 one plan per exact row
 *                 count
 *   "profile"     1: run eagerly and time every kernel class with CUDA events (jc_engine_profile)
 * Failure injection on the host, for tests of the error paths (no GPU fault is involved):
 *   "fail_plan_allocs"  N: the next N plan allocations report out of device memory. As the reference's
 *                 PlanCache.run (tornado/PlanCache.java:70-100), a failed allocation with other plans cached
 *                 drops them and retries once; with none cached, or when the retry fails too, the call
 *                 returns JC_ERR_OOM and the engine stays usable
 *   "fail_slot"   s: the next forward's shard on engine slot s fails before it enqueues any work; the call
 *                 gathers every shard, then returns JC_ERR_CUDA naming the slot (-1: none)
 */
jc_status jc_engine_set_option(jc_engine* engine, const char* key, long long value);

/* Kernel-class timings collected while "profile" is 1, summed since the last read (then reset).
 * names/ms/launches have room for `cap` entries; *count receives the number written. */
jc_status jc_engine_profile(jc_engine* engine, int slot, const char** names, double* ms, long long* launches,
                            double* flops, int cap, int* count);

/* Frees the engine's device memory, graphs and streams. NULL is a no-op; returns JC_OK. */
jc_status jc_engine_destroy(jc_engine* engine);

#ifdef __cplusplus
}
#endif

#endif /* JITCAST_B200_H */

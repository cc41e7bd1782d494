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
 *   JC_FP32  FP32 operands as TF32 hi/lo pairs, three TF32 MMAs per product (≈ FP32 accuracy)
 *   JC_TF32  TF32 operands, FP32 accumulation (the reference's CUBLAS_TF32)
 *   JC_BF16  BF16 operands, FP32 accumulation and FP32 residual stream (replaces CUBLAS_FP16) */
typedef enum jc_precision { JC_FP32 = 0, JC_TF32 = 1, JC_BF16 = 2 } jc_precision;

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

/* Waits for all work on `device`, then returns and clears the device's kernel error word:
 * JC_ERR_TIMEOUT if a kernel's bounded wait gave up since the last call. */
jc_status jc_device_sync(int device);

#ifdef __cplusplus
}
#endif

#endif /* JITCAST_B200_H */

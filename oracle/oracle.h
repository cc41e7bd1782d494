/*
 * ORACLE — test infrastructure only (see ops.c). CPU restatements of the reference's FP32
 * operators and forward passes; the checker for the CUDA path, never part of it.
 */
#ifndef JC_ORACLE_H
#define JC_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* Kernels.gemm flag values (tornado/Kernels.java:50-56) plus GELU. */
#define JCO_BIAS 1
#define JCO_ACCUMULATE 2
#define JCO_SILU 4
#define JCO_RELU 16
#define JCO_GELU 32

/* Operand formats of jco_set_operand_format (a reduced-precision run of the reference arithmetic). */
#define JCO_OPERANDS_FP32 0
#define JCO_OPERANDS_TF32 1
#define JCO_OPERANDS_BF16 2
#define JCO_OPERANDS_FP16 3

/* Every later jco_linear rounds its x and w elements to `fmt` before the double accumulation
 * (JCO_OPERANDS_FP32, the default: the reference's own arithmetic). Process-wide, not thread-safe. */
void jco_set_operand_format(int fmt);
int jco_operand_format(void);
/* v rounded to nearest even in `fmt` (FP16 saturating at ±65504). */
float jco_round_operand(float v, int fmt);

float jco_silu(float v);
double jco_sigmoid(double v);

/* Ops.linear (cpu/Ops.java:33-51): y [rows, out] = x [rows, in] · w[out, in]ᵀ + b. */
void jco_linear(const float* x, int rows, const float* w, const float* b, int in, int out, float* y, int threads);

/* Ops.rmsNorm (cpu/Ops.java:53-67). */
void jco_rmsnorm(const float* x, int rows, int cols, const float* w, float eps, float* y);

/* Kernels.gemm's expected result as KernelsAccelTest builds it: linear (+bias), SiLU, ReLU, += C. */
void jco_gemm(const float* a, const float* w, const float* bias, float* c, int m, int n, int k, int flags, int threads);

#ifdef __cplusplus
}
#endif

#endif

/*
 * ORACLE — test infrastructure only. A plain-C restatement of the reference's FP32 CPU
 * operators, used by tests/, __graft_entry__.smoke() and bench.py's CPU baseline as the
 * checker. Nothing in the product path (libjitcast_b200.so, jitcast_b200/) may call it.
 *
 * Restates src/main/java/ai/beestream/jitcast/cpu/Ops.java of jitCast:
 *   linear   Ops.java:32-51   y[r] = W·x[r] + b, double accumulation in index order, cast to float
 *   rmsNorm  Ops.java:52-67   double sum of squares, inv = (float)(1/sqrt(ss/cols + eps))
 *   silu     Ops.java:68-70   (float)(v / (1 + exp(-v))) in double
 *   sigmoid  Ops.java:71-73
 * and the epilogue order of tornado/Kernels.java:86-100 (bias, SiLU, ReLU, += C), as
 * KernelsAccelTest composes it from the Ops operators (KernelsAccelTest.java:66-89).
 *
 * Java evaluates double arithmetic in IEEE binary64 without contraction; this file must be
 * compiled with -ffp-contract=off and without -ffast-math so every sum and product rounds
 * the way Java's does (linear is then bit-identical to Ops.linear).
 *
 * linear runs row chunks of 16 (Ops.java:31 PARALLEL_ROWS) on a pthread pool; the result does
 * not depend on the thread count.
 *
 * jco_set_operand_format selects a reduced-precision run of the same arithmetic: every linear
 * rounds its x and w elements (to nearest even) to TF32, BF16 or FP16 before the double
 * accumulation, as tensor-core operands are rounded. This is the reference's yardstick for its
 * reduced-precision device paths — no further from the FP32 reference than a reduced-precision run
 * of the reference arithmetic (tirex2/tornado/TornadoForwardAccelTest.java:39-44,
 * GoldenData.nxaiGpuError) — and the tests use it to measure that distance. The default (0) is the
 * reference's FP32 arithmetic.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define PARALLEL_ROWS 16

static int g_operand_format = JCO_OPERANDS_FP32;

void jco_set_operand_format(int fmt) { g_operand_format = fmt; }

int jco_operand_format(void) { return g_operand_format; }

/* v rounded to nearest even, keeping `bits` explicit mantissa bits (FP32 exponent range). */
static float round_mantissa(float v, int bits) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0x7f800000u) == 0x7f800000u) return v; /* inf, nan */
  const int sh = 23 - bits;
  const uint64_t w = (uint64_t)u + ((1u << (sh - 1)) - 1) + ((u >> sh) & 1u);
  u = (uint32_t)((w >> sh) << sh);
  memcpy(&v, &u, 4);
  return v;
}

/* v as IEEE half (nearest even, subnormals kept), saturated to ±65504 as the device's operand stores. */
static float round_half(float v) {
  if (v != v) return v;
  if (v > 65504.0f) return 65504.0f;
  if (v < -65504.0f) return -65504.0f;
  const float a = fabsf(v);
  if (a < 6.103515625e-05f) { /* subnormal half: a multiple of 2^-24 */
    const double q = nearbyint((double)a * 16777216.0) / 16777216.0;
    return copysignf((float)q, v);
  }
  return round_mantissa(v, 10);
}

float jco_round_operand(float v, int fmt) {
  switch (fmt) {
    case JCO_OPERANDS_TF32: return round_mantissa(v, 10);
    case JCO_OPERANDS_BF16: return round_mantissa(v, 7);
    case JCO_OPERANDS_FP16: return round_half(v);
    default: return v;
  }
}

static float* rounded_copy(const float* a, size_t n, int fmt) {
  float* r = (float*)malloc(n * sizeof(float));
  for (size_t i = 0; i < n; i++) r[i] = jco_round_operand(a[i], fmt);
  return r;
}

float jco_silu(float v) { return (float)(v / (1.0 + exp(-(double)v))); }

double jco_sigmoid(double v) { return 1.0 / (1.0 + exp(-v)); }

static void linear_rows(const float* x, const float* w, const float* b, int in, int out, float* y, int r0, int r1) {
  for (int r = r0; r < r1; r++) {
    const float* xr = x + (size_t)r * in;
    float* yr = y + (size_t)r * out;
    for (int o = 0; o < out; o++) {
      const float* wr = w + (size_t)o * in;
      double acc = 0;
      for (int i = 0; i < in; i++) acc += (double)xr[i] * (double)wr[i];
      yr[o] = (float)(b == NULL ? acc : acc + (double)b[o]);
    }
  }
}

typedef struct {
  const float *x, *w, *b;
  int rows, in, out;
  float* y;
  atomic_int next;
} linear_job;

static void* linear_worker(void* arg) {
  linear_job* j = (linear_job*)arg;
  const int chunks = (j->rows + PARALLEL_ROWS - 1) / PARALLEL_ROWS;
  for (;;) {
    int c = atomic_fetch_add(&j->next, 1);
    if (c >= chunks) break;
    int r0 = c * PARALLEL_ROWS, r1 = r0 + PARALLEL_ROWS < j->rows ? r0 + PARALLEL_ROWS : j->rows;
    linear_rows(j->x, j->w, j->b, j->in, j->out, j->y, r0, r1);
  }
  return NULL;
}

static void linear_exact(const float* x, int rows, const float* w, const float* b, int in, int out, float* y,
                         int threads);

void jco_linear(const float* x, int rows, const float* w, const float* b, int in, int out, float* y, int threads) {
  const int fmt = g_operand_format;
  if (fmt == JCO_OPERANDS_FP32) {
    linear_exact(x, rows, w, b, in, out, y, threads);
    return;
  }
  float* xr = rounded_copy(x, (size_t)rows * in, fmt);
  float* wr = rounded_copy(w, (size_t)out * in, fmt);
  linear_exact(xr, rows, wr, b, in, out, y, threads);
  free(xr);
  free(wr);
}

static void linear_exact(const float* x, int rows, const float* w, const float* b, int in, int out, float* y,
                         int threads) {
  if (rows <= PARALLEL_ROWS || threads <= 1) {
    linear_rows(x, w, b, in, out, y, 0, rows);
    return;
  }
  linear_job job = {x, w, b, rows, in, out, y, 0};
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  int started = 0;
  for (int t = 1; t < threads; t++)
    if (pthread_create(&tid[started], NULL, linear_worker, &job) == 0) started++;
  linear_worker(&job);
  for (int t = 0; t < started; t++) pthread_join(tid[t], NULL);
}

void jco_rmsnorm(const float* x, int rows, int cols, const float* w, float eps, float* y) {
  for (int r = 0; r < rows; r++) {
    const float* xr = x + (size_t)r * cols;
    float* yr = y + (size_t)r * cols;
    double ss = 0;
    for (int c = 0; c < cols; c++) ss += (double)xr[c] * (double)xr[c];
    float inv = (float)(1.0 / sqrt(ss / cols + (double)eps));
    for (int c = 0; c < cols; c++) yr[c] = w == NULL ? xr[c] * inv : xr[c] * inv * w[c];
  }
}

void jco_gemm(const float* a, const float* w, const float* bias, float* c, int m, int n, int k, int flags,
              int threads) {
  size_t mn = (size_t)m * n;
  float* y = (float*)malloc(mn * sizeof(float));
  jco_linear(a, m, w, (flags & JCO_BIAS) ? bias : NULL, k, n, y, threads);
  if (flags & JCO_SILU)
    for (size_t i = 0; i < mn; i++) y[i] = jco_silu(y[i]);
  if (flags & JCO_RELU)
    for (size_t i = 0; i < mn; i++) y[i] = y[i] > 0.0f ? y[i] : 0.0f;
  if (flags & JCO_GELU)
    for (size_t i = 0; i < mn; i++) y[i] = (float)(0.5 * y[i] * (1.0 + erf((double)y[i] / sqrt(2.0))));
  if (flags & JCO_ACCUMULATE)
    for (size_t i = 0; i < mn; i++) y[i] += c[i];
  memcpy(c, y, mn * sizeof(float));
  free(y);
}

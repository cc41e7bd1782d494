// C-ABI entry points of the op-level GEMM: jc_linear (host buffers) and jc_linear_device
// (HBM-resident buffers), with the epilogue flags of the reference's Kernels.gemm
// (tornado/Kernels.java:50-102) and the operator of Ops.linear (cpu/Ops.java:33-51).
#include <cstring>
#include <string>

#include "gemm.h"
#include "kernels.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace {

// One thread waits, with the library's bounded mbarrier wait, for a phase that nothing completes.
__global__ void wait_selftest_kernel(uint32_t* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    jc::mbar_init(&bar, 1);
    jc::fence_mbar_init();
    if (!jc::mbar_wait(&bar, 0, limit_ns)) atomicOr(err, jc::kErrTimeoutFlag);
  }
}

}  // namespace

using namespace jc;

namespace {

enum Slot { kSlotA = 0, kSlotALo, kSlotW, kSlotWLo, kSlotAF32, kSlotWF32, kSlotBias, kSlotC };

int op_of(jc_precision p) { return p == JC_BF16 ? kOpBF16 : p == JC_FP16 ? kOpF16 : p == JC_TF32 ? kOpTF32 : kOpSplit; }

// Maps Kernels.gemm flags to an activation; false for flags this engine rejects.
bool act_of(int flags, int* act, std::string* why) {
  const int known = JC_BIAS | JC_ACCUMULATE | JC_SILU | JC_RELU | JC_GELU | JC_TWIN_ONLY;
  if (flags & ~known) {
    *why = "unknown flag bits " + std::to_string(flags & ~known);
    return false;
  }
  if (flags & JC_TWIN_ONLY) {
    *why = "JC_TWIN_ONLY writes only an FP16 twin of C and does not apply to an FP32 C";
    return false;
  }
  const bool silu = flags & JC_SILU, relu = flags & JC_RELU, gelu = flags & JC_GELU;
  if (gelu && (silu || relu)) {
    *why = "JC_GELU cannot be combined with JC_SILU or JC_RELU";
    return false;
  }
  *act = silu && relu ? kActSiluRelu : silu ? kActSilu : relu ? kActRelu : gelu ? kActGelu : kActNone;
  return true;
}

bool valid_precision(int p) { return p == JC_FP32 || p == JC_TF32 || p == JC_BF16 || p == JC_FP16; }

// Converts fp32 A [rows, cols] (pitch ld) into the operand buffers of slot pair (hi, lo),
// K padded to a multiple of 64 elements.
bool stage_operand(DeviceRt* rt, int op, const float* src, long long ld, long long rows, int cols, int slot_hi,
                   int slot_lo, void** hi, void** lo, long long* ldp, cudaStream_t s) {
  const long long kp = round_up(cols, 64);
  const size_t esz = (op == kOpBF16 || op == kOpF16) ? 2 : 4;
  *hi = scratch(rt, slot_hi, rows * kp * esz);
  *lo = op == kOpSplit ? scratch(rt, slot_lo, rows * kp * esz) : nullptr;
  if (!*hi || (op == kOpSplit && !*lo)) return false;
  launch_convert(op, src, ld, *hi, *lo, kp, rows, cols, s);
  *ldp = kp;
  return true;
}

}  // namespace

extern "C" {

const char* jc_version(void) { return "jitcast_b200 0.1.0 (sm_100a)"; }

const char* jc_last_error(void) { return last_error(); }

int jc_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Enqueues the GEMM on `s`; the caller holds rt->mu with the device current.
static jc_status linear_locked(DeviceRt* rt, jc_precision precision, const float* a, long long lda, const float* w,
                               long long ldw, const float* bias, float* c, long long ldc, int m, int n, int k,
                               int flags, int act, cudaStream_t s) {
  const int op = op_of(precision);
  GemmArgs g{};
  g.op = op;
  g.M = m;
  g.N = n;
  g.K = k;
  void *ahi, *alo, *whi, *wlo;
  long long lda_p, ldw_p;
  if (!stage_operand(rt, op, a, lda, m, k, kSlotA, kSlotALo, &ahi, &alo, &lda_p, s) ||
      !stage_operand(rt, op, w, ldw, n, k, kSlotW, kSlotWLo, &whi, &wlo, &ldw_p, s))
    return fail(JC_ERR_OOM, "scratch allocation failed");
  g.a_hi = ahi;
  g.a_lo = alo;
  g.lda = lda_p;
  g.w_hi = whi;
  g.w_lo = wlo;
  g.ldw = ldw_p;
  g.ep = epi_default();
  g.ep.act = act;
  g.ep.bias_on = (flags & JC_BIAS) != 0;
  g.ep.bias = bias;
  g.ep.accumulate = (flags & JC_ACCUMULATE) != 0;
  g.ep.c = c;
  g.ep.ldc = ldc;
  g.ep.cin = c;
  g.ep.ldcin = ldc;
  if (const char* msg = check_gemm(g)) return fail(JC_ERR_UNSUPPORTED_SHAPE, msg);
  cudaError_t e = launch_gemm(g, s, rt->err);
  if (e != cudaSuccess) return fail_cuda(e, "GEMM launch");
  return JC_OK;
}

jc_status jc_linear_device(int device, jc_precision precision, const float* a, long long lda, const float* w,
                           long long ldw, const float* bias, float* c, long long ldc, int m, int n, int k, int flags,
                           void* stream) {
  clear_error();
  if (!valid_precision(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (m < 1 || n < 1 || k < 1) return fail(JC_ERR_INVALID_ARG, "m, n and k must be positive");
  if (!a || !w || !c) return fail(JC_ERR_INVALID_ARG, "null buffer");
  if ((flags & JC_BIAS) && !bias) return fail(JC_ERR_INVALID_ARG, "JC_BIAS without a bias");
  if (lda < k || ldw < k || ldc < n) return fail(JC_ERR_INVALID_ARG, "leading dimension smaller than the row");
  int act = 0;
  std::string why;
  if (!act_of(flags, &act, &why)) return fail(JC_ERR_INVALID_ARG, why);
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  return linear_locked(rt, precision, a, lda, w, ldw, bias, c, ldc, m, n, k, flags, act,
                       static_cast<cudaStream_t>(stream));
}

jc_status jc_linear(int device, jc_precision precision, const float* a, const float* w, const float* bias, float* c,
                    int m, int n, int k, int flags) {
  clear_error();
  if (!valid_precision(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (m < 1 || n < 1 || k < 1) return fail(JC_ERR_INVALID_ARG, "m, n and k must be positive");
  if (!a || !w || !c) return fail(JC_ERR_INVALID_ARG, "null buffer");
  if ((flags & JC_BIAS) && !bias) return fail(JC_ERR_INVALID_ARG, "JC_BIAS without a bias");
  int act = 0;
  std::string why;
  if (!act_of(flags, &act, &why)) return fail(JC_ERR_INVALID_ARG, why);
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  float* da = static_cast<float*>(scratch(rt, kSlotAF32, sizeof(float) * (size_t)m * k));
  float* dw = static_cast<float*>(scratch(rt, kSlotWF32, sizeof(float) * (size_t)n * k));
  float* dc = static_cast<float*>(scratch(rt, kSlotC, sizeof(float) * (size_t)m * n));
  float* db = (flags & JC_BIAS) ? static_cast<float*>(scratch(rt, kSlotBias, sizeof(float) * (size_t)n)) : nullptr;
  if (!da || !dw || !dc || ((flags & JC_BIAS) && !db)) return fail(JC_ERR_OOM, "device buffers for jc_linear");
  cudaStream_t s = rt->stream;
  cudaError_t e = cudaMemcpyAsync(da, a, sizeof(float) * (size_t)m * k, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(dw, w, sizeof(float) * (size_t)n * k, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && db) e = cudaMemcpyAsync(db, bias, sizeof(float) * n, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && (flags & JC_ACCUMULATE))
    e = cudaMemcpyAsync(dc, c, sizeof(float) * (size_t)m * n, cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return fail_cuda(e, "upload");
  jc_status st = linear_locked(rt, precision, da, k, dw, k, db, dc, n, m, n, k, flags, act, s);
  if (st != JC_OK) return st;
  e = cudaMemcpyAsync(c, dc, sizeof(float) * (size_t)m * n, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail_cuda(e, "download");
  return take_device_error(rt);
}

jc_status jc_gemm_device(int device, jc_precision precision, const void* a_hi, const void* a_lo, long long lda,
                         const void* w_hi, const void* w_lo, long long ldw, const float* bias, float* c,
                         long long ldc, int m, int n, int k, int flags, void* stream) {
  clear_error();
  if (!valid_precision(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (m < 1 || n < 1 || k < 1) return fail(JC_ERR_INVALID_ARG, "m, n and k must be positive");
  if (!a_hi || !w_hi || !c) return fail(JC_ERR_INVALID_ARG, "null buffer");
  if ((flags & JC_BIAS) && !bias) return fail(JC_ERR_INVALID_ARG, "JC_BIAS without a bias");
  if (ldc < n) return fail(JC_ERR_INVALID_ARG, "ldc smaller than n");
  int act = 0;
  std::string why;
  if (!act_of(flags, &act, &why)) return fail(JC_ERR_INVALID_ARG, why);
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  GemmArgs g{};
  g.op = op_of(precision);
  g.a_hi = a_hi;
  g.a_lo = a_lo;
  g.lda = lda;
  g.w_hi = w_hi;
  g.w_lo = w_lo;
  g.ldw = ldw;
  g.M = m;
  g.N = n;
  g.K = k;
  g.ep = epi_default();
  g.ep.act = act;
  g.ep.bias_on = (flags & JC_BIAS) != 0;
  g.ep.bias = bias;
  g.ep.accumulate = (flags & JC_ACCUMULATE) != 0;
  g.ep.c = c;
  g.ep.ldc = ldc;
  g.ep.cin = c;
  g.ep.ldcin = ldc;
  if (const char* msg = check_gemm(g)) return fail(JC_ERR_UNSUPPORTED_SHAPE, msg);
  cudaError_t e = launch_gemm(g, static_cast<cudaStream_t>(stream), rt->err);
  if (e != cudaSuccess) return fail_cuda(e, "GEMM launch");
  return JC_OK;
}

jc_status jc_gemm_group_device(int device, jc_precision precision, const jc_gemm_problem* problems, int count,
                               void* stream) {
  clear_error();
  if (!valid_precision(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (!problems || count < 1 || count > kMaxGemmGroup)
    return fail(JC_ERR_INVALID_ARG, "a group holds 1 to " + std::to_string(kMaxGemmGroup) + " problems");
  GemmArgs g[kMaxGemmGroup];
  std::string why;
  for (int i = 0; i < count; ++i) {
    const jc_gemm_problem& q = problems[i];
    const std::string at = "problem " + std::to_string(i) + ": ";
    if (q.m < 1 || q.n < 1 || q.k < 1) return fail(JC_ERR_INVALID_ARG, at + "m, n and k must be positive");
    if (!q.a_hi || !q.w_hi || !q.c) return fail(JC_ERR_INVALID_ARG, at + "null buffer");
    if ((q.flags & JC_BIAS) && !q.bias) return fail(JC_ERR_INVALID_ARG, at + "JC_BIAS without a bias");
    if (q.ldc < q.n) return fail(JC_ERR_INVALID_ARG, at + "ldc smaller than n");
    int act = 0;
    if (!act_of(q.flags, &act, &why)) return fail(JC_ERR_INVALID_ARG, at + why);
    GemmArgs& x = g[i];
    x = GemmArgs{};
    x.op = op_of(precision);
    x.a_hi = q.a_hi;
    x.a_lo = q.a_lo;
    x.lda = q.lda;
    x.w_hi = q.w_hi;
    x.w_lo = q.w_lo;
    x.ldw = q.ldw;
    x.M = q.m;
    x.N = q.n;
    x.K = q.k;
    x.ep = epi_default();
    x.ep.act = act;
    x.ep.bias_on = (q.flags & JC_BIAS) != 0;
    x.ep.bias = q.bias;
    x.ep.accumulate = (q.flags & JC_ACCUMULATE) != 0;
    x.ep.c = q.c;
    x.ep.ldc = q.ldc;
    x.ep.cin = q.c;
    x.ep.ldcin = q.ldc;
  }
  if (const char* msg = check_gemm_group(g, count)) return fail(JC_ERR_UNSUPPORTED_SHAPE, msg);
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  cudaError_t e = launch_gemm_group(g, count, static_cast<cudaStream_t>(stream), rt->err);
  if (e != cudaSuccess) return fail_cuda(e, "grouped GEMM launch");
  return JC_OK;
}

jc_status jc_timestral_prep_device(int device, int rows, int encoder, int patch, const float* window,
                                   const uint8_t* observed, const int32_t* known, float minimum_scale, int use_asinh,
                                   float* tokens_out, void* stream) {
  clear_error();
  if (rows < 1 || encoder < 1 || patch < 1) return fail(JC_ERR_INVALID_ARG, "rows, encoder and patch must be >= 1");
  if (!window || !observed || !known || !tokens_out) return fail(JC_ERR_INVALID_ARG, "null pointer");
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  TsEnds ep;
  ep.rows = rows;
  ep.enc = encoder;
  ep.P = patch;
  ep.ll = encoder;
  ep.min_scale = minimum_scale;
  ep.use_asinh = use_asinh ? 1 : 0;
  // the per-patch frames and asinh flags live only for this call, in stream-ordered memory
  void* scratch = nullptr;
  const size_t frame_bytes = sizeof(float2) * static_cast<size_t>(rows) * encoder;
  cudaError_t e = cudaMallocAsync(&scratch, frame_bytes + rows, s);
  if (e != cudaSuccess) return fail(JC_ERR_OOM, std::string("scratch: ") + cudaGetErrorString(e));
  float2* frame = static_cast<float2*>(scratch);
  uint8_t* row_asinh = static_cast<uint8_t*>(scratch) + frame_bytes;
  launch_ts_scaler(window, observed, known, ep, frame, row_asinh, s);
  launch_ts_tokens(window, observed, frame, row_asinh, ep, tokens_out, s);
  e = cudaGetLastError();
  cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return fail_cuda(e, "prep launch");
  return JC_OK;
}

jc_status jc_chronos2_prep_device(int device, int rows, int context_patches, int output_patches, int patch,
                                  const float* window, const float* future, float time_encoding_scale,
                                  int use_arcsinh, float* tokens_out, void* stream) {
  clear_error();
  if (rows < 1 || context_patches < 1 || output_patches < 1 || patch < 1)
    return fail(JC_ERR_INVALID_ARG, "rows, patch counts and patch must be >= 1");
  if (!(time_encoding_scale > 0.0f)) return fail(JC_ERR_INVALID_ARG, "time encoding scale must be > 0");
  if (!window || !future || !tokens_out) return fail(JC_ERR_INVALID_ARG, "null pointer");
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  C2Ends ep;
  ep.rows = rows;
  ep.nc = context_patches;
  ep.h = output_patches;
  ep.P = patch;
  ep.use_arcsinh = use_arcsinh ? 1 : 0;
  ep.time_scale = time_encoding_scale;
  void* scratch = nullptr;  // the rows' (loc, scale), stream-ordered
  cudaError_t e = cudaMallocAsync(&scratch, sizeof(float2) * static_cast<size_t>(rows), s);
  if (e != cudaSuccess) return fail(JC_ERR_OOM, std::string("scratch: ") + cudaGetErrorString(e));
  float2* norm = static_cast<float2*>(scratch);
  launch_c2_norm(window, ep, norm, s);
  launch_c2_tokens(window, future, norm, ep, tokens_out, s);
  e = cudaGetLastError();
  cudaFreeAsync(scratch, s);
  if (e != cudaSuccess) return fail_cuda(e, "prep launch");
  return JC_OK;
}

jc_status jc_timestral_finish_device(int device, int rows, int steps, int quantiles, int median,
                                     const float* quantile_scale, int use_asinh, const float* loc_scale, float* raw,
                                     void* stream) {
  clear_error();
  if (rows < 1 || steps < 1 || quantiles < 1) return fail(JC_ERR_INVALID_ARG, "rows, steps and quantiles must be >= 1");
  if (quantiles > kMaxQuantiles)
    return fail(JC_ERR_UNSUPPORTED_SHAPE, "at most " + std::to_string(kMaxQuantiles) + " quantiles");
  if (median < 0 || median >= quantiles) return fail(JC_ERR_INVALID_ARG, "median index out of range");
  if (!quantile_scale || !loc_scale || !raw) return fail(JC_ERR_INVALID_ARG, "null pointer");
  if (reinterpret_cast<uintptr_t>(loc_scale) % 8 != 0) return fail(JC_ERR_INVALID_ARG, "loc_scale not 8-byte aligned");
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  TsEnds ep;
  ep.rows = rows;
  ep.enc = 1;  // one frame per row: the last context patch's
  ep.ll = 1;
  ep.Q = quantiles;
  ep.median = median;
  ep.use_asinh = use_asinh ? 1 : 0;
  for (int i = 0; i < quantiles; ++i) ep.qscale[i] = quantile_scale[i];
  launch_ts_finish(raw, reinterpret_cast<const float2*>(loc_scale), ep, steps, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? JC_OK : fail_cuda(e, "finish launch");
}

jc_status jc_chronos2_finish_device(int device, int rows, int output_patches, int patch, int quantiles,
                                    int use_arcsinh, const float* loc_scale, const float* raw, float* out,
                                    void* stream) {
  clear_error();
  if (rows < 1 || output_patches < 1 || patch < 1 || quantiles < 1)
    return fail(JC_ERR_INVALID_ARG, "rows, output patches, patch and quantiles must be >= 1");
  if (!loc_scale || !raw || !out) return fail(JC_ERR_INVALID_ARG, "null pointer");
  if (reinterpret_cast<uintptr_t>(loc_scale) % 8 != 0) return fail(JC_ERR_INVALID_ARG, "loc_scale not 8-byte aligned");
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  C2Ends ep;
  ep.rows = rows;
  ep.nc = 1;
  ep.h = output_patches;
  ep.P = patch;
  ep.Q = quantiles;
  ep.use_arcsinh = use_arcsinh ? 1 : 0;
  launch_c2_finish(raw, reinterpret_cast<const float2*>(loc_scale), ep, out, static_cast<cudaStream_t>(stream));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? JC_OK : fail_cuda(e, "finish launch");
}

jc_status jc_device_wait_selftest(int device, int limit_us) {
  clear_error();
  if (limit_us < 1 || limit_us > 1000000) return fail(JC_ERR_INVALID_ARG, "limit_us must be in [1, 1000000]");
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  wait_selftest_kernel<<<1, 32, 0, rt->stream>>>(rt->err, static_cast<uint64_t>(limit_us) * 1000ull);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) return fail_cuda(e, "wait self-test");
  return take_device_error(rt);
}

jc_status jc_device_sync(int device) {
  clear_error();
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  cudaSetDevice(device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail_cuda(e, "device synchronize");
  return take_device_error(rt);
}

}  // extern "C"

// The host ends of a Chronos-2 forward on the device: ModelPrep.of's instance norm and token
// assembly in front of the encoder (chronos2/ModelPrep.java:29-110: instanceNorm :73-95, scaled
// :98-101, asinh :103-107) and ModelPrep.finish after the output patch embedding (:116-137).
//
// The arithmetic is the reference's: the row statistics in double in the reference's order, the
// affine transform and the denormalisation in float with each product and sum rounded on its own
// (explicit _rn intrinsics, so nothing is contracted into an FMA). Only the double log and sinh
// are CUDA's own, within an ulp of the JDK's in double.
//
//   c2_norm_kernel    one thread per row: InstanceNorm's (loc, scale) of the row's window
//   c2_tokens_kernel  element-parallel: time encoding, scaled value, observed flag per step
//   c2_finish_kernel  element-parallel over the output: sinh·scale + loc, level-major per row

#include <cmath>
#include <cstdint>

#include "kernels.cuh"

namespace jc {
namespace {

// ModelPrep.asinh: log(a + sqrt(a² + 1)) in double on |v|, the sign put back, rounded to float.
__device__ __forceinline__ float asinh_ref(float v) {
  const double a = fabs(static_cast<double>(v));
  const double r = log(__dadd_rn(a, sqrt(__dadd_rn(__dmul_rn(a, a), 1.0))));
  return __double2float_rn(v < 0.0f ? -r : r);
}

// InstanceNorm's floor for a constant row (ModelPrep.EPS).
constexpr float kNormEps = 1e-5f;

__device__ __forceinline__ float f4_get(const float4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// Calls f(v) on x[0 .. W) in order. With vec (W a multiple of 32, x 16-byte aligned) 32 values are
// loaded together per round, one memory latency instead of 32, then visited in order.
template <typename F>
__device__ __forceinline__ void for_each_in_order(const float* x, long long W, bool vec, F&& f) {
  long long i = 0;
  if (vec) {
    for (; i + 32 <= W; i += 32) {
      float4 v[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = __ldg(reinterpret_cast<const float4*>(x + i) + k);
#pragma unroll
      for (int k = 0; k < 32; ++k) f(f4_get(v[k >> 2], k & 3));
    }
  }
  for (; i < W; ++i) f(x[i]);
}

__global__ void c2_norm_kernel(const float* __restrict__ window, C2Ends ep, float2* __restrict__ norm, bool vec) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= ep.rows) return;
  const long long W = static_cast<long long>(ep.nc) * ep.P;
  const float* x = window + row * W;
  double sum = 0.0;
  long long n = 0;
  for_each_in_order(x, W, vec, [&](float v) {
    if (!isnan(v)) {
      sum = __dadd_rn(sum, static_cast<double>(v));
      ++n;
    }
  });
  if (n == 0) {
    norm[row] = make_float2(0.0f, 1.0f);
    return;
  }
  const double dn = static_cast<double>(n);
  const float loc = __double2float_rn(__ddiv_rn(sum, dn));
  double ss = 0.0;
  for_each_in_order(x, W, vec, [&](float v) {
    if (!isnan(v)) {
      const float d = __fsub_rn(v, loc);
      ss = __dadd_rn(ss, __dmul_rn(static_cast<double>(d), static_cast<double>(d)));
    }
  });
  const float scale = __double2float_rn(sqrt(__ddiv_rn(ss, dn)));
  norm[row] = make_float2(loc, scale == 0.0f ? kNormEps : scale);
}

// ModelPrep.tokens [rows · (nc + h) · 3P]: per token its P time encodings, P scaled values, P
// observed flags; context tokens from the window (time t − nc·P), future tokens from the future
// covariates (time t).
__global__ void c2_tokens_kernel(const float* __restrict__ window, const float* __restrict__ future,
                                 const float2* __restrict__ norm, C2Ends ep, float* __restrict__ tok) {
  const int P = ep.P, nc = ep.nc, ne = ep.nc + ep.h;
  const long long per_row = static_cast<long long>(ne) * P;
  const long long total = static_cast<long long>(ep.rows) * per_row;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long i = e / per_row;
    const int rem = static_cast<int>(e - i * per_row);
    const int tp = rem / P, s = rem - tp * P;
    float time, x;
    if (tp < nc) {
      const int t = tp * P + s;
      time = __fdiv_rn(static_cast<float>(t - nc * P), ep.time_scale);
      x = window[i * nc * P + t];
    } else {
      const int t = (tp - nc) * P + s;
      time = __fdiv_rn(static_cast<float>(t), ep.time_scale);
      x = future[i * ep.h * P + t];
    }
    const bool obs = !isnan(x);
    float val = 0.0f;
    if (obs) {
      const float2 f = norm[i];
      const float v = __fdiv_rn(__fsub_rn(x, f.x), f.y);
      val = ep.use_arcsinh ? asinh_ref(v) : v;
    }
    float* out = tok + (i * ne + tp) * 3 * P + s;
    out[0] = time;
    out[P] = val;
    out[2 * P] = obs ? 1.0f : 0.0f;
  }
}

// out [rows · Q · h·P] from raw [rows · h · Q · P] (each output token's quantiles level-major).
__global__ void c2_finish_kernel(const float* __restrict__ raw, const float2* __restrict__ norm, C2Ends ep,
                                 float* __restrict__ out) {
  const int P = ep.P, Q = ep.Q, hp = ep.h * ep.P;
  const long long per_row = static_cast<long long>(Q) * hp;
  const long long total = static_cast<long long>(ep.rows) * per_row;
  for (long long o = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; o < total;
       o += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long i = o / per_row;
    const int rem = static_cast<int>(o - i * per_row);
    const int k = rem / hp, j = rem - k * hp;
    const int p = j / P, s = j - p * P;
    float v = raw[((i * ep.h + p) * Q + k) * P + s];
    if (ep.use_arcsinh) v = __double2float_rn(sinh(static_cast<double>(v)));
    const float2 f = norm[i];
    out[o] = __fadd_rn(__fmul_rn(v, f.y), f.x);
  }
}

}  // namespace

void launch_c2_norm(const float* window, const C2Ends& ep, float2* norm, cudaStream_t s) {
  if (ep.rows <= 0) return;
  const long long W = static_cast<long long>(ep.nc) * ep.P;
  const bool vec = W % 32 == 0 && reinterpret_cast<uintptr_t>(window) % 16 == 0;
  c2_norm_kernel<<<(ep.rows + 31) / 32, 32, 0, s>>>(window, ep, norm, vec);
}

void launch_c2_tokens(const float* window, const float* future, const float2* norm, const C2Ends& ep, float* tok,
                      cudaStream_t s) {
  const long long n = static_cast<long long>(ep.rows) * (ep.nc + ep.h) * ep.P;
  if (n <= 0) return;
  c2_tokens_kernel<<<grid_for(n, 256), 256, 0, s>>>(window, future, norm, ep, tok);
}

void launch_c2_finish(const float* raw, const float2* norm, const C2Ends& ep, float* out, cudaStream_t s) {
  const long long n = static_cast<long long>(ep.rows) * ep.Q * ep.h * ep.P;
  if (n <= 0) return;
  c2_finish_kernel<<<grid_for(n, 256), 256, 0, s>>>(raw, norm, ep, out);
}

}  // namespace jc

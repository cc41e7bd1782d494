// The host ends of a Timestral decode block on the device: the scaler and the patch tokens in
// front of the transformer (BlockPrep.of, timestral/BlockPrep.java:40-73, with Scaler.java's
// causalPatchLocScale :36-58, instanceNorm :100-124, affine :81-87 and asinh :89-93), and the
// monotone quantiles, denormalisation and clamping of infinities after the head
// (BlockPrep.finish, timestral/BlockPrep.java:81-101, with Quantiles.apply,
// timestral/Quantiles.java:53-69, Scaler.invert :127-130 and Scaler.clampNonFinite :136-148).
//
// Every operation is the reference's, in its order and at its precision: the statistics in
// double, the affine transform and the quantile sums in float, each product and sum rounded on
// its own (explicit _rn intrinsics, so nothing is contracted into an FMA), max/min with Java's
// NaN and signed-zero rules. Only the double transcendental functions (log, exp, log1p, sinh)
// are CUDA's own, within an ulp of the JDK's in double, so a float result can differ from the
// reference's only where its double value lies within an ulp of a float rounding boundary.
//
// Three kernels, each HBM- or FP64-bound and small next to the forward:
//   ts_scaler_kernel  one thread per row walks the row once in order (the Welford recurrence is
//                     sequential) and writes one (loc, scale) frame per patch
//   ts_tokens_kernel  element-parallel: scaled values and missing flags into the token rows
//   ts_finish_kernel  one thread per (row, step): the Q levels of that step in place

#include <cfloat>
#include <cmath>
#include <cstdint>

#include "kernels.cuh"

namespace jc {
namespace {

// Math.max / Math.min on doubles and floats: NaN if either argument is NaN, +0 over −0.
__device__ __forceinline__ double jmax(double a, double b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

__device__ __forceinline__ float jmaxf(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}

__device__ __forceinline__ float jminf(float a, float b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}

// Quantiles.clamp: ±inf to ±Float.MAX_VALUE, NaN kept.
__device__ __forceinline__ float clamp_finite(float v) { return jmaxf(-FLT_MAX, jminf(FLT_MAX, v)); }

// Scaler.asinh: log(a + sqrt(a² + 1)) in double on |v|, the sign put back, rounded to float.
__device__ __forceinline__ float asinh_ref(float v) {
  const double a = fabs(static_cast<double>(v));
  const double r = log(__dadd_rn(a, sqrt(__dadd_rn(__dmul_rn(a, a), 1.0))));
  return __double2float_rn(v < 0.0f ? -r : r);
}

// Quantiles.softplus: x above 20, else log1p(exp(x)) in double rounded to float.
__device__ __forceinline__ float softplus_ref(float x) {
  return x > 20.0f ? x : __double2float_rn(log1p(exp(static_cast<double>(x))));
}

// torch.finfo(torch.float32).eps, the floor of the affine transform's divisor (Scaler.FLOAT32_EPS).
constexpr float kFloat32Eps = 1.1920928955078125e-7f;

// The running state of Scaler.causalPatchLocScale: one step per value, in the reference's operation order.
struct Welford {
  double cum_w = 0.0, cum_x = 0.0, m2 = 0.0, prev = 0.0, mean = 0.0;

  __device__ __forceinline__ void step(float x, bool observed) {
    const double w = observed ? 1.0 : 0.0;
    const double xi = static_cast<double>(x);
    cum_w = __dadd_rn(cum_w, w);
    cum_x = __dadd_rn(cum_x, __dmul_rn(w, xi));
    mean = __ddiv_rn(cum_x, jmax(cum_w, 1.0));
    m2 = __dadd_rn(m2, __dmul_rn(__dmul_rn(__dsub_rn(xi, prev), __dsub_rn(xi, mean)), w));
    prev = mean;
  }

  // (loc, scale) at a patch's end: the Bessel-corrected std floored at min_scale, both rounded to float
  __device__ __forceinline__ float2 frame(double min_scale) const {
    const double var = __ddiv_rn(m2, jmax(__dsub_rn(jmax(cum_w, 1.0), 1.0), 1.0));
    return make_float2(__double2float_rn(mean), __double2float_rn(jmax(sqrt(var), min_scale)));
  }
};

__device__ __forceinline__ float f4_get(const float4& v, int k) {
  return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

__device__ __forceinline__ uint32_t u4_byte(const uint4& v, int k) {
  const int w = k >> 2;
  const uint32_t word = w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
  return (word >> ((k & 3) * 8)) & 0xffu;
}

// vec: rows of a multiple of 32 steps, window and flags 16-byte aligned
__global__ void ts_scaler_kernel(const float* __restrict__ win, const uint8_t* __restrict__ obs,
                                 const int* __restrict__ known, TsEnds ep, float2* __restrict__ frame,
                                 uint8_t* __restrict__ row_asinh, bool vec) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= ep.rows) return;
  const int P = ep.P, enc = ep.enc;
  const long long W = static_cast<long long>(enc) * P;
  const float* x = win + row * W;
  const uint8_t* o = obs + row * W;
  float2* fr = frame + static_cast<long long>(row) * enc;
  if (known[row]) {
    // Scaler.instanceNorm: whole-row statistics of a known-future covariate
    double n = 0.0, sum = 0.0;
    bool zero_one = true, any = false;
    for (long long i = 0; i < W; ++i) {
      const float xi = x[i];
      const bool ob = o[i] != 0;
      if (ob) {
        n = __dadd_rn(n, 1.0);
        sum = __dadd_rn(sum, static_cast<double>(xi));
        any = true;
      }
      zero_one &= xi == 0.0f || xi == 1.0f || !ob;
    }
    n = jmax(n, 1.0);
    const float loc = __double2float_rn(__ddiv_rn(sum, n));
    double ss = 0.0;
    for (long long i = 0; i < W; ++i) {
      const float d = o[i] ? __fsub_rn(x[i], loc) : 0.0f;
      ss = __dadd_rn(ss, __dmul_rn(static_cast<double>(d), static_cast<double>(d)));
    }
    const float sd = __double2float_rn(sqrt(static_cast<double>(__double2float_rn(__ddiv_rn(ss, n)))));
    const float scale = jmaxf(sd, ep.min_scale);
    const bool binary = zero_one && any;
    const float2 f = binary ? make_float2(0.0f, 1.0f) : make_float2(loc, scale);
    for (int p = 0; p < enc; ++p) fr[p] = f;
    row_asinh[row] = ep.use_asinh && !binary;
    return;
  }
  // Scaler.causalPatchLocScale: Welford over every observed value up to each patch's end
  Welford s;
  const double min_scale = static_cast<double>(ep.min_scale);
  int st = 0, p = 0;
  long long i = 0;
  if (vec) {
    // 32 steps per round: their values and flags loaded together (one memory latency instead of 32), then
    // walked in order
    for (; i + 32 <= W; i += 32) {
      float4 xv[8];
      uint4 ov[2];
#pragma unroll
      for (int k = 0; k < 8; ++k) xv[k] = __ldg(reinterpret_cast<const float4*>(x + i) + k);
#pragma unroll
      for (int k = 0; k < 2; ++k) ov[k] = __ldg(reinterpret_cast<const uint4*>(o + i) + k);
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        s.step(f4_get(xv[k >> 2], k & 3), u4_byte(ov[k >> 4], k & 15) != 0);
        if (++st == P) {
          fr[p++] = s.frame(min_scale);
          st = 0;
        }
      }
    }
  }
  for (; i < W; ++i) {
    s.step(x[i], o[i] != 0);
    if (++st == P) {
      fr[p++] = s.frame(min_scale);
      st = 0;
    }
  }
  row_asinh[row] = ep.use_asinh != 0;
}

// One scaled value (Scaler.affine) of step t of a row with frame f.
__device__ __forceinline__ float scaled_value(float x, bool observed, float2 f, bool use_asinh) {
  if (!observed) return 0.0f;
  const float v = __fdiv_rn(__fsub_rn(x, f.x), jmaxf(f.y, kFloat32Eps));
  return use_asinh ? asinh_ref(v) : v;
}

// V consecutive steps of one patch per thread (V = 4 when the patch size is a multiple of 4 and
// the window and flags are 16- and 4-byte aligned, else 1).
template <int V>
__global__ void ts_tokens_kernel(const float* __restrict__ win, const uint8_t* __restrict__ obs,
                                 const float2* __restrict__ frame, const uint8_t* __restrict__ row_asinh, TsEnds ep,
                                 float* __restrict__ tok) {
  const int P = ep.P, enc = ep.enc;
  const long long W = static_cast<long long>(enc) * P;
  const long long groups = static_cast<long long>(ep.rows) * W / V;
  for (long long g = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; g < groups;
       g += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long e = g * V;
    const long long row = e / W;
    const int t = static_cast<int>(e - row * W);
    const int p = t / P, st = t - p * P;
    const float2 f = frame[row * enc + p];
    const bool use = row_asinh[row] != 0;
    float* out = tok + (row * enc + p) * 2 * P + st;
    if constexpr (V == 4) {
      const float4 x = *reinterpret_cast<const float4*>(win + e);
      const uint32_t ob = *reinterpret_cast<const uint32_t*>(obs + e);
      const bool o0 = (ob & 0xffu) != 0, o1 = (ob & 0xff00u) != 0, o2 = (ob & 0xff0000u) != 0,
                 o3 = (ob & 0xff000000u) != 0;
      *reinterpret_cast<float4*>(out) = make_float4(scaled_value(x.x, o0, f, use), scaled_value(x.y, o1, f, use),
                                                    scaled_value(x.z, o2, f, use), scaled_value(x.w, o3, f, use));
      *reinterpret_cast<float4*>(out + P) = make_float4(o0 ? 0.0f : 1.0f, o1 ? 0.0f : 1.0f, o2 ? 0.0f : 1.0f,
                                                        o3 ? 0.0f : 1.0f);
    } else {
      const bool ob = obs[e] != 0;
      out[0] = scaled_value(win[e], ob, f, use);
      out[P] = ob ? 0.0f : 1.0f;
    }
  }
}

__global__ void ts_finish_kernel(float* __restrict__ q, const float2* __restrict__ frame, TsEnds ep, int steps) {
  const int Q = ep.Q, med = ep.median;
  const long long vectors = static_cast<long long>(ep.rows) * steps;
  for (long long vec = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; vec < vectors;
       vec += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = vec / steps;
    const float2 f = frame[row * ep.enc + ep.ll - 1];  // the last context patch's frame
    float* r = q + vec * Q;
    float v[kMaxQuantiles];
    for (int k = 0; k < Q; ++k) v[k] = r[k];
    // Quantiles.apply: each level's increment is read before the level is overwritten
    const float m = v[med];
    float up = 0.0f;
    for (int i = med + 1; i < Q; ++i) {
      up = __fadd_rn(up, __fmul_rn(ep.qscale[i], softplus_ref(v[i])));
      v[i] = clamp_finite(__fadd_rn(m, up));
    }
    float down = 0.0f;
    for (int i = med - 1; i >= 0; --i) {
      down = __fadd_rn(down, __fmul_rn(ep.qscale[i], softplus_ref(v[i])));
      v[i] = clamp_finite(__fsub_rn(m, down));
    }
    v[med] = clamp_finite(m);
    // Scaler.invert, then Scaler.clampNonFinite along the levels
    float mx = -INFINITY, mn = INFINITY;
    for (int k = 0; k < Q; ++k) {
      const float s = ep.use_asinh ? __double2float_rn(sinh(static_cast<double>(v[k]))) : v[k];
      const float y = __fadd_rn(__fmul_rn(s, f.y), f.x);
      v[k] = y;
      if (isfinite(y)) {
        mx = jmaxf(mx, y);
        mn = jminf(mn, y);
      }
    }
    for (int k = 0; k < Q; ++k) {
      const float y = v[k] == INFINITY ? mx : v[k] == -INFINITY ? mn : v[k];
      r[k] = isinf(y) ? 0.0f : y;
    }
  }
}

}  // namespace

void launch_ts_scaler(const float* win, const uint8_t* obs, const int* known, const TsEnds& ep, float2* frame,
                      uint8_t* row_asinh, cudaStream_t s) {
  if (ep.rows <= 0) return;
  // one warp per CTA spreads the rows' sequential walks over as many SMs as possible
  const long long W = static_cast<long long>(ep.enc) * ep.P;
  const bool vec = W % 32 == 0 && reinterpret_cast<uintptr_t>(win) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(obs) % 16 == 0;
  ts_scaler_kernel<<<(ep.rows + 31) / 32, 32, 0, s>>>(win, obs, known, ep, frame, row_asinh, vec);
}

void launch_ts_tokens(const float* win, const uint8_t* obs, const float2* frame, const uint8_t* row_asinh,
                      const TsEnds& ep, float* tok, cudaStream_t s) {
  const long long n = static_cast<long long>(ep.rows) * ep.enc * ep.P;
  if (n <= 0) return;
  const bool vec = ep.P % 4 == 0 && reinterpret_cast<uintptr_t>(win) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(obs) % 4 == 0 && reinterpret_cast<uintptr_t>(tok) % 16 == 0;
  if (vec) {
    ts_tokens_kernel<4><<<grid_for(n / 4, 256), 256, 0, s>>>(win, obs, frame, row_asinh, ep, tok);
  } else {
    ts_tokens_kernel<1><<<grid_for(n, 256), 256, 0, s>>>(win, obs, frame, row_asinh, ep, tok);
  }
}

void launch_ts_finish(float* raw, const float2* frame, const TsEnds& ep, int steps, cudaStream_t s) {
  const long long n = static_cast<long long>(ep.rows) * steps;
  if (n <= 0) return;
  ts_finish_kernel<<<grid_for(n, 128), 128, 0, s>>>(raw, frame, ep, steps);
}

}  // namespace jc

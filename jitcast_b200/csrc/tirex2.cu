// The TiRex-2 forward on B200: weights bound by checkpoint name and converted once per GPU; one plan
// (activation buffers + CUDA graph) per (rows, known covariates, kept rows); every dense layer a
// tcgen05 GEMM with its elementwise work fused into the epilogue, and the recurrent cells as
// companion kernels:
//
//   input stage      scaler (nanmean / nanstd, binary-aware, arcsinh) + patching → embedding tokens
//   input embedding  hidden (bias, SiLU) → output (bias) → residual (bias, += h)
//   per block        RMSNorm → cell → (+= h), or for known covariates: the cell on the time-reversed
//                    rows too, [forward | reverse] → combination → scatter, then h += cell, RMSNorm;
//                    SwiGLU FFN as one GEMM (gate and up rows interleaved, product in the epilogue)
//                    → down (+= h); variate mixer over the rows of multi-row groups
//     mLSTM cell     fused q|k|v|o|i|f projection GEMM (bias on the gates) → chunked stabilised
//                    parallel mLSTM with the per-head LayerNorm and σ(o) gate in its epilogue → out_proj
//     sLSTM cell     four headwise gate GEMMs (one per head, K = 128) → recurrence kernel (R·y per step
//                    on the SMs, state in registers) with the per-head LayerNorm in its epilogue
//   output           RMSNorm → hidden (bias, SiLU) → output (bias) → residual (+=) → unpatch (sinh,
//                    scale, loc) into [rows, Q, len]
//
// This replaces TornadoForward's task graph (tirex2/tornado/TornadoForward.java:561-658), its GEMM
// dispatch (:910-1085) and TiRexKernels (scalePatch :48, mlstmChunk :283, slstmRecurrence* :447-700,
// headLayerNorm :133, gather/scatter/concat :1004-1036, qkNorm :1065, variateAttention :1110, unpatch
// :979); the arithmetic is CpuReference.forward's (tirex2/cpu/CpuReference.java:67-266, Cells.java).
#include <cmath>
#include <cstring>
#include <thread>

#include "engine.h"
#include "kernels.cuh"
#include "opstore.cuh"
#include "runtime.h"

namespace jc {
namespace {

constexpr float kNormEps = 1e-6f;
constexpr float kMlstmEps = 1e-6f;
constexpr float kGateCap = 15.0f;
constexpr float kScalerEps = 1e-8f;
constexpr float kSinhClamp = 20.0f;
constexpr float kFloat32Eps = 1.1920928955078125e-07f;
constexpr int kDqk = 64, kDv = 128, kDh = 128;  // head widths the cells and the variate attention take

// ---- device kernels -----------------------------------------------------------------------------

__device__ __forceinline__ double asinh_d(double z) {
  const double a = fabs(z);
  const double r = log(a + sqrt(a * a + 1.0));
  return z < 0 ? -r : r;
}

// InputStage.apply (InputStage.java:37-93) on the uploaded x (0 where absent) and is-present flags:
// one block per row; sums in double. tok [(r·S + t), 0..P) = scaled values, [P, 2P) = is-present.
__global__ void scale_patch_kernel(const float* __restrict__ x, const float* __restrict__ present, int rows, int len,
                                   int P, int arcsinh, int binary_aware, int tok_kind, void* tok_hi, void* tok_lo,
                                   long long ld_tok, float* __restrict__ stats) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  __shared__ double s_sum[256];
  __shared__ int s_cnt[256], s_nb[256];
  const float* xr = x + static_cast<long long>(r) * len;
  const float* pr = present + static_cast<long long>(r) * len;
  double sum = 0;
  int cnt = 0, nb = 0;
  for (int t = threadIdx.x; t < len; t += blockDim.x) {
    if (pr[t] != 0.0f) {
      const float v = xr[t];
      sum += v;
      ++cnt;
      if (v != 0.0f && v != 1.0f) nb = 1;
    }
  }
  s_sum[threadIdx.x] = sum;
  s_cnt[threadIdx.x] = cnt;
  s_nb[threadIdx.x] = nb;
  __syncthreads();
  for (int st = blockDim.x / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) {
      s_sum[threadIdx.x] += s_sum[threadIdx.x + st];
      s_cnt[threadIdx.x] += s_cnt[threadIdx.x + st];
      s_nb[threadIdx.x] |= s_nb[threadIdx.x + st];
    }
    __syncthreads();
  }
  const int n = s_cnt[0];
  float loc = n == 0 ? 0.0f : static_cast<float>(s_sum[0] / n);
  const bool binary = binary_aware && s_nb[0] == 0;
  __syncthreads();
  double ss = 0;
  for (int t = threadIdx.x; t < len; t += blockDim.x)
    if (pr[t] != 0.0f) {
      const double dv = static_cast<double>(xr[t] - loc);
      ss += dv * dv;
    }
  s_sum[threadIdx.x] = ss;
  __syncthreads();
  for (int st = blockDim.x / 2; st > 0; st >>= 1) {
    if (threadIdx.x < st) s_sum[threadIdx.x] += s_sum[threadIdx.x + st];
    __syncthreads();
  }
  float scale = n == 0 ? 1.0f : static_cast<float>(sqrt(s_sum[0] / n));
  scale = fmaxf(scale, kScalerEps);
  if (binary) {
    loc = 0.0f;
    scale = 1.0f;
  }
  if (threadIdx.x == 0) {
    stats[r * 3] = loc;
    stats[r * 3 + 1] = scale;
    stats[r * 3 + 2] = binary ? 1.0f : 0.0f;
  }
  const bool do_asinh = arcsinh && !binary;
  const int S = len / P;
  for (int pos = threadIdx.x; pos < len; pos += blockDim.x) {
    const int t = pos / P, i = pos - t * P;
    const long long o = (static_cast<long long>(r) * S + t) * ld_tok;
    const bool here = pr[pos] != 0.0f;
    float z = (xr[pos] - loc) / scale;
    if (do_asinh) z = static_cast<float>(asinh_d(static_cast<double>(z)));
    put_op(tok_kind, tok_hi, tok_lo, o + i, here ? z : 0.0f);
    put_op(tok_kind, tok_hi, tok_lo, o + P + i, here ? 1.0f : 0.0f);
  }
}

__device__ __forceinline__ double log_sigmoid_d(double z) { return fmin(z, 0.0) - log1p(exp(-fabs(z))); }
__device__ __forceinline__ float soft_cap(float z) {
  return static_cast<float>(static_cast<double>(kGateCap) * tanh(static_cast<double>(z / kGateCap)));
}

constexpr int kMlT = 64;       // query and key tokens per block
constexpr int kMlThreads = 256;
constexpr int kMlPad = kMlT + 1;

// Dynamic shared memory of the mLSTM kernel for a sequence of S tokens.
size_t mlstm_smem(int S) {
  return sizeof(float) * (kMlT * kMlPad * 3 + kMlT * kDv) + sizeof(double) * 2 * S;
}

// The stabilised parallel mLSTM of one (row, head, 64-query block) (Cells.mlstmCore, Cells.java:74-118)
// with Cells.mlstm's per-head LayerNorm and σ(o) gate (:58-69) as its epilogue. proj [(r·S + t), ldp]
// holds q (heads·64) | k (heads·64) | v (heads·128) | o (heads·128) | i (heads) | f (heads).
//   F[t] = Σ_{u≤t} logσ(cap(f_u)),  a[s] = cap(i_s) − F[s],  M[t] = max(0, max_{s≤t} a[s]),  m[t] = F[t] + M[t]
//   C[t,s] = (q_t·k_s)/8 · exp(a[s] − M[t])   (= exp(F[t] − F[s] + i_s − m[t]), s ≤ t)
//   h_t = Σ_s C[t,s] v_s / (max(|Σ_s C[t,s]|, exp(−m[t])) + eps)
// Keys stream through shared memory 64 at a time, so any S fits.
__global__ void __launch_bounds__(kMlThreads) mlstm_kernel(const float* __restrict__ proj, long long ldp, int rows,
                                                           int S, int heads, const float* __restrict__ norm_w,
                                                           int out_kind, void* out_hi, void* out_lo, long long ld_out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  float* qs = reinterpret_cast<float*>(sm_raw);  // [64][65]
  float* ks = qs + kMlT * kMlPad;               // [64][65]
  float* cs = ks + kMlT * kMlPad;               // [64][65]
  float* vs = cs + kMlT * kMlPad;               // [64][128]
  double* cumf = reinterpret_cast<double*>(vs + kMlT * kDv);  // [S]: F, then reused
  double* aa = cumf + S;                                       // [S]: a[s], then prefix max
  const int rh = blockIdx.x;
  const int r = rh / heads, head = rh % heads;
  const int qb = blockIdx.y;
  const int tid = threadIdx.x;
  if (r >= rows) return;
  const long long row0 = static_cast<long long>(r) * S;
  const int k_off = heads * kDqk, v_off = 2 * heads * kDqk, o_off = v_off + heads * kDv, i_off = o_off + heads * kDv,
            f_off = i_off + heads;
  // gates over the whole prefix this query block needs
  const int t_end = min(S, (qb + 1) * kMlT);
  for (int s = tid; s < t_end; s += kMlThreads) {
    const float* ps = proj + (row0 + s) * ldp;
    cumf[s] = log_sigmoid_d(static_cast<double>(soft_cap(ps[f_off + head])));
    aa[s] = static_cast<double>(soft_cap(ps[i_off + head]));
  }
  __syncthreads();
  // inclusive prefix sum of F (Hillis-Steele over t_end ≤ S elements)
  for (int off = 1; off < t_end; off <<= 1) {
    double v[4];
    int c = 0;
    for (int s = tid; s < t_end; s += kMlThreads) v[c++] = s >= off ? cumf[s - off] : 0.0;
    __syncthreads();
    c = 0;
    for (int s = tid; s < t_end; s += kMlThreads) cumf[s] += v[c++];
    __syncthreads();
  }
  for (int s = tid; s < t_end; s += kMlThreads) aa[s] -= cumf[s];
  __syncthreads();
  // m[t] needs the prefix max of a; the key weights need a itself, kept in ks-sized scratch per key block
  // below, so the prefix max goes into a second pass stored in cumf (F is only needed as F[t] + M[t]).
  // First store F[t] for the query block's tokens, then overwrite cumf with the prefix max of a.
  __shared__ double fq[kMlT];
  for (int t = tid; t < kMlT; t += kMlThreads) fq[t] = qb * kMlT + t < S ? cumf[qb * kMlT + t] : 0.0;
  __syncthreads();
  for (int s = tid; s < t_end; s += kMlThreads) cumf[s] = aa[s];
  __syncthreads();
  for (int off = 1; off < t_end; off <<= 1) {
    double v[4];
    int c = 0;
    for (int s = tid; s < t_end; s += kMlThreads) v[c++] = s >= off ? cumf[s - off] : -INFINITY;
    __syncthreads();
    c = 0;
    for (int s = tid; s < t_end; s += kMlThreads) cumf[s] = fmax(cumf[s], v[c++]);
    __syncthreads();
  }
  // query block
  const int tq = tid >> 2, lq = tid & 3;
  const int tglob = qb * kMlT + tq;
  const bool tlive = tglob < S;
  for (int i = tid; i < kMlT * kDqk; i += kMlThreads) {
    const int t = i / kDqk, j = i % kDqk;
    const int tg = qb * kMlT + t;
    qs[t * kMlPad + j] = tg < S ? proj[(row0 + tg) * ldp + head * kDqk + j] : 0.0f;
  }
  const double Mt = tlive ? fmax(0.0, cumf[tglob]) : 0.0;
  const double mt = tlive ? fq[tq] + Mt : 0.0;
  float num[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) num[i] = 0.0f;
  float den = 0.0f;
  const float scale = 0.125f;  // 1/√64
  for (int kb = 0; kb <= qb; ++kb) {
    __syncthreads();
    for (int i = tid; i < kMlT * kDqk; i += kMlThreads) {
      const int s = i / kDqk, j = i % kDqk;
      const int sg = kb * kMlT + s;
      ks[s * kMlPad + j] = sg < S ? proj[(row0 + sg) * ldp + k_off + head * kDqk + j] : 0.0f;
    }
    for (int i = tid; i < kMlT * kDv / 4; i += kMlThreads) {
      const int s = i / (kDv / 4), j4 = i % (kDv / 4);
      const int sg = kb * kMlT + s;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (sg < S) v = *reinterpret_cast<const float4*>(proj + (row0 + sg) * ldp + v_off + head * kDv + 4 * j4);
      *reinterpret_cast<float4*>(vs + s * kDv + 4 * j4) = v;
    }
    __syncthreads();
    // C[t, s] for this thread's token and keys s ≡ lq (mod 4)
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int s = lq + 4 * i;
      const int sg = kb * kMlT + s;
      float c = 0.0f;
      if (tlive && sg <= tglob) {
        float dot = 0.0f;
#pragma unroll 16
        for (int j = 0; j < kDqk; ++j) dot = fmaf(qs[tq * kMlPad + j], ks[s * kMlPad + j], dot);
        c = dot * scale * expf(static_cast<float>(aa[sg] - Mt));
      }
      cs[tq * kMlPad + s] = c;
      den += c;
    }
    __syncthreads();
    // num[t, j] += Σ_s C[t, s] v[s, j] for j ≡ lq (mod 4)
    for (int s = 0; s < kMlT; ++s) {
      const float c = cs[tq * kMlPad + s];
#pragma unroll
      for (int i = 0; i < 32; ++i) num[i] = fmaf(c, vs[s * kDv + lq + 4 * i], num[i]);
    }
  }
  den += __shfl_xor_sync(0xffffffffu, den, 1);
  den += __shfl_xor_sync(0xffffffffu, den, 2);
  const float norm = static_cast<float>(fmax(fabs(static_cast<double>(den)), exp(-mt)) + static_cast<double>(kMlstmEps));
  float mean = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    num[i] /= norm;
    mean += num[i];
  }
  mean += __shfl_xor_sync(0xffffffffu, mean, 1);
  mean += __shfl_xor_sync(0xffffffffu, mean, 2);
  mean *= 1.0f / kDv;
  float var = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const float dv = num[i] - mean;
    var = fmaf(dv, dv, var);
  }
  var += __shfl_xor_sync(0xffffffffu, var, 1);
  var += __shfl_xor_sync(0xffffffffu, var, 2);
  var *= 1.0f / kDv;
  const float inv = rsqrtf(var + kNormEps);
  if (!tlive) return;
  const float* og = proj + (row0 + tglob) * ldp + o_off + head * kDv;
  const long long orow = (row0 + tglob) * ld_out + head * kDv;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int j = lq + 4 * i;
    const float v = (num[i] - mean) * inv * norm_w[head * kDv + j];
    const float g = 1.0f / (1.0f + expf(-og[j]));
    put_op(out_kind, out_hi, out_lo, orow + j, g * v);
  }
}

constexpr int kSlRows = 16;  // rows per block: one warp per row in the state update
constexpr int kSlThreads = 4 * kDh;

// The sLSTM recurrence of kSlRows rows and one head (Cells.slstmRecurrence, Cells.java:170-218) with the
// per-head LayerNorm of its output (Cells.slstm :139-140) in the epilogue. wx [(r·S + t), ldwx] holds the
// headwise gate pre-activations at columns head·512 + g·128 + e (g = i, f, z, o); R [H, 128, 4, 128],
// bias [H, 4, 128]. out (+)= LN(y)·w at columns head·128 + e.
__global__ void __launch_bounds__(kSlThreads) slstm_kernel(const float* __restrict__ wx, long long ldwx, int rows,
                                                           int S, int heads, const float* __restrict__ R,
                                                           const float* __restrict__ bias,
                                                           const float* __restrict__ norm_w, float* out,
                                                           long long ld_out, int accumulate) {
  __shared__ __align__(16) float ys[kSlRows][kDh];
  __shared__ float raws[kSlRows][4 * kDh];
  const int head = blockIdx.y;
  const int r0 = blockIdx.x * kSlRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < kSlRows * kDh; i += kSlThreads) ys[i / kDh][i % kDh] = 0.0f;
  const float* Rh = R + static_cast<long long>(head) * kDh * 4 * kDh;
  const float bcol = bias[head * 4 * kDh + tid];
  float c[4] = {0, 0, 0, 0}, n[4] = {0, 0, 0, 0}, m[4] = {0, 0, 0, 0};
  const int row = r0 + warp;
  const bool live = row < rows;
  __syncthreads();
  for (int t = 0; t < S; ++t) {
    // phase A: raw[rb][col] = (wx + b) + Σ_p y[rb][p]·R[p][col], col = tid
    float acc[kSlRows];
#pragma unroll
    for (int rb = 0; rb < kSlRows; ++rb) acc[rb] = 0.0f;
    for (int p = 0; p < kDh; p += 4) {
      const float w0 = __ldg(Rh + (p + 0) * 4 * kDh + tid);
      const float w1 = __ldg(Rh + (p + 1) * 4 * kDh + tid);
      const float w2 = __ldg(Rh + (p + 2) * 4 * kDh + tid);
      const float w3 = __ldg(Rh + (p + 3) * 4 * kDh + tid);
#pragma unroll
      for (int rb = 0; rb < kSlRows; ++rb) {
        const float4 y4 = *reinterpret_cast<const float4*>(&ys[rb][p]);
        acc[rb] = fmaf(y4.x, w0, fmaf(y4.y, w1, fmaf(y4.z, w2, fmaf(y4.w, w3, acc[rb]))));
      }
    }
#pragma unroll
    for (int rb = 0; rb < kSlRows; ++rb) {
      const int rr = r0 + rb;
      const float g = rr < rows ? wx[(static_cast<long long>(rr) * S + t) * ldwx + head * 4 * kDh + tid] : 0.0f;
      raws[rb][tid] = (g + bcol) + acc[rb];
    }
    __syncthreads();
    // phase B: warp `warp` updates row r0 + warp, lanes own e = 4·lane .. 4·lane + 3
    float y[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = 4 * lane + u;
      const float ir = raws[warp][e], fr = raws[warp][kDh + e], zr = raws[warp][2 * kDh + e],
                  orw = raws[warp][3 * kDh + e];
      const float logf_ = (fminf(fr, 0.0f) - log1pf(expf(-fabsf(fr)))) + m[u];
      const float mn = t == 0 ? ir : fmaxf(ir, logf_);
      const float ig = expf(ir - mn), fg = expf(logf_ - mn);
      c[u] = fg * c[u] + ig * tanhf(zr);
      n[u] = fmaxf(fg * n[u] + ig, 1.0f);
      y[u] = (1.0f / (1.0f + expf(-orw))) * c[u] / n[u];
      m[u] = mn;
      ys[warp][e] = y[u];
    }
    float mean = y[0] + y[1] + y[2] + y[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mean += __shfl_xor_sync(0xffffffffu, mean, o);
    mean *= 1.0f / kDh;
    float var = 0.0f;
#pragma unroll
    for (int u = 0; u < 4; ++u) var = fmaf(y[u] - mean, y[u] - mean, var);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
    var *= 1.0f / kDh;
    const float inv = rsqrtf(var + kNormEps);
    if (live) {
      float* dst = out + (static_cast<long long>(row) * S + t) * ld_out + head * kDh + 4 * lane;
      float4 v;
      v.x = (y[0] - mean) * inv * norm_w[head * kDh + 4 * lane];
      v.y = (y[1] - mean) * inv * norm_w[head * kDh + 4 * lane + 1];
      v.z = (y[2] - mean) * inv * norm_w[head * kDh + 4 * lane + 2];
      v.w = (y[3] - mean) * inv * norm_w[head * kDh + 4 * lane + 3];
      if (accumulate) {
        const float4 o = *reinterpret_cast<const float4*>(dst);
        v.x += o.x;
        v.y += o.y;
        v.z += o.z;
        v.w += o.w;
      }
      *reinterpret_cast<float4*>(dst) = v;
    }
    __syncthreads();
  }
}

// Attention across the kept rows of a group at one patch and head (CpuReference.variateMixer,
// CpuReference.java:182-223): one warp per (kept query row, patch, head), 128-wide heads (4 per lane),
// optional RMS qk-norm without weight (eps = FLT_EPSILON), covariate queries do not see targets.
// qkv [(k·S + t), ld_qkv] fp32 with q | k | v at 0, d, 2d.
__global__ void variate_attention_kernel(const float* __restrict__ qkv, long long ld_qkv, int nk, int S, int heads,
                                         int d, const int* __restrict__ gs, const int* __restrict__ ge,
                                         const int* __restrict__ kt, int qk_norm, int out_kind, void* out_hi,
                                         void* out_lo, long long ld_out) {
  const long long wid = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const long long total = static_cast<long long>(nk) * S * heads;
  if (wid >= total) return;
  const int head = static_cast<int>(wid % heads);
  const long long qt = wid / heads;  // qi·S + t
  const int t = static_cast<int>(qt % S);
  const int qi = static_cast<int>(qt / S);
  const float4 q = *reinterpret_cast<const float4*>(qkv + qt * ld_qkv + head * kDh + 4 * lane);
  float qv[4] = {q.x, q.y, q.z, q.w};
  auto rms4 = [&](float* v) {
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(ss) / kDh + kFloat32Eps));
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] *= inv;
  };
  if (qk_norm) rms4(qv);
  const float scale = rsqrtf(static_cast<float>(kDh));
  const bool q_target = kt[qi] != 0;
  float mx = -INFINITY, l = 0.0f, acc[4] = {0, 0, 0, 0};
  for (int ki = gs[qi]; ki < ge[qi]; ++ki) {
    if (!q_target && kt[ki] != 0) continue;
    const long long kr = (static_cast<long long>(ki) * S + t) * ld_qkv;
    const float4 k4 = *reinterpret_cast<const float4*>(qkv + kr + d + head * kDh + 4 * lane);
    float kv[4] = {k4.x, k4.y, k4.z, k4.w};
    if (qk_norm) rms4(kv);
    float dot = qv[0] * kv[0] + qv[1] * kv[1] + qv[2] * kv[2] + qv[3] * kv[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float s = dot * scale;
    const float mn = fmaxf(mx, s);
    const float corr = expf(mx - mn), p = expf(s - mn);
    const float4 v4 = *reinterpret_cast<const float4*>(qkv + kr + 2 * d + head * kDh + 4 * lane);
    l = l * corr + p;
    acc[0] = acc[0] * corr + p * v4.x;
    acc[1] = acc[1] * corr + p * v4.y;
    acc[2] = acc[2] * corr + p * v4.z;
    acc[3] = acc[3] * corr + p * v4.w;
    mx = mn;
  }
  const long long o = qt * ld_out + head * kDh + 4 * lane;
#pragma unroll
  for (int u = 0; u < 4; ++u) put_op(out_kind, out_hi, out_lo, o + u, acc[u] / l);
}

// Row copies in 16-byte units. gather: dst row k·S + t ← src row idx[k]·S + (reverse ? S−1−t : t);
// scatter: dst row idx[k]·S + t ← src row k·S + t. Rows are row_bytes long (a multiple of 16) at
// pitches ld_dst / ld_src bytes.
__global__ void rows_kernel(const uint8_t* __restrict__ src, long long ld_src, uint8_t* __restrict__ dst,
                            long long ld_dst, const int* __restrict__ idx, int n, int S, int row_bytes, int reverse,
                            int scatter) {
  const int per_row = row_bytes / 16;
  const long long total = static_cast<long long>(n) * S * per_row;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % per_row);
    const long long kt = i / per_row;
    const int k = static_cast<int>(kt / S), t = static_cast<int>(kt % S);
    long long sr, dr;
    if (scatter) {
      sr = kt;
      dr = static_cast<long long>(idx[k]) * S + t;
    } else {
      sr = static_cast<long long>(idx[k]) * S + (reverse ? S - 1 - t : t);
      dr = kt;
    }
    reinterpret_cast<uint4*>(dst + dr * ld_dst)[c] = reinterpret_cast<const uint4*>(src + sr * ld_src)[c];
  }
}

// [forward | reverse] for the combination GEMM (CpuReference.java:128-136):
// cat[k·S + t] = yc[known[k]·S + t] (d values) then rev[k·S + S−1−t] (d values), as an operand.
__global__ void concat_kernel(const float* __restrict__ yc, const float* __restrict__ rev, const int* __restrict__ known,
                              int nk, int S, int d, int kind, void* hi, void* lo, long long ld) {
  const long long total = static_cast<long long>(nk) * S * 2 * d;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % (2 * d));
    const long long kt = i / (2 * d);
    const int k = static_cast<int>(kt / S), t = static_cast<int>(kt % S);
    const float v = c < d ? yc[(static_cast<long long>(known[k]) * S + t) * d + c]
                          : rev[(static_cast<long long>(k) * S + (S - 1 - t)) * d + (c - d)];
    put_op(kind, hi, lo, kt * ld + c, v);
  }
}

// h[r] += y[r]; xn[r] = RMSNorm(h[r])·w as an operand (one warp per row).
__global__ void add_rmsnorm_kernel(float* __restrict__ h, const float* __restrict__ y, long long rows, int d,
                                   const float* __restrict__ w, float eps, int kind, void* hi, void* lo, long long ld) {
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long r = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    float* hr = h + r * d;
    const float* yr = y + r * d;
    float ss = 0.0f;
    for (int c = lane; c < d; c += 32) {
      const float v = hr[c] + yr[c];
      hr[c] = v;
      ss += v * v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(ss) / d + eps));
    for (int c = lane; c < d; c += 32) put_op(kind, hi, lo, r * ld + c, hr[c] * inv * w[c]);
  }
}

// CpuReference.unpatch (CpuReference.java:238-266): y [(r·S + t), Q·P] → out [r, Q, S·P],
// sinh(clamp(v, ±20)) unless the row is binary (or arcsinh is off), then ·scale + loc.
__global__ void unpatch_kernel(const float* __restrict__ y, const float* __restrict__ stats, float* __restrict__ out,
                               int rows, int S, int Q, int P, int arcsinh) {
  const long long len = static_cast<long long>(S) * P;
  const long long total = static_cast<long long>(rows) * Q * len;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long pos = i % len;
    const long long rq = i / len;
    const int q = static_cast<int>(rq % Q), r = static_cast<int>(rq / Q);
    const int t = static_cast<int>(pos / P), k = static_cast<int>(pos % P);
    float v = y[(static_cast<long long>(r) * S + t) * Q * P + q * P + k];
    if (arcsinh && stats[r * 3 + 2] == 0.0f) v = sinhf(fmaxf(-kSinhClamp, fminf(kSinhClamp, v)));
    out[i] = v * stats[r * 3 + 1] + stats[r * 3];
  }
}

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

// ---- engine -------------------------------------------------------------------------------------

struct TxBlock {
  int kind = 0;
  float* norm_lstm = nullptr;
  DevLinear proj, out_proj;  // mLSTM
  float* head_norm = nullptr;
  std::vector<DevLinear> gates;  // sLSTM, one [4·128, 128] linear per head
  float *rec = nullptr, *sbias = nullptr, *group_norm = nullptr;
  DevLinear comb, w12, down;
  float* norm_ffn = nullptr;
  float *norm_attn = nullptr, *norm_ffn_attn = nullptr;
  DevLinear vqkv, vo, vin, vout;
};

struct TxWeights {
  DevLinear in_h, in_o, in_r;
  std::vector<TxBlock> blocks;
  float* out_norm = nullptr;
  DevLinear out_h, out_o, out_r;
};

struct TxPlan {
  int rows = 0, nk = 0, nv = 0;
  DeviceMem mem;
  float *x = nullptr, *present = nullptr, *stats = nullptr;
  int *known = nullptr, *kept = nullptr, *gs = nullptr, *ge = nullptr, *kt = nullptr;
  OpBuf tok, emb_h, xn, hn, rev_in, cat, act, vatt, vhid, oh;
  float *h = nullptr, *proj = nullptr, *yc = nullptr, *rev_out = nullptr, *comb = nullptr, *xk = nullptr,
        *vqkv = nullptr, *y = nullptr, *out = nullptr;
  GraphRunner graph;
};

struct TxDevice : DeviceSlot {
  TxWeights w;
  std::list<std::unique_ptr<TxPlan>> plans;
  Profiler prof;
  cudaEvent_t ev_in = nullptr, ev_out = nullptr;
  ~TxDevice() {
    if (ev_in) cudaEventDestroy(ev_in);
    if (ev_out) cudaEventDestroy(ev_out);
  }
};

struct Tirex2Engine : jc_engine {
  int d = 0, nb = 0, P = 0, in_ff = 0, out_ff = 0, ctx = 0, fut = 0, Q = 0, H = 0, SH = 0, VH = 0;
  int arcsinh = 0, binary_aware = 0, qk_norm = 0, F = 0, qk = 0;
  float out_eps = 0;
  std::vector<int> kinds;
  int op = kOpBF16;
  std::vector<std::unique_ptr<TxDevice>> devs;

  int S() const { return (ctx + fut) / P; }
  int L() const { return ctx + fut; }
  int proj_cols() const { return 2 * qk + 2 * d + 2 * H; }
  int slots() const override { return static_cast<int>(devs.size()); }
  DeviceSlot* slot(int i) override { return devs[i].get(); }
  Profiler* profiler(int i) override { return &devs[i]->prof; }
  void drop_plans() override {
    for (auto& dv : devs) {
      cudaSetDevice(dv->device);
      cudaStreamSynchronize(dv->stream);
      dv->plans.clear();
    }
  }
};

struct HostBlock {
  const float *norm_lstm = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *igw = nullptr,
              *igb = nullptr, *fgw = nullptr, *fgb = nullptr, *head_norm = nullptr, *out_proj = nullptr;
  const float* sg[4] = {nullptr, nullptr, nullptr, nullptr};
  const float *rec = nullptr, *sbias = nullptr, *group_norm = nullptr;
  const float *comb = nullptr, *norm_ffn = nullptr, *up_gate = nullptr, *up = nullptr, *down = nullptr;
  const float *norm_attn = nullptr, *wq = nullptr, *wk = nullptr, *wv = nullptr, *wo = nullptr,
              *norm_ffn_attn = nullptr, *ffn_in = nullptr, *ffn_out = nullptr;
};

struct HostTx {
  const float* in[6];
  std::vector<HostBlock> blocks;
  const float* out_norm;
  const float* out[6];
};

// TiRex2Weights.load / Binder.block (TiRex2Weights.java:128-247): every tensor once, exact shapes.
bool bind(const Tirex2Engine& e, Binder& b, HostTx* hw) {
  const long long d = e.d, p = e.P;
  auto residual = [&](const std::string& pre, long long in, long long hid, long long out, const float** w) {
    w[0] = b.take(pre + ".hidden_layer.weight", {hid, in});
    w[1] = b.take(pre + ".hidden_layer.bias", {hid});
    w[2] = b.take(pre + ".output_layer.weight", {out, hid});
    w[3] = b.take(pre + ".output_layer.bias", {out});
    w[4] = b.take(pre + ".residual_layer.weight", {out, in});
    w[5] = b.take(pre + ".residual_layer.bias", {out});
  };
  residual("input_patch_embedding", 2 * p, e.in_ff, d, hw->in);
  for (int i = 0; i < e.nb; ++i) {
    HostBlock B;
    const std::string s = "stack." + std::to_string(i), cell = s + ".time_mixer.fwd_cell";
    if (e.kinds[i] == JC_TIREX_MLSTM) {
      B.q = b.take(cell + ".q.weight", {e.qk, d});
      B.k = b.take(cell + ".k.weight", {e.qk, d});
      B.v = b.take(cell + ".v.weight", {d, d});
      B.o = b.take(cell + ".ogate_preact.weight", {d, d});
      B.igw = b.take(cell + ".igate_preact.weight", {e.H, d});
      B.igb = b.take(cell + ".igate_preact.bias", {e.H});
      B.fgw = b.take(cell + ".fgate_preact.weight", {e.H, d});
      B.fgb = b.take(cell + ".fgate_preact.bias", {e.H});
      B.head_norm = b.take(cell + ".multihead_norm.weight", {d});
      B.out_proj = b.take(cell + ".out_proj.weight", {d, d});
    } else {
      const long long h = e.SH, dh = d / e.SH;
      // FlashRNN gate slots (i, f, z, o) come from the checkpoint's (fgate, igate, zgate, ogate)
      // tensors in that order (TiRex2Weights.java:211-216)
      const char* slot_src[4] = {"fgate", "igate", "zgate", "ogate"};
      for (int g = 0; g < 4; ++g) B.sg[g] = b.take(cell + "." + slot_src[g] + ".weight", {h, dh, dh});
      B.rec = b.take(cell + "._recurrent_kernel_", {h, dh, 4, dh});
      B.sbias = b.take(cell + "._bias_", {h, 4, dh});
      B.group_norm = b.take(cell + ".group_norm.weight", {d});
    }
    const std::string tm = s + ".time_mixer";
    B.norm_lstm = b.take(tm + ".norm_lstm.weight", {d});
    B.comb = b.take(tm + ".combination.weight", {d, 2 * d});
    B.norm_ffn = b.take(tm + ".norm_ffn.weight", {d});
    B.up_gate = b.take(tm + ".ffn.proj_up_gate.weight", {e.F, d});
    B.up = b.take(tm + ".ffn.proj_up.weight", {e.F, d});
    B.down = b.take(tm + ".ffn.proj_down.weight", {d, e.F});
    const std::string vm = s + ".variate_mixer";
    B.norm_attn = b.take(vm + ".norm_attn.weight", {d});
    B.wq = b.take(vm + ".attn.WQ.weight", {d, d});
    B.wk = b.take(vm + ".attn.WK.weight", {d, d});
    B.wv = b.take(vm + ".attn.WV.weight", {d, d});
    B.wo = b.take(vm + ".attn.WO.weight", {d, d});
    B.norm_ffn_attn = b.take(vm + ".norm_ffn.weight", {d});
    B.ffn_in = b.take(vm + ".ffn.wi.weight", {4 * d, d});
    B.ffn_out = b.take(vm + ".ffn.wo.weight", {d, 4 * d});
    hw->blocks.push_back(B);
  }
  hw->out_norm = b.take("stack_out_norm.weight", {d});
  residual("output_patch_embedding", d, e.out_ff, static_cast<long long>(e.Q) * p, hw->out);
  return b.require_all_bound();
}

std::vector<float> stack_rows(std::initializer_list<std::pair<const float*, long long>> parts, int cols) {
  long long rows = 0;
  for (auto& pr : parts) rows += pr.second;
  std::vector<float> out(static_cast<size_t>(rows) * cols);
  size_t at = 0;
  for (auto& pr : parts) {
    std::memcpy(out.data() + at, pr.first, sizeof(float) * pr.second * cols);
    at += static_cast<size_t>(pr.second) * cols;
  }
  return out;
}

bool upload(Tirex2Engine& e, const HostTx& hw, TxDevice& dv, std::string* err) {
  const int d = e.d, P = e.P, op = e.op, F = e.F;
  DeviceMem& m = dv.weights;
  TxWeights& w = dv.w;
  if (!upload_linear(m, op, hw.in[0], hw.in[1], 2 * P, e.in_ff, &w.in_h, err) ||
      !upload_linear(m, op, hw.in[2], hw.in[3], e.in_ff, d, &w.in_o, err) ||
      !upload_linear(m, op, hw.in[4], hw.in[5], 2 * P, d, &w.in_r, err))
    return false;
  for (int i = 0; i < e.nb; ++i) {
    const HostBlock& B = hw.blocks[i];
    TxBlock T;
    T.kind = e.kinds[i];
    if (!(T.norm_lstm = upload_f32(m, B.norm_lstm, d, err))) return false;
    if (T.kind == JC_TIREX_MLSTM) {
      // q | k | v | o | i | f as one projection; the bias is zero except on the two gates
      std::vector<float> wcat = stack_rows({{B.q, e.qk}, {B.k, e.qk}, {B.v, d}, {B.o, d}, {B.igw, e.H}, {B.fgw, e.H}},
                                           d);
      std::vector<float> bcat(e.proj_cols(), 0.0f);
      std::memcpy(bcat.data() + 2 * e.qk + 2 * d, B.igb, sizeof(float) * e.H);
      std::memcpy(bcat.data() + 2 * e.qk + 2 * d + e.H, B.fgb, sizeof(float) * e.H);
      if (!upload_linear(m, op, wcat.data(), bcat.data(), d, e.proj_cols(), &T.proj, err) ||
          !(T.head_norm = upload_f32(m, B.head_norm, d, err)) ||
          !upload_linear(m, op, B.out_proj, nullptr, d, d, &T.out_proj, err))
        return false;
    } else {
      // per head h: rows g·128 + o of a [512, 128] linear are slot g's gates[h][o][:]
      std::vector<float> gh(static_cast<size_t>(4) * kDh * kDh);
      for (int h = 0; h < e.SH; ++h) {
        for (int g = 0; g < 4; ++g)
          std::memcpy(gh.data() + static_cast<size_t>(g) * kDh * kDh, B.sg[g] + static_cast<size_t>(h) * kDh * kDh,
                      sizeof(float) * kDh * kDh);
        DevLinear lin;
        if (!upload_linear(m, op, gh.data(), nullptr, kDh, 4 * kDh, &lin, err)) return false;
        T.gates.push_back(lin);
      }
      if (!(T.rec = upload_f32(m, B.rec, static_cast<size_t>(e.SH) * kDh * 4 * kDh, err)) ||
          !(T.sbias = upload_f32(m, B.sbias, static_cast<size_t>(e.SH) * 4 * kDh, err)) ||
          !(T.group_norm = upload_f32(m, B.group_norm, d, err)))
        return false;
    }
    // the SwiGLU GEMM: rows 64u..64u+31 are proj_up_gate rows 32u.. (SiLU), 64u+32.. proj_up rows 32u..
    std::vector<float> w12(static_cast<size_t>(2) * F * d);
    for (int u = 0; u < F / 32; ++u)
      for (int r = 0; r < 32; ++r) {
        std::memcpy(&w12[(static_cast<size_t>(64) * u + r) * d], B.up_gate + (static_cast<size_t>(32) * u + r) * d,
                    sizeof(float) * d);
        std::memcpy(&w12[(static_cast<size_t>(64) * u + 32 + r) * d], B.up + (static_cast<size_t>(32) * u + r) * d,
                    sizeof(float) * d);
      }
    std::vector<float> qkv = stack_rows({{B.wq, d}, {B.wk, d}, {B.wv, d}}, d);
    if (!upload_linear(m, op, B.comb, nullptr, 2 * d, d, &T.comb, err) ||
        !(T.norm_ffn = upload_f32(m, B.norm_ffn, d, err)) ||
        !upload_linear(m, op, w12.data(), nullptr, d, 2 * F, &T.w12, err) ||
        !upload_linear(m, op, B.down, nullptr, F, d, &T.down, err) ||
        !(T.norm_attn = upload_f32(m, B.norm_attn, d, err)) ||
        !upload_linear(m, op, qkv.data(), nullptr, d, 3 * d, &T.vqkv, err) ||
        !upload_linear(m, op, B.wo, nullptr, d, d, &T.vo, err) ||
        !(T.norm_ffn_attn = upload_f32(m, B.norm_ffn_attn, d, err)) ||
        !upload_linear(m, op, B.ffn_in, nullptr, d, 4 * d, &T.vin, err) ||
        !upload_linear(m, op, B.ffn_out, nullptr, 4 * d, d, &T.vout, err))
      return false;
    w.blocks.push_back(std::move(T));
  }
  if (!(w.out_norm = upload_f32(m, hw.out_norm, d, err))) return false;
  const int qp = e.Q * P;
  return upload_linear(m, op, hw.out[0], hw.out[1], d, e.out_ff, &w.out_h, err) &&
         upload_linear(m, op, hw.out[2], hw.out[3], e.out_ff, qp, &w.out_o, err) &&
         upload_linear(m, op, hw.out[4], hw.out[5], d, qp, &w.out_r, err);
}

std::unique_ptr<TxPlan> make_plan(const Tirex2Engine& e, int rows, int nk, int nv) {
  auto p = std::make_unique<TxPlan>();
  p->rows = rows;
  p->nk = nk;
  p->nv = nv;
  const int S = e.S(), d = e.d, op = e.op, L = e.L();
  const long long T = static_cast<long long>(rows) * S, TK = static_cast<long long>(nk) * S,
                  TV = static_cast<long long>(nv) * S, TC = std::max(T, TK);
  const long long cell_cols = std::max<long long>(round_up(e.proj_cols(), 8), 4LL * d);
  DeviceMem& m = p->mem;
  auto f32 = [&](long long n) { return static_cast<float*>(m.alloc(sizeof(float) * std::max(n, 1LL))); };
  auto i32 = [&](long long n) { return static_cast<int*>(m.alloc(sizeof(int) * std::max(n, 1LL))); };
  bool ok = (p->x = f32(static_cast<long long>(rows) * L)) && (p->present = f32(static_cast<long long>(rows) * L)) &&
            (p->stats = f32(3LL * rows)) && (p->known = i32(nk)) && (p->kept = i32(nv)) && (p->gs = i32(nv)) &&
            (p->ge = i32(nv)) && (p->kt = i32(nv)) && alloc_op(m, op, T, 2 * e.P, &p->tok) &&
            alloc_op(m, op, T, e.in_ff, &p->emb_h) && (p->h = f32(T * d)) && alloc_op(m, op, TC, d, &p->xn) &&
            alloc_op(m, op, TC, d, &p->hn) && (p->proj = f32(TC * cell_cols)) && alloc_op(m, op, T, e.F, &p->act) &&
            alloc_op(m, op, T, e.out_ff, &p->oh) && (p->y = f32(T * e.Q * e.P)) &&
            (p->out = f32(static_cast<long long>(rows) * e.Q * L));
  if (ok && nk > 0)
    ok = (p->yc = f32(T * d)) && alloc_op(m, op, TK, d, &p->rev_in) && (p->rev_out = f32(TK * d)) &&
         alloc_op(m, op, TK, 2 * d, &p->cat) && (p->comb = f32(TK * d));
  if (ok && nv > 0)
    ok = (p->xk = f32(TV * d)) && (p->vqkv = f32(TV * 3 * d)) && alloc_op(m, op, TV, d, &p->vatt) &&
         alloc_op(m, op, TV, 4 * d, &p->vhid);
  if (!ok) {
    cudaGetLastError();
    return nullptr;
  }
  return p;
}

TxPlan* get_plan(Tirex2Engine& e, TxDevice& dv, int rows, int nk, int nv, std::string* err) {
  for (auto it = dv.plans.begin(); it != dv.plans.end(); ++it) {
    TxPlan* p = it->get();
    if (p->rows == rows && p->nk == nk && p->nv == nv) {
      dv.plans.splice(dv.plans.begin(), dv.plans, it);
      return p;
    }
  }
  while (static_cast<int>(dv.plans.size()) >= std::max(1, e.max_plans)) dv.plans.pop_back();
  auto p = make_plan(e, rows, nk, nv);
  if (!p && !dv.plans.empty()) {
    cudaStreamSynchronize(dv.stream);
    dv.plans.clear();
    p = make_plan(e, rows, nk, nv);
  }
  if (!p) {
    *err = "out of device memory for a plan of " + std::to_string(rows) + " rows";
    return nullptr;
  }
  dv.plans.push_front(std::move(p));
  return dv.plans.front().get();
}

cudaError_t gemm(TxDevice& dv, GemmArgs& g, cudaStream_t s, const char* name) {
  dv.prof.begin(s, name, 2.0 * g.M * g.N * g.K);
  cudaError_t r = launch_gemm(g, s, dv.err);
  dv.prof.end(s);
  return r;
}

void set_out(EpiParams& ep, int op, const OpBuf& o) {
  ep.o_kind = out_of_op(op);
  ep.o_hi = o.hi;
  ep.o_lo = o.lo;
  ep.ldo = o.ld;
}

void into_f32(GemmArgs& g, float* c, long long ldc, bool accumulate) {
  g.ep.c = c;
  g.ep.ldc = ldc;
  if (accumulate) {
    g.ep.cin = c;
    g.ep.ldcin = ldc;
    g.ep.accumulate = 1;
  }
}

// A column window of an operand buffer (the K slice of one sLSTM head).
OpBuf cols_of(const OpBuf& a, int op, long long col0) {
  OpBuf v = a;
  const long long off = col0 * static_cast<long long>(op_esize(op));
  v.hi = static_cast<uint8_t*>(a.hi) + off;
  v.lo = a.lo ? static_cast<uint8_t*>(a.lo) + off : nullptr;
  return v;
}

#define JC_TRY(x)                   \
  do {                              \
    if ((r = (x)) != cudaSuccess) { \
      return r;                     \
    }                               \
  } while (0)

// One cell pass over `rows` rows of `in` (already RMS-normalised) into dst [rows·S, d] fp32, stored or
// added (TornadoForward.Plan.cell, TornadoForward.java:698-766).
cudaError_t run_cell(const Tirex2Engine& e, TxDevice& dv, TxPlan& p, const TxBlock& B, const OpBuf& in, int rows,
                     float* dst, bool accumulate, cudaStream_t s) {
  const int S = e.S(), d = e.d, op = e.op;
  const long long T = static_cast<long long>(rows) * S;
  Profiler& prof = dv.prof;
  cudaError_t r;
  if (B.kind == JC_TIREX_MLSTM) {
    const long long ldp = round_up(e.proj_cols(), 8);
    GemmArgs g = gemm_args(op, in, T, B.proj);
    into_f32(g, p.proj, ldp, false);
    JC_TRY(gemm(dv, g, s, "gemm.proj"));
    const size_t smem = mlstm_smem(S);
    dim3 grid(rows * e.H, (S + kMlT - 1) / kMlT);
    prof.begin(s, "mlstm", 2.0 * rows * e.H * (0.5 * S * S) * (kDqk + kDv));
    mlstm_kernel<<<grid, kMlThreads, smem, s>>>(p.proj, ldp, rows, S, e.H, B.head_norm, out_of_op(op), p.hn.hi,
                                                  p.hn.lo, p.hn.ld);
    prof.end(s);
    JC_TRY(cudaGetLastError());
    g = gemm_args(op, p.hn, T, B.out_proj);
    into_f32(g, dst, d, accumulate);
    JC_TRY(gemm(dv, g, s, "gemm.out_proj"));
  } else {
    const long long ldw = 4LL * d;
    for (int h = 0; h < e.SH; ++h) {
      GemmArgs g = gemm_args(op, cols_of(in, op, static_cast<long long>(h) * kDh), T, B.gates[h]);
      into_f32(g, p.proj + h * 4 * kDh, ldw, false);
      JC_TRY(gemm(dv, g, s, "gemm.gates"));
    }
    dim3 grid((rows + kSlRows - 1) / kSlRows, e.SH);
    prof.begin(s, "slstm", 2.0 * T * e.SH * kDh * 4 * kDh);
    slstm_kernel<<<grid, kSlThreads, 0, s>>>(p.proj, ldw, rows, S, e.SH, B.rec, B.sbias, B.group_norm, dst, d,
                                               accumulate ? 1 : 0);
    prof.end(s);
    JC_TRY(cudaGetLastError());
  }
  return cudaSuccess;
}

cudaError_t enqueue_forward(const Tirex2Engine& e, TxDevice& dv, TxPlan& p, cudaStream_t s) {
  const int R = p.rows, nk = p.nk, nv = p.nv, S = e.S(), d = e.d, op = e.op, L = e.L(), P = e.P;
  const long long T = static_cast<long long>(R) * S, TK = static_cast<long long>(nk) * S,
                  TV = static_cast<long long>(nv) * S;
  const int ok_kind = out_of_op(op);
  const size_t es = op_esize(op);
  const TxWeights& w = dv.w;
  Profiler& prof = dv.prof;
  cudaError_t r;
  prof.begin(s, "scale", 0);
  scale_patch_kernel<<<R, 256, 0, s>>>(p.x, p.present, R, L, P, e.arcsinh, e.binary_aware, ok_kind, p.tok.hi,
                                       p.tok.lo, p.tok.ld, p.stats);
  prof.end(s);
  JC_TRY(cudaGetLastError());
  GemmArgs g = gemm_args(op, p.tok, T, w.in_h);
  g.ep.act = kActSilu;
  set_out(g.ep, op, p.emb_h);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  g = gemm_args(op, p.emb_h, T, w.in_o);
  into_f32(g, p.h, d, false);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  g = gemm_args(op, p.tok, T, w.in_r);
  into_f32(g, p.h, d, true);
  JC_TRY(gemm(dv, g, s, "gemm.embed"));
  for (const TxBlock& B : w.blocks) {
    prof.begin(s, "rmsnorm", 0);
    launch_rmsnorm(p.h, d, B.norm_lstm, d, kNormEps, ok_kind, p.xn.hi, p.xn.lo, p.xn.ld, T, 0, 0, 0, s);
    prof.end(s);
    if (nk > 0) {
      // the reverse pass first, while xn still holds RMSNorm(h) (TornadoForward.java:590-612)
      prof.begin(s, "gather", 0);
      for (int part = 0; part < (op == kOpSplit ? 2 : 1); ++part) {
        const void* src = part ? p.xn.lo : p.xn.hi;
        void* dst = part ? p.rev_in.lo : p.rev_in.hi;
        rows_kernel<<<grid_for(TK * p.xn.ld * es / 16, 256), 256, 0, s>>>(
            static_cast<const uint8_t*>(src), p.xn.ld * es, static_cast<uint8_t*>(dst), p.rev_in.ld * es, p.known, nk,
            S, static_cast<int>(p.xn.ld * es), 1, 0);
      }
      prof.end(s);
      JC_TRY(run_cell(e, dv, p, B, p.rev_in, nk, p.rev_out, false, s));
      JC_TRY(run_cell(e, dv, p, B, p.xn, R, p.yc, false, s));
      prof.begin(s, "gather", 0);
      concat_kernel<<<grid_for(TK * 2 * d, 256), 256, 0, s>>>(p.yc, p.rev_out, p.known, nk, S, d, ok_kind, p.cat.hi,
                                                              p.cat.lo, p.cat.ld);
      prof.end(s);
      g = gemm_args(op, p.cat, TK, B.comb);
      into_f32(g, p.comb, d, false);
      JC_TRY(gemm(dv, g, s, "gemm.comb"));
      prof.begin(s, "gather", 0);
      rows_kernel<<<grid_for(TK * d * 4 / 16, 256), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(p.comb),
                                                                 4LL * d, reinterpret_cast<uint8_t*>(p.yc), 4LL * d,
                                                                 p.known, nk, S, 4 * d, 0, 1);
      prof.end(s);
      prof.begin(s, "rmsnorm", 0);
      add_rmsnorm_kernel<<<grid_for(T * 32, 256), 256, 0, s>>>(p.h, p.yc, T, d, B.norm_ffn, kNormEps, ok_kind, p.xn.hi,
                                                               p.xn.lo, p.xn.ld);
      prof.end(s);
    } else {
      JC_TRY(run_cell(e, dv, p, B, p.xn, R, p.h, true, s));
      prof.begin(s, "rmsnorm", 0);
      launch_rmsnorm(p.h, d, B.norm_ffn, d, kNormEps, ok_kind, p.xn.hi, p.xn.lo, p.xn.ld, T, 0, 0, 0, s);
      prof.end(s);
    }
    JC_TRY(cudaGetLastError());
    g = gemm_args(op, p.xn, T, B.w12);
    g.ep.mode = kEpiSwiGLU;
    set_out(g.ep, op, p.act);
    JC_TRY(gemm(dv, g, s, "gemm.w12"));
    g = gemm_args(op, p.act, T, B.down);
    into_f32(g, p.h, d, true);
    JC_TRY(gemm(dv, g, s, "gemm.down"));
    if (nv > 0) {
      // the variate mixer over the kept rows (TornadoForward.java:768-827)
      prof.begin(s, "gather", 0);
      rows_kernel<<<grid_for(TV * d * 4 / 16, 256), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(p.h), 4LL * d,
                                                                 reinterpret_cast<uint8_t*>(p.xk), 4LL * d, p.kept, nv,
                                                                 S, 4 * d, 0, 0);
      prof.end(s);
      prof.begin(s, "rmsnorm", 0);
      launch_rmsnorm(p.xk, d, B.norm_attn, d, kNormEps, ok_kind, p.xn.hi, p.xn.lo, p.xn.ld, TV, 0, 0, 0, s);
      prof.end(s);
      g = gemm_args(op, p.xn, TV, B.vqkv);
      into_f32(g, p.vqkv, 3LL * d, false);
      JC_TRY(gemm(dv, g, s, "gemm.variate"));
      prof.begin(s, "variate", 4.0 * TV * d);
      const long long warps = TV * e.VH;
      variate_attention_kernel<<<static_cast<int>((warps * 32 + 255) / 256), 256, 0, s>>>(
          p.vqkv, 3LL * d, nv, S, e.VH, d, p.gs, p.ge, p.kt, e.qk_norm, ok_kind, p.vatt.hi, p.vatt.lo, p.vatt.ld);
      prof.end(s);
      JC_TRY(cudaGetLastError());
      g = gemm_args(op, p.vatt, TV, B.vo);
      into_f32(g, p.xk, d, true);
      JC_TRY(gemm(dv, g, s, "gemm.variate"));
      prof.begin(s, "rmsnorm", 0);
      launch_rmsnorm(p.xk, d, B.norm_ffn_attn, d, kNormEps, ok_kind, p.xn.hi, p.xn.lo, p.xn.ld, TV, 0, 0, 0, s);
      prof.end(s);
      g = gemm_args(op, p.xn, TV, B.vin);
      g.ep.act = kActSilu;
      set_out(g.ep, op, p.vhid);
      JC_TRY(gemm(dv, g, s, "gemm.variate"));
      g = gemm_args(op, p.vhid, TV, B.vout);
      into_f32(g, p.xk, d, true);
      JC_TRY(gemm(dv, g, s, "gemm.variate"));
      prof.begin(s, "gather", 0);
      rows_kernel<<<grid_for(TV * d * 4 / 16, 256), 256, 0, s>>>(reinterpret_cast<const uint8_t*>(p.xk), 4LL * d,
                                                                 reinterpret_cast<uint8_t*>(p.h), 4LL * d, p.kept, nv,
                                                                 S, 4 * d, 0, 1);
      prof.end(s);
      JC_TRY(cudaGetLastError());
    }
  }
  prof.begin(s, "rmsnorm", 0);
  launch_rmsnorm(p.h, d, w.out_norm, d, e.out_eps, ok_kind, p.xn.hi, p.xn.lo, p.xn.ld, T, 0, 0, 0, s);
  prof.end(s);
  g = gemm_args(op, p.xn, T, w.out_h);
  g.ep.act = kActSilu;
  set_out(g.ep, op, p.oh);
  JC_TRY(gemm(dv, g, s, "gemm.head"));
  const long long qp = static_cast<long long>(e.Q) * P;
  g = gemm_args(op, p.oh, T, w.out_o);
  into_f32(g, p.y, qp, false);
  JC_TRY(gemm(dv, g, s, "gemm.head"));
  g = gemm_args(op, p.xn, T, w.out_r);
  into_f32(g, p.y, qp, true);
  JC_TRY(gemm(dv, g, s, "gemm.head"));
  prof.begin(s, "unpatch", 0);
  unpatch_kernel<<<grid_for(static_cast<long long>(R) * e.Q * L, 256), 256, 0, s>>>(p.y, p.stats, p.out, R, S, e.Q,
                                                                                     P, e.arcsinh);
  prof.end(s);
  return cudaGetLastError();
}
#undef JC_TRY

jc_status check_batch(const Tirex2Engine& e, const jc_tirex2_batch* b, bool host) {
  if (!b) return fail(JC_ERR_INVALID_ARG, "null batch");
  if (b->rows < 1) return fail(JC_ERR_INVALID_ARG, "rows must be >= 1");
  if (!b->x || !b->present) return fail(JC_ERR_INVALID_ARG, "null x or present");
  if (b->n_known < 0 || b->n_known > b->rows || b->n_kept < 0 || b->n_kept > b->rows)
    return fail(JC_ERR_INVALID_ARG, "known / kept counts out of range");
  if (b->n_known > 0 && !b->known) return fail(JC_ERR_INVALID_ARG, "null known list");
  if (b->n_kept > 0 && (!b->kept || !b->group_start || !b->group_end || !b->kept_target))
    return fail(JC_ERR_INVALID_ARG, "null kept lists");
  if (!host) return JC_OK;
  for (int i = 0; i < b->n_known; ++i)
    if (b->known[i] < 0 || b->known[i] >= b->rows || (i > 0 && b->known[i] <= b->known[i - 1]))
      return fail(JC_ERR_INVALID_ARG, "known rows must be increasing row indices");
  for (int i = 0; i < b->n_kept; ++i) {
    const int s = b->group_start[i], t = b->group_end[i];
    if (b->kept[i] < 0 || b->kept[i] >= b->rows || (i > 0 && b->kept[i] <= b->kept[i - 1]))
      return fail(JC_ERR_INVALID_ARG, "kept rows must be increasing row indices");
    if (s < 0 || s > i || t <= i || t > b->n_kept || b->group_start[s] != s || b->group_end[s] != t ||
        t - s < 2 || b->kept[t - 1] - b->kept[s] != t - 1 - s)
      return fail(JC_ERR_INVALID_ARG, "rows of a group are not contiguous (kept " + std::to_string(i) + ")");
  }
  (void)e;
  return JC_OK;
}

// The structure lists of rows [r0, r1) of a host batch, rebased to the shard.
struct ShardLists {
  std::vector<int> known, kept, gs, ge, kt;
};

ShardLists shard_lists(const jc_tirex2_batch* b, int r0, int r1) {
  ShardLists l;
  for (int i = 0; i < b->n_known; ++i)
    if (b->known[i] >= r0 && b->known[i] < r1) l.known.push_back(b->known[i] - r0);
  int base = -1;
  for (int i = 0; i < b->n_kept; ++i)
    if (b->kept[i] >= r0 && b->kept[i] < r1) {
      if (base < 0) base = i;
      l.kept.push_back(b->kept[i] - r0);
      l.gs.push_back(b->group_start[i] - base);
      l.ge.push_back(b->group_end[i] - base);
      l.kt.push_back(b->kept_target[i]);
    }
  return l;
}

jc_status run_shard(Tirex2Engine& e, TxDevice& dv, const jc_tirex2_batch* b, int r0, int r1, float* out, bool host,
                    cudaStream_t stream, std::string* err) {
  if (cudaSetDevice(dv.device) != cudaSuccess) {
    *err = "cannot select device " + std::to_string(dv.device);
    return JC_ERR_CUDA;
  }
  cudaStream_t s = dv.stream;
  if (!host && (cudaEventRecord(dv.ev_in, stream) != cudaSuccess || cudaStreamWaitEvent(s, dv.ev_in, 0) != cudaSuccess)) {
    *err = "cannot order the caller's stream before the forward";
    return JC_ERR_CUDA;
  }
  const int rows = r1 - r0, L = e.L();
  ShardLists lists;
  int nk = b->n_known, nv = b->n_kept;
  if (host) {
    lists = shard_lists(b, r0, r1);
    nk = static_cast<int>(lists.known.size());
    nv = static_cast<int>(lists.kept.size());
  }
  TxPlan* p = get_plan(e, dv, rows, nk, nv, err);
  if (!p) return JC_ERR_OOM;
  const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  const size_t xbytes = sizeof(float) * static_cast<size_t>(rows) * L;
  cudaError_t ce = cudaMemcpyAsync(p->x, b->x + static_cast<size_t>(r0) * L, xbytes, kind, s);
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(p->present, b->present + static_cast<size_t>(r0) * L, xbytes, kind, s);
  auto put = [&](int* dst, const int* src, int n) {
    if (ce == cudaSuccess && n > 0) ce = cudaMemcpyAsync(dst, src, sizeof(int) * n, kind, s);
  };
  if (host) {
    put(p->known, lists.known.data(), nk);
    put(p->kept, lists.kept.data(), nv);
    put(p->gs, lists.gs.data(), nv);
    put(p->ge, lists.ge.data(), nv);
    put(p->kt, lists.kt.data(), nv);
    // the host vectors must outlive the copies from pageable memory
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  } else {
    put(p->known, b->known, nk);
    put(p->kept, b->kept, nv);
    put(p->gs, b->group_start, nv);
    put(p->ge, b->group_end, nv);
    put(p->kt, b->kept_target, nv);
  }
  if (ce != cudaSuccess) {
    *err = std::string("upload: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  dv.prof.on = e.profile;
  Tirex2Engine& ec = e;
  TxDevice& dvc = dv;
  ce = p->graph.run(s, [&](cudaStream_t st) { return enqueue_forward(ec, dvc, *p, st); }, e.use_graph && !e.profile);
  if (ce != cudaSuccess) {
    *err = std::string("forward: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  const size_t per_row = static_cast<size_t>(e.Q) * L;
  ce = cudaMemcpyAsync(out + static_cast<size_t>(r0) * per_row, p->out, sizeof(float) * rows * per_row,
                       host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s);
  if (ce != cudaSuccess) {
    *err = std::string("download: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  if (!host) {
    if (cudaEventRecord(dv.ev_out, s) != cudaSuccess || cudaStreamWaitEvent(stream, dv.ev_out, 0) != cudaSuccess) {
      *err = "cannot order the caller's stream after the forward";
      return JC_ERR_CUDA;
    }
    return JC_OK;
  }
  ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) {
    *err = std::string("forward: ") + cudaGetErrorString(ce);
    return JC_ERR_CUDA;
  }
  if (e.profile) dv.prof.collect();
  uint32_t word = 0;
  cudaMemcpy(&word, dv.err, sizeof word, cudaMemcpyDeviceToHost);
  if (word) {
    cudaMemset(dv.err, 0, sizeof word);
    *err = "a device wait gave up (error bits " + std::to_string(word) + ")";
    return JC_ERR_TIMEOUT;
  }
  return JC_OK;
}

}  // namespace
}  // namespace jc

using namespace jc;

extern "C" {

jc_status jc_engine_create_tirex2(const jc_tirex2_desc* desc, const jc_tensor_view* weights, int n_weights,
                                  const int* devices, int n_devices, jc_precision precision, jc_engine** out) {
  clear_error();
  if (!out) return fail(JC_ERR_INVALID_ARG, "null engine out-pointer");
  *out = nullptr;
  if (!desc || !weights || n_weights < 1) return fail(JC_ERR_INVALID_ARG, "null description or weights");
  if (!valid_precision_code(precision)) return fail(JC_ERR_INVALID_ARG, "unknown precision");
  const jc_tirex2_desc& c = *desc;
  if (c.embedding_dim < 1 || c.num_blocks < 1 || c.patch_size < 1 || c.input_ff_dim < 1 || c.output_ff_dim < 1 ||
      c.context_len < 1 || c.future_len < 0 || c.num_quantiles < 1 || !c.block_types)
    return fail(JC_ERR_INVALID_ARG, "non-positive model dimensions or no block types");
  if ((c.context_len + c.future_len) % c.patch_size != 0)
    return fail(JC_ERR_INVALID_ARG, "context_len + future_len must be a multiple of the patch size");
  if (c.time_mixer_heads < 1 || c.slstm_heads < 1 || c.variate_heads < 1 || c.embedding_dim % c.time_mixer_heads ||
      c.embedding_dim % c.slstm_heads || c.embedding_dim % c.variate_heads)
    return fail(JC_ERR_INVALID_ARG, "embedding_dim is not divisible by the head counts");
  for (int i = 0; i < c.num_blocks; ++i)
    if (c.block_types[i] != JC_TIREX_MLSTM && c.block_types[i] != JC_TIREX_SLSTM)
      return fail(JC_ERR_INVALID_ARG, "unknown block type at block " + std::to_string(i));
  // the cells and the variate attention take 128-wide heads (64-wide mLSTM q/k), as the reference's
  // device kernels do (TornadoForward.java:261-264, :708-710, :784-786)
  if (c.embedding_dim / c.time_mixer_heads != kDv || c.embedding_dim / c.slstm_heads != kDh ||
      c.embedding_dim / c.variate_heads != kDh)
    return fail(JC_ERR_UNSUPPORTED_SHAPE, "unsupported head widths (this engine takes 128-wide heads: embedding_dim " +
                                              std::to_string(c.embedding_dim) + ")");
  auto e = std::make_unique<Tirex2Engine>();
  e->family = 3;
  e->d = c.embedding_dim;
  e->nb = c.num_blocks;
  e->P = c.patch_size;
  e->in_ff = c.input_ff_dim;
  e->out_ff = c.output_ff_dim;
  e->ctx = c.context_len;
  e->fut = c.future_len;
  e->Q = c.num_quantiles;
  e->H = c.time_mixer_heads;
  e->SH = c.slstm_heads;
  e->VH = c.variate_heads;
  e->arcsinh = c.use_arcsinh ? 1 : 0;
  e->binary_aware = c.binary_aware ? 1 : 0;
  e->qk_norm = c.use_qk_norm ? 1 : 0;
  e->out_eps = c.stack_out_norm_eps;
  e->kinds.assign(c.block_types, c.block_types + c.num_blocks);
  e->qk = static_cast<int>(static_cast<float>(c.embedding_dim) * 0.5f);
  {
    const int raw = static_cast<int>(static_cast<float>(c.embedding_dim) * 2.6667f);
    e->F = (raw + 63) / 64 * 64;  // TiRex2Config.ffnDim (TiRex2Config.java:119-122)
  }
  e->op = op_of_precision(precision);
  Binder binder(weights, n_weights);
  HostTx hw;
  if (!bind(*e, binder, &hw)) return fail(JC_ERR_INVALID_ARG, binder.error());
  std::vector<int> devs = (n_devices <= 0 || !devices) ? std::vector<int>{0}
                                                       : std::vector<int>(devices, devices + n_devices);
  for (int dev : devs) {
    std::string why;
    if (!device_rt(dev, &why)) return fail(JC_ERR_NO_DEVICE, why);
    auto dv = std::make_unique<TxDevice>();
    dv->device = dev;
    cudaSetDevice(dev);
    if (cudaStreamCreateWithFlags(&dv->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&dv->err, sizeof(uint32_t)) != cudaSuccess || cudaMemset(dv->err, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_in, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&dv->ev_out, cudaEventDisableTiming) != cudaSuccess)
      return fail_cuda(cudaGetLastError(), "engine device setup");
    // the mLSTM kernel's prefix scans hold 4 tokens per thread, and its gate prefix lives in shared memory
    const size_t smem = mlstm_smem(e->S());
    if (e->S() > 4 * kMlThreads || smem > 227 * 1024)
      return fail(JC_ERR_UNSUPPORTED_SHAPE, "sequence of " + std::to_string(e->S()) + " patches is too long (max " +
                                                std::to_string(4 * kMlThreads) + ")");
    if (cudaFuncSetAttribute(mlstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
        cudaSuccess)
      return fail_cuda(cudaGetLastError(), "mLSTM kernel setup");
    std::string err;
    if (!upload(*e, hw, *dv, &err)) return fail(JC_ERR_OOM, err);
    e->devs.push_back(std::move(dv));
  }
  *out = e.release();
  return JC_OK;
}

jc_status jc_forward_tirex2(jc_engine* engine, const jc_tirex2_batch* batch, float* out) {
  clear_error();
  if (!engine || engine->family != 3) return fail(JC_ERR_INVALID_ARG, "not a TiRex-2 engine");
  auto* e = static_cast<Tirex2Engine*>(engine);
  if (!out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_batch(*e, batch, true);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  // every row's group range: a kept row's group, or the row alone
  const int rows = batch->rows;
  std::vector<int> gstart(rows), gend(rows);
  for (int i = 0; i < rows; ++i) {
    gstart[i] = i;
    gend[i] = i + 1;
  }
  for (int i = 0; i < batch->n_kept; ++i) {
    gstart[batch->kept[i]] = batch->kept[batch->group_start[i]];
    gend[batch->kept[i]] = batch->kept[batch->group_end[i] - 1] + 1;
  }
  const int parts = std::min<int>(static_cast<int>(e->devs.size()), rows);
  std::vector<int> cuts = shard_rows(rows, gstart.data(), gend.data(), parts);
  std::vector<jc_status> status(parts, JC_OK);
  std::vector<std::string> errs(parts);
  auto work = [&](int i) {
    if (cuts[i + 1] > cuts[i])
      status[i] = run_shard(*e, *e->devs[i], batch, cuts[i], cuts[i + 1], out, true, nullptr, &errs[i]);
  };
  if (parts == 1) {
    work(0);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < parts; ++i) th.emplace_back(work, i);
    for (auto& t : th) t.join();
  }
  for (int i = 0; i < parts; ++i)
    if (status[i] != JC_OK) return fail(status[i], "GPU " + std::to_string(e->devs[i]->device) + ": " + errs[i]);
  return JC_OK;
}

jc_status jc_forward_tirex2_device(jc_engine* engine, int slot, const jc_tirex2_batch* batch, float* out,
                                   void* stream) {
  clear_error();
  if (!engine || engine->family != 3) return fail(JC_ERR_INVALID_ARG, "not a TiRex-2 engine");
  auto* e = static_cast<Tirex2Engine*>(engine);
  if (slot < 0 || slot >= static_cast<int>(e->devs.size())) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  if (!out) return fail(JC_ERR_INVALID_ARG, "null output");
  jc_status st = check_batch(*e, batch, false);
  if (st != JC_OK) return st;
  std::lock_guard<std::mutex> lk(e->mu);
  std::string err;
  st = run_shard(*e, *e->devs[slot], batch, 0, batch->rows, out, false, static_cast<cudaStream_t>(stream), &err);
  return st == JC_OK ? JC_OK : fail(st, err);
}

}  // extern "C"

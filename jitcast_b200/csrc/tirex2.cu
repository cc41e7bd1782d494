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
#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>

#include "engine.h"
#include "kernels.cuh"
#include "opstore.cuh"
#include "ptx.cuh"
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

constexpr int kMlT = 64;          // query and key tokens per block
constexpr int kMlThreads = 256;   // 16 × 16: ty owns 4 query tokens, tx 4 keys (q·k) or 8 value dims (C·v)
constexpr int kMlPitch = kMlT + 4;  // q, k and C row pitch in floats: 16-byte rows, conflict-free 128-bit reads

// Dynamic shared memory of the mLSTM kernel for a sequence of S tokens.
size_t mlstm_smem(int S) {
  return sizeof(float) * (3 * kMlT * kMlPitch + kMlT * kDv) + sizeof(double) * (2 * S + 2 * kMlT);
}

// Starts the asynchronous copy of a 64-token × W-float slab of proj (token rows t0.., zeros past S) into
// shared memory with row pitch P.
template <int W, int P>
__device__ __forceinline__ void mlstm_stage(float* dst, const float* __restrict__ src, long long ldp, int t0, int S) {
  constexpr int V = W / 4, N = kMlT * V / kMlThreads;
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const int i = threadIdx.x + k * kMlThreads, t = i / V, c = i % V;
    const bool in = t0 + t < S;
    cp_async16(dst + t * P + 4 * c, in ? src + (t0 + t) * ldp + 4 * c : src, in ? 16 : 0);
  }
}

// The stabilised parallel mLSTM of one (row, head, 64-query block) (Cells.mlstmCore, Cells.java:74-118)
// with Cells.mlstm's per-head LayerNorm and σ(o) gate (:58-69) as its epilogue. proj [(r·S + t), ldp]
// (ldp a multiple of 4, 16-byte aligned) holds q (heads·64) | k (heads·64) | v (heads·128) | o (heads·128) |
// i (heads) | f (heads).
//   F[t] = Σ_{u≤t} logσ(cap(f_u)),  a[s] = cap(i_s) − F[s],  M[t] = max(0, max_{s≤t} a[s]),  m[t] = F[t] + M[t]
//   C[t,s] = (q_t·k_s)/8 · exp(a[s] − M[t])   (= exp(F[t] − F[s] + i_s − m[t]), s ≤ t)
//   h_t = Σ_s C[t,s] v_s / (max(|Σ_s C[t,s]|, exp(−m[t])) + eps)
// The gate transcendentals run one token per thread while q, k and v copy in; warp 0 then scans them
// (double, 32 tokens per step with a carry). Keys stream through shared memory 64 at a time, so any S fits. Both products are register-tiled from 16-byte shared-memory reads: q·k as
// 4 tokens × 4 keys per thread, C·v as 4 tokens × 8 value dims, the latter stopping at the warp's last
// token on the diagonal block.
__global__ void __launch_bounds__(kMlThreads, 2) mlstm_kernel(const float* __restrict__ proj, long long ldp, int rows,
                                                              int S, int heads, const float* __restrict__ norm_w,
                                                              int out_kind, void* out_hi, void* out_lo, long long ld_out) {
  extern __shared__ __align__(16) uint8_t sm_raw[];
  float* qs = reinterpret_cast<float*>(sm_raw);  // [64 t][68]
  float* ks = qs + kMlT * kMlPitch;             // [64 s][68]
  float* cs = ks + kMlT * kMlPitch;             // [64 s][68]: C transposed (key-major)
  float* vs = cs + kMlT * kMlPitch;             // [64 s][128]
  double* aa = reinterpret_cast<double*>(vs + kMlT * kDv);  // [S]: cap(i_s), then a[s]
  double* lf = aa + S;                                       // [S]: logσ(cap(f_s))
  double* fq = lf + S;                                       // [64]: F[t] of the query block
  double* mq = fq + kMlT;                                    // [64]: M[t] of the query block
  const int r = blockIdx.x / heads, head = blockIdx.x % heads;
  const int qb = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ty = tid >> 4, tx = tid & 15;
  if (r >= rows) return;
  const float* base = proj + static_cast<long long>(r) * S * ldp;
  const int k_off = heads * kDqk, v_off = 2 * heads * kDqk, o_off = v_off + heads * kDv, i_off = o_off + heads * kDv,
            f_off = i_off + heads;
  const int q0 = qb * kMlT;
  const int t_end = min(S, q0 + kMlT);  // the gates of every key this query block reads
  // q and the first key block's k, v in flight while the gates are computed; the epilogue's o rows
  // (64 tokens × 512 bytes, one 128-byte line per thread) are pulled into L2
  mlstm_stage<kDqk, kMlPitch>(qs, base + head * kDqk, ldp, q0, S);
  mlstm_stage<kDqk, kMlPitch>(ks, base + k_off + head * kDqk, ldp, 0, S);
  mlstm_stage<kDv, kDv>(vs, base + v_off + head * kDv, ldp, 0, S);
  cp_async_commit();
  if (q0 + (tid >> 2) < S) prefetch_l2(base + (q0 + (tid >> 2)) * ldp + o_off + head * kDv + 32 * (tid & 3));
  for (int s = tid; s < t_end; s += kMlThreads) {
    const float* ps = base + s * ldp;
    lf[s] = log_sigmoid_d(static_cast<double>(soft_cap(ps[f_off + head])));
    aa[s] = static_cast<double>(soft_cap(ps[i_off + head]));
  }
  __syncthreads();
  // F and the prefix max of a, 32 tokens per step with a carry
  if (warp == 0) {
    double carry_f = 0.0, carry_m = -INFINITY;
    for (int c0 = 0; c0 < t_end; c0 += 32) {
      const int s = c0 + lane;
      double F = s < t_end ? lf[s] : 0.0;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, F, off);
        if (lane >= off) F += y;
      }
      F += carry_f;
      carry_f = __shfl_sync(0xffffffffu, F, 31);
      const double a = s < t_end ? aa[s] - F : -INFINITY;
      double M = a;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, M, off);
        if (lane >= off) M = fmax(M, y);
      }
      M = fmax(M, carry_m);
      carry_m = __shfl_sync(0xffffffffu, M, 31);
      if (s < t_end) {
        aa[s] = a;
        if (s >= q0) {
          fq[s - q0] = F;
          mq[s - q0] = fmax(0.0, M);
        }
      }
    }
  }
  cp_async_wait_all();
  const float scale = 0.125f;  // 1/√64
  float num[4][8], den[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    den[a] = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) num[a][e] = 0.0f;
  }
  __syncthreads();
  for (int kb = 0; kb <= qb; ++kb) {
    if (kb > 0) {
      __syncthreads();  // the previous key block's k, v and C are consumed
      mlstm_stage<kDqk, kMlPitch>(ks, base + k_off + head * kDqk, ldp, kb * kMlT, S);
      mlstm_stage<kDv, kDv>(vs, base + v_off + head * kDv, ldp, kb * kMlT, S);
      cp_async_commit();
      cp_async_wait_all();
      __syncthreads();
    }
    // C[t, s] for tokens 4ty + a and keys tx + 16b
    {
      float c[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) c[a][b] = 0.0f;
#pragma unroll 4
      for (int j = 0; j < kDqk; j += 4) {
        float4 q4[4], k4[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) q4[a] = *reinterpret_cast<const float4*>(qs + (4 * ty + a) * kMlPitch + j);
#pragma unroll
        for (int b = 0; b < 4; ++b) k4[b] = *reinterpret_cast<const float4*>(ks + (tx + 16 * b) * kMlPitch + j);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            c[a][b] = fmaf(q4[a].x, k4[b].x, c[a][b]);
            c[a][b] = fmaf(q4[a].y, k4[b].y, c[a][b]);
            c[a][b] = fmaf(q4[a].z, k4[b].z, c[a][b]);
            c[a][b] = fmaf(q4[a].w, k4[b].w, c[a][b]);
          }
      }
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int sg = kb * kMlT + tx + 16 * b;
        float w[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const int tg = q0 + 4 * ty + a;
          w[a] = tg < S && sg <= tg ? c[a][b] * scale * expf(static_cast<float>(aa[sg] - mq[4 * ty + a])) : 0.0f;
          den[a] += w[a];
        }
        *reinterpret_cast<float4*>(cs + (tx + 16 * b) * kMlPitch + 4 * ty) = make_float4(w[0], w[1], w[2], w[3]);
      }
    }
    __syncthreads();
    // num[t, :] += Σ_s C[t, s] v[s, :] over dims 4tx.. and 64 + 4tx.. (C is zero past each token)
    const int smax = kb == qb ? min(kMlT - 1, 8 * warp + 7) : kMlT - 1;
    for (int s = 0; s <= smax; ++s) {
      const float4 cc = *reinterpret_cast<const float4*>(cs + s * kMlPitch + 4 * ty);
      const float4 v0 = *reinterpret_cast<const float4*>(vs + s * kDv + 4 * tx);
      const float4 v1 = *reinterpret_cast<const float4*>(vs + s * kDv + 64 + 4 * tx);
      const float cv[4] = {cc.x, cc.y, cc.z, cc.w};
      const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 8; ++e) num[a][e] = fmaf(cv[a], vv[e], num[a][e]);
    }
  }
  // epilogue per token: normaliser, LayerNorm over the head's 128 dims (16 lanes × 8), σ(o) gate
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int tl = 4 * ty + a, tg = q0 + tl;
    float dn = den[a];
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) dn += __shfl_xor_sync(0xffffffffu, dn, off);
    const double mt = tg < S ? fq[tl] + mq[tl] : 0.0;
    const float rnorm =
        1.0f / static_cast<float>(fmax(fabs(static_cast<double>(dn)), exp(-mt)) + static_cast<double>(kMlstmEps));
    float mean = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      num[a][e] *= rnorm;
      mean += num[a][e];
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) mean += __shfl_xor_sync(0xffffffffu, mean, off);
    mean *= 1.0f / kDv;
    float var = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float dv = num[a][e] - mean;
      var = fmaf(dv, dv, var);
    }
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) var += __shfl_xor_sync(0xffffffffu, var, off);
    var *= 1.0f / kDv;
    const float inv = rsqrtf(var + kNormEps);
    if (tg >= S) continue;
    const float* og = base + tg * ldp + o_off + head * kDv;
    const long long orow = (static_cast<long long>(r) * S + tg) * ld_out + head * kDv;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int j0 = 64 * h + 4 * tx;
      const float4 o4 = __ldg(reinterpret_cast<const float4*>(og + j0));
      const float4 w4 = __ldg(reinterpret_cast<const float4*>(norm_w + head * kDv + j0));
      const float ov[4] = {o4.x, o4.y, o4.z, o4.w}, wv[4] = {w4.x, w4.y, w4.z, w4.w};
      float r4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float v = (num[a][4 * h + e] - mean) * inv * wv[e];
        const float g = 1.0f / (1.0f + expf(-ov[e]));
        r4[e] = g * v;
      }
      put_op4(out_kind, out_hi, out_lo, orow + j0, make_float4(r4[0], r4[1], r4[2], r4[3]));
    }
  }
}

constexpr int kSlRows = 64;            // rows per cluster: the MMA's N
constexpr int kSlCta = 4;              // CTAs per cluster, each owning 32 of the head's 128 cell dims
constexpr int kSlE = kDh / kSlCta;     // cell dims per CTA
constexpr int kSlThreads = 512;      // 16 warps: warp w moves TMEM lane quarter w % 4, rows 16·(w / 4) ..
constexpr int kSlM = 4 * kSlE;         // gate columns per CTA (4 gates × 32 dims): the MMA's M
// TMEM columns: R hi [0, 64) and R lo·2^11 [64, 128) as FP16 pairs (two K elements per 32-bit column),
// the main accumulator D1 [128, 192) and the correction accumulator D2 [192, 256)
constexpr uint32_t kSlTmemCols = 256;
constexpr int kSlYPitch = kSlE + 4;
constexpr float kSlLoScale = 2048.0f;  // 2^11: lo parts scaled into FP16's normal range
// shared memory (bytes from a 1024-aligned base): y(t-1) as the MMA's B operand in FP16 hi and lo·2^11
// parts ([64 rows × 128] K-major, 128-byte swizzle), two inboxes the cluster's y(t) lands in, the raw
// gates [4][64][32], this CTA's y(t) [64][36], the wx of the next two steps [2][64][128], mbarriers and
// the TMEM address
constexpr int kSlBHi = 0;
constexpr int kSlBLo = kSlBHi + kSlRows * kDh * 2;
constexpr int kSlInbox = kSlBLo + kSlRows * kDh * 2;
constexpr int kSlRaw = kSlInbox + 2 * kSlRows * kDh * 4;
constexpr int kSlYs = kSlRaw + 4 * kSlRows * kSlE * 4;
constexpr int kSlWx = kSlYs + kSlRows * kSlYPitch * 4;  // wx slices of the next two steps [2][64][128]
constexpr int kSlBar = kSlWx + 2 * kSlRows * kSlM * 4;
constexpr int kSlSmem = kSlBar + 64 + 1024;
constexpr uint32_t kSlInBytes = kSlCta * kSlRows * kSlE * 4;  // one step's y of the whole cluster
// A step's waits take microseconds; one that has not completed after 50 ms gives up (and flags the error),
// so even a broken exchange ends a launch in seconds.
constexpr uint64_t kSlWaitNs = 50000000ull;

// Dynamic shared memory of the sLSTM kernel.
size_t slstm_smem() { return kSlSmem; }

// Byte offset of element (n, k) (k a multiple of 8) in a [64 × 128] FP16 K-major operand stored with the
// 128-byte swizzle: 64-element K blocks of 64 rows × 128 bytes, 8-row groups 1024 bytes apart, the 16-byte
// chunks of row n permuted by XOR with n mod 8.
__device__ __forceinline__ uint32_t sl_sw128(int n, int k) {
  return static_cast<uint32_t>((k >> 6) * (kSlRows * 128) + (n >> 3) * 1024 + (n & 7) * 128 +
                               ((((k & 63) >> 3) ^ (n & 7)) << 4));
}

// x split as hi + lo·2^-11 with hi and lo FP16: hi = fp16(x), lo = fp16((x − hi)·2^11). The products of
// two such splits, hi·hi + 2^-11(hi·lo + lo·hi), carry 22-bit operands like a three-pass TF32 split.
__device__ __forceinline__ void sl_split(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn((x - __half2float(hi)) * kSlLoScale);
}
__device__ __forceinline__ uint32_t sl_pack(__half a, __half b) {
  return static_cast<uint32_t>(__half_as_ushort(a)) | (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
}
// The same split of two values with packed conversions; a in the low halves.
__device__ __forceinline__ void sl_split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(a, b);
  const float2 hf = __half22float2(h);
  const __half2 l = __floats2half2_rn((a - hf.x) * kSlLoScale, (b - hf.y) * kSlLoScale);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// LayerNorm over the head's 128 dims of one y row (Cells.slstm :139-140), out (+)= LN(y)·w; one warp, lane
// holding dims 4·lane .. 4·lane + 3. `prev` is out's current value (read only when accumulating).
__device__ __forceinline__ float4 sl_layernorm(float4 v4, float4 w4, float4 prev, int accumulate) {
  float mean = v4.x + v4.y + v4.z + v4.w;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mean += __shfl_xor_sync(0xffffffffu, mean, o);
  mean *= 1.0f / kDh;
  float var = 0.0f;
  var = fmaf(v4.x - mean, v4.x - mean, var);
  var = fmaf(v4.y - mean, v4.y - mean, var);
  var = fmaf(v4.z - mean, v4.z - mean, var);
  var = fmaf(v4.w - mean, v4.w - mean, var);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  var *= 1.0f / kDh;
  const float inv = rsqrtf(var + kNormEps);
  float4 v;
  v.x = (v4.x - mean) * inv * w4.x;
  v.y = (v4.y - mean) * inv * w4.y;
  v.z = (v4.z - mean) * inv * w4.z;
  v.w = (v4.w - mean) * inv * w4.w;
  if (accumulate) {
    v.x += prev.x;
    v.y += prev.y;
    v.z += prev.z;
    v.w += prev.w;
  }
  return v;
}

// The sLSTM recurrence (Cells.slstmRecurrence, Cells.java:170-218) as a per-step GEMM on the tensor cores.
// A cluster of 4 CTAs takes 64 rows and one head; CTA q owns cell dims 32q .. 32q + 31, i.e. 128 of the
// head's 512 gate columns. Per step, raw[m][n] = wx + b + Σ_p R[p][m]·y(t-1)[n][p] is a tcgen05 MMA
// chain (M = 128 gate columns, N = 64 rows, K = 128) over FP16 splits of both operands: D1 = wx + b +
// R_hi·y_hi and D2 = R_hi·y_lo + R_lo·y_hi (lo parts scaled by 2^11), raw = D1 + 2^-11·D2, which keeps
// 22-bit operands (FP32-grade products) in 24 MMAs of K = 16. R^T stays resident in tensor memory as the
// A operand. The gate update follows on the CUDA cores (gate order i, f, z, o),
// and each CTA's y(t) quarter is stored into every CTA's inbox with st.async, completing on the
// receiver's mbarrier. While step t's MMAs run, each CTA applies the per-head LayerNorm (Cells.slstm
// :139-140) to its 16 rows of y(t-1) straight from the inbox. wx [(r·S + t), ldwx] holds the headwise
// gate pre-activations at columns head·512 + g·128 + e; R [H, 128, 4, 128], bias [H, 4, 128];
// out (+)= LN(y)·w at columns head·128 + e.
__global__ void __launch_bounds__(kSlThreads, 1) slstm_kernel(const float* __restrict__ wx, long long ldwx, int rows,
                                                              int S, const float* __restrict__ R,
                                                              const float* __restrict__ bias,
                                                              const float* __restrict__ norm_w, float* out,
                                                              long long ld_out, int accumulate, uint32_t* err) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = sm_raw + (((smem_u32(sm_raw) + 1023u) & ~1023u) - smem_u32(sm_raw));
  float* bhi = reinterpret_cast<float*>(sm + kSlBHi);
  float* blo = reinterpret_cast<float*>(sm + kSlBLo);
  float* inbox = reinterpret_cast<float*>(sm + kSlInbox);  // [2][64][128]
  float* raw = reinterpret_cast<float*>(sm + kSlRaw);      // [4][64][32]
  float* ys = reinterpret_cast<float*>(sm + kSlYs);        // [64][36]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kSlBar);  // [2]: the cluster's y landed in inbox b
  uint64_t* mma_bar = full + 2;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  const uint32_t q = cluster_ctarank();
  const int head = blockIdx.y;
  const int r0 = (blockIdx.x / kSlCta) * kSlRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, rq = warp >> 2;  // the TMEM lane quarter (= gate) and row quarter this warp moves
  const int e = kSlE * static_cast<int>(q) + lane;

  for (int i = tid; i < 2 * kSlRows * kDh / 4; i += kSlThreads)  // y(-1) = 0 in both B parts
    reinterpret_cast<float4*>(bhi)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  if (warp == 0) {
    tmem_alloc(tslot, kSlTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(mma_bar, 1);
    fence_mbar_init();
    mbar_arrive_expect_tx(&full[0], kSlInBytes);              // y(0)
    if (S >= 2) mbar_arrive_expect_tx(&full[1], kSlInBytes);  // y(1)
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t tlane = static_cast<uint32_t>(32 * sp) << 16;
  // R^T of this CTA's gate columns into TMEM lanes 32g + e' (g = sp), K = p along the columns, two FP16
  // K elements per column (the lower K in the low half)
  if (rq == 0) {
    const float* rp = R + static_cast<long long>(head) * kDh * 4 * kDh + sp * kDh + e;
    for (int k0 = 0; k0 < kDh; k0 += 32) {
      uint32_t hi[16], lo[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        __half h0, l0, h1, l1;
        sl_split(__ldg(rp + static_cast<long long>(k0 + 2 * i) * 4 * kDh), h0, l0);
        sl_split(__ldg(rp + static_cast<long long>(k0 + 2 * i + 1) * 4 * kDh), h1, l1);
        hi[i] = sl_pack(h0, h1);
        lo[i] = sl_pack(l0, l1);
      }
      tmem_st_32x32b_x16(tmem + tlane + k0 / 2, hi);
      tmem_st_32x32b_x16(tmem + tlane + 64 + k0 / 2, lo);
    }
    tmem_st_wait();
  }
  const float bcol = __ldg(bias + head * 4 * kDh + sp * kDh + e);
  // wx of a step: this CTA's 128 gate columns (4 gates × 32 dims) of the cluster's 64 rows, copied
  // asynchronously into shared memory two steps ahead (8 × 16 bytes per thread); every step commits one
  // cp.async group (empty past the last step), so waiting for all but the newest group means step t+1's
  // slice has landed
  auto wxs = [&](int t) { return reinterpret_cast<float*>(sm + kSlWx) + (t & 1) * kSlRows * kSlM; };
  auto stage_wx = [&](int t) {
#pragma unroll
    for (int j = 0; j < kSlRows * kSlM / 4 / kSlThreads; ++j) {
      if (t >= S) break;
      const int cidx = tid + j * kSlThreads, nn = cidx >> 5, c4 = cidx & 31, g = c4 >> 3, e4 = c4 & 7;
      const int row = r0 + nn;
      const float* src = wx + (static_cast<long long>(row < rows ? row : 0) * S + t) * ldwx + head * 4 * kDh +
                         g * kDh + kSlE * static_cast<int>(q) + 4 * e4;
      cp_async16(wxs(t) + nn * kSlM + 4 * c4, src, row < rows ? 16 : 0);
    }
    cp_async_commit();
  };
  stage_wx(0);
  stage_wx(1);
  // LayerNorm rows of this CTA: 16q + (warp - 1) + 15j (j < 2, below 16) on warps 1-15, so that warp 0,
  // whose lane 0 issues the MMAs, has none; out's previous value is fetched a step ahead
  const float4 w4 = __ldg(reinterpret_cast<const float4*>(norm_w + head * kDh + 4 * lane));
  float4 prev[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
  auto lrow = [&](int j) { return warp - 1 + 15 * j; };  // within the cluster's 64 rows: + 16q
  auto has_row = [&](int j) { return warp > 0 && lrow(j) < 16 && r0 + 16 * static_cast<int>(q) + lrow(j) < rows; };
  auto out_at = [&](int j, int t) {
    return out + (static_cast<long long>(r0 + 16 * static_cast<int>(q) + lrow(j)) * S + t) * ld_out + head * kDh +
           4 * lane;
  };
  auto load_prev = [&](int t) {
#pragma unroll
    for (int j = 0; j < 2; ++j)
      if (accumulate && has_row(j)) prev[j] = *reinterpret_cast<const float4*>(out_at(j, t));
  };
  auto layernorm = [&](int t) {  // y(t), complete in inbox t & 1
    const float* ib = inbox + (t & 1) * kSlRows * kDh + 16 * static_cast<int>(q) * kDh;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (warp == 0 || lrow(j) >= 16) break;  // warp-uniform
      const float4 v4 = *reinterpret_cast<const float4*>(ib + lrow(j) * kDh + 4 * lane);
      const float4 o = sl_layernorm(v4, w4, prev[j], accumulate);
      if (has_row(j)) *reinterpret_cast<float4*>(out_at(j, t)) = o;
    }
  };
  load_prev(0);
  float c[4], n[4], m[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = n[i] = m[i] = 0.0f;
  bool ok = true;
  cp_async_wait_all();
  cluster_sync();  // every CTA's barriers set before any st.async reaches them; wx(0) staged
  const uint32_t idesc = idesc_f32acc(0, kSlM, kSlRows);  // FP16 A and B
  for (int t = 0; t < S; ++t) {
    if (t > 0) {
      // y(t-1) of the whole cluster → the B operand, split into FP16 hi and lo·2^11 parts
      const int b = (t - 1) & 1;
      if (!mbar_wait(&full[b], ((t - 1) >> 1) & 1, kSlWaitNs)) ok = false;
      if (tid == 0 && t + 1 < S) mbar_arrive_expect_tx(&full[b], kSlInBytes);  // y(t+1) lands in inbox b
      const float* ib = inbox + b * kSlRows * kDh;
#pragma unroll
      for (int j = 0; j < kSlRows * kDh / 8 / kSlThreads; ++j) {
        const int cidx = tid + j * kSlThreads, nn = cidx >> 4, k = 8 * (cidx & 15);
        const float4 v0 = *reinterpret_cast<const float4*>(ib + nn * kDh + k);
        const float4 v1 = *reinterpret_cast<const float4*>(ib + nn * kDh + k + 4);
        const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        uint32_t h[4], l[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) sl_split2(x[2 * u], x[2 * u + 1], h[u], l[u]);
        const uint32_t off = sl_sw128(nn, k);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bhi) + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(blo) + off) = make_uint4(l[0], l[1], l[2], l[3]);
      }
      fence_proxy_async_smem();
    }
    {  // main accumulator = wx(t) + b for this warp's (gate columns, rows)
      uint32_t d[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) d[i] = __float_as_uint(wxs(t)[(16 * rq + i) * kSlM + 32 * sp + lane] + bcol);
      tmem_st_32x32b_x16(tmem + tlane + 128 + 16 * rq, d);
      tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      // D1 += R_hi·y_hi; D2 = R_hi·y_lo + R_lo·y_hi (K = 16 per MMA: 8 TMEM columns of A, 32 bytes of B)
#pragma unroll
      for (int pass = 0; pass < 3; ++pass) {
        const uint32_t a = tmem + (pass == 2 ? 64u : 0u);
        const uint32_t bb = smem_u32(pass == 1 ? blo : bhi);
        const uint32_t d = tmem + (pass == 0 ? 128u : 192u);
#pragma unroll
        for (int k = 0; k < kDh / 16; ++k)
          umma_f16_ts(d, a + 8 * k, sdesc_k_sw128(bb + (k >> 2) * (kSlRows * 128) + (k & 3) * 32), idesc,
                      pass == 1 && k == 0 ? 0u : 1u);
      }
      umma_commit(mma_bar);
    }
    // while the MMAs run: the next step's wx and the LayerNorm of y(t-1)
    stage_wx(t + 2);  // into the slice read before the barrier above
    if (t > 0) {
      layernorm(t - 1);
      load_prev(t);
    }
    if (!mbar_wait(mma_bar, t & 1, kSlWaitNs)) ok = false;
    tc_fence_after();
    {  // raw gates out of TMEM: gate sp of cell dim e for rows 16·rq .. 16·rq + 15, D1 + 2^-11·D2
      uint32_t v[16], w[16];
      tmem_ld_32x32b_x16(tmem + tlane + 128 + 16 * rq, v);
      tmem_ld_32x32b_x16(tmem + tlane + 192 + 16 * rq, w);
      tmem_ld_wait();
      float* rg = raw + sp * kSlRows * kSlE;
#pragma unroll
      for (int i = 0; i < 16; ++i)
        rg[(16 * rq + i) * kSlE + lane] = fmaf(__uint_as_float(w[i]), 1.0f / kSlLoScale, __uint_as_float(v[i]));
    }
    __syncthreads();
    // gate update of cell dim e for rows warp + 16i; the exponentials of the bounded terms and the
    // divisions by n ≥ 1 use the fast intrinsics (errors of a few ulp, below the split products')
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = warp + 16 * i;
      const float ir = raw[(0 * kSlRows + rl) * kSlE + lane], fr = raw[(1 * kSlRows + rl) * kSlE + lane],
                  zr = raw[(2 * kSlRows + rl) * kSlE + lane], orw = raw[(3 * kSlRows + rl) * kSlE + lane];
      const float logf_ = (fminf(fr, 0.0f) - __logf(1.0f + __expf(-fabsf(fr)))) + m[i];
      const float mn = t == 0 ? ir : fmaxf(ir, logf_);
      const float ig = __expf(ir - mn), fg = __expf(logf_ - mn);
      // tanh(z) = sign(z)·(1 − 2/(e^{2|z|} + 1)) on the fast exponential (absolute error ~1e-7)
      const float th = copysignf(1.0f - __fdividef(2.0f, __expf(2.0f * fabsf(zr)) + 1.0f), zr);
      c[i] = fg * c[i] + ig * th;
      n[i] = fmaxf(fg * n[i] + ig, 1.0f);
      m[i] = mn;
      ys[rl * kSlYPitch + lane] = __fdividef(__fdividef(c[i], n[i]), 1.0f + __expf(-orw));
    }
    cp_async_wait_group<1>();  // wx(t + 1) staged by every thread once past the barrier
    __syncthreads();
    // y(t) quarter → every CTA's inbox (t & 1)
#pragma unroll
    for (int j = 0; j < kSlRows * kSlE / 4 / kSlThreads; ++j) {
      const int cidx = tid + j * kSlThreads, nn = cidx >> 3, k = 4 * (cidx & 7);
      const float4 v = *reinterpret_cast<const float4*>(ys + nn * kSlYPitch + k);
      float* dst = inbox + (t & 1) * kSlRows * kDh + nn * kDh + kSlE * static_cast<int>(q) + k;
#pragma unroll
      for (uint32_t p = 0; p < kSlCta; ++p)
        st_async_v4(mapa_shared(smem_u32(dst), p), v, mapa_shared(smem_u32(&full[t & 1]), p));
    }
  }
  // the last step's y: wait for it and normalise it
  if (!mbar_wait(&full[(S - 1) & 1], ((S - 1) >> 1) & 1, kSlWaitNs)) ok = false;
  layernorm(S - 1);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kSlTmemCols);
  if (!ok && tid == 0) atomicOr(err, kErrTimeoutPeer);
  cluster_sync();  // no st.async in flight into any CTA of the cluster
}

constexpr int kMtThreads = 256;        // 8 warps: warp w moves TMEM lane quarter w % 4 and column half w / 4
constexpr uint32_t kMtTmemCols = 256;  // S, then O: main [0, 128) and correction [128, 256)
// shared memory (bytes from a 1024-aligned base): Q hi | Q lo | K hi | K lo ([128 rows × 64] FP16 K-major with
// the 128-byte swizzle, 16 KB each), overlaid after the q·kᵀ MMA by C hi | C lo ([128 × 128 keys], two
// 64-key atoms, 32 KB each); Vᵀ hi | Vᵀ lo ([128 dims × 128 keys], 32 KB each), which first holds the fp32
// q|k rows as copied ([128][128], 512-byte pitch); the fp32 v rows as copied, later the o rows ([128][128],
// 528-byte pitch so a warp reading one 16-byte chunk of 32 rows hits distinct banks); the gate arrays, the
// row-half partial sums, mbarrier, TMEM address
constexpr int kMtQ = 0, kMtK = 32768, kMtC = 0, kMtV = 65536, kMtQKs = 65536, kMtVs = 131072;
constexpr int kMtVPitch = 528;
constexpr int kMtGate = kMtVs + 128 * kMtVPitch;
constexpr int kMtRed = kMtGate + 3 * 128 * 8 + 8 * 8;
constexpr int kMtSmem = kMtRed + 2 * 2 * 128 * 4 + 64 + 1024;

// Byte offset of element (r, c) in a [rows × 64] 16-bit K-major tile with the 128-byte swizzle (1024-aligned).
__device__ __forceinline__ uint32_t mt_sw(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((((c >> 3) ^ r) & 7) << 4) + ((c & 7) << 1));
}

// The mLSTM core with its per-head LayerNorm and σ(o) gate (Cells.mlstmCore :74-118, Cells.mlstm :58-69) on the
// tensor cores, for sequences of at most 64 tokens. A CTA stacks two (row, head) pairs into the 128 rows of
// a tcgen05 tile: S = q·kᵀ (M 128 × N 128 × K 64; the two off-diagonal 64 × 64 blocks are discarded) and
// O = C·v (M 128 × N 128 × K 128, C zero outside the pair's block) run over FP16 splits of both operands —
// x = hi + 2^-11·lo, main = hi·hi, correction = hi·lo + lo·hi, result = main + 2^-11·correction — which
// keeps 22-bit operands (FP32-grade products). Each C row is scaled by a power of two before its split so
// small decay weights keep their bits. The gates (log-sigmoid, prefix sums, the stabiliser) stay in double,
// as the reference. q, k, v and o arrive by cp.async; every stacked row is worked by two threads (TMEM column
// halves) that exchange partial sums through shared memory. proj [(r·S + t), ldp] (16-byte aligned rows)
// holds q (heads·64) | k | v (heads·128) | o (heads·128) | i (heads) | f (heads).
__global__ void __launch_bounds__(kMtThreads, 1) mlstm_tc_kernel(const float* __restrict__ proj, long long ldp,
                                                                 int rows, int S, int heads,
                                                                 const float* __restrict__ norm_w, int out_kind,
                                                                 void* out_hi, void* out_lo, long long ld_out,
                                                                 uint32_t* err) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = sm_raw + (((smem_u32(sm_raw) + 1023u) & ~1023u) - smem_u32(sm_raw));
  double* aa = reinterpret_cast<double*>(sm + kMtGate);  // [128]: a[s] of the stacked keys
  double* fq = aa + 128;                                  // [128]: F[t]
  double* mq = fq + 128;                                  // [128]: M[t]
  double* wt = mq + 128;                                  // [8]: per-warp totals of the scans
  float* red = reinterpret_cast<float*>(sm + kMtRed);     // [2 stats][2 halves][128 rows]
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(red + 2 * 2 * 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ch = warp >> 2;                 // column half of this thread's TMEM row
  const int row = 32 * (warp & 3) + lane;   // stacked row = TMEM lane this thread reads
  const int pr = row >> 6, t = row & 63;    // pair of the CTA, token
  const int npairs = rows * heads;
  int prow[2], phead[2];
  bool pval[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int pair = 2 * blockIdx.x + p;
    pval[p] = pair < npairs;
    prow[p] = pval[p] ? pair / heads : 0;
    phead[p] = pval[p] ? pair % heads : 0;
  }
  const bool live = pval[pr] && t < S;
  const int head = phead[pr];
  const float* base = proj + (static_cast<long long>(prow[pr]) * S + (live ? t : 0)) * ldp;
  const int k_off = heads * kDqk, v_off = 2 * heads * kDqk, o_off = v_off + heads * kDv, i_off = o_off + heads * kDv,
            f_off = i_off + heads;
  // the proj row of stacked row rr and whether it is a real token
  auto row_base = [&](int rr, bool& ok, int& hd) {
    const int pp = rr >> 6, tt = rr & 63;
    ok = pval[pp] && tt < S;
    hd = phead[pp];
    return proj + (static_cast<long long>(prow[pp]) * S + (ok ? tt : 0)) * ldp;
  };
  if (warp == 0) {
    tmem_alloc(tslot, kMtTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(mma_bar, 1);
    fence_mbar_init();
  }
  // q|k and v copied asynchronously (16 bytes per copy, zeros past the sequence): q|k rows into the Vᵀ region, v
  // rows into their own buffer, 16 + 16 copies per thread
  {
    uint8_t* qks = sm + kMtQKs;
    uint8_t* vs = sm + kMtVs;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      const int cidx = tid + kMtThreads * j, rr = cidx >> 5, c = cidx & 31;  // stacked row, 16-byte chunk
      bool ok;
      int hd;
      const float* rb = row_base(rr, ok, hd);
      const float* src = c < 16 ? rb + hd * kDqk + 4 * c : rb + k_off + hd * kDqk + 4 * (c - 16);
      cp_async16(qks + rr * 512 + 16 * c, src, ok ? 16 : 0);
    }
    cp_async_commit();
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      const int cidx = tid + kMtThreads * j, rr = cidx >> 5, c = cidx & 31;
      bool ok;
      int hd;
      const float* rb = row_base(rr, ok, hd);
      cp_async16(vs + rr * kMtVPitch + 16 * c, rb + v_off + hd * kDv + 4 * c, ok ? 16 : 0);
    }
    cp_async_commit();
  }
  // gates of this row's token (double, as the reference), on the first column half; F = prefix sum of the
  // log-sigmoid forget gates and M = max(0, prefix max of a = cap(i) − F) per pair: each warp scans 32 tokens,
  // the pair's second warp adds the first's totals
  double lf = 0.0, ai = 0.0;
  if (ch == 0 && live) {
    lf = log_sigmoid_d(static_cast<double>(soft_cap(base[f_off + head])));
    ai = static_cast<double>(soft_cap(base[i_off + head]));
  }
  double F = lf;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, F, off);
    if (lane >= off) F += y;
  }
  if (lane == 31) wt[warp] = F;
  __syncthreads();
  if (warp & 1) F += wt[warp - 1];
  const double a = live ? ai - F : -INFINITY;
  double M = a;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, M, off);
    if (lane >= off) M = fmax(M, y);
  }
  __syncthreads();  // wt read above before it is reused
  if (lane == 31) wt[warp] = M;
  __syncthreads();
  if (warp & 1) M = fmax(M, wt[warp - 1]);
  if (ch == 0) {
    aa[row] = a;
    fq[row] = F;
    mq[row] = fmax(0.0, M);
  }
  cp_async_wait_group<1>();  // this thread's q|k copies
  __syncthreads();
  // q|k rows → FP16 split tiles: a warp per row, lane l holding 4 consecutive floats (q for l < 16, k after)
  {
    const int hk = lane >> 4, c4 = lane & 15;
    uint8_t* th = sm + (hk ? kMtK : kMtQ);
    uint8_t* tl = th + 16384;
#pragma unroll 4
    for (int rr = warp; rr < 128; rr += kMtThreads / 32) {
      const float4 v = *reinterpret_cast<const float4*>(sm + kMtQKs + rr * 512 + 16 * lane);
      uint32_t h0, l0, h1, l1;
      sl_split2(v.x, v.y, h0, l0);
      sl_split2(v.z, v.w, h1, l1);
      const uint32_t off = mt_sw(rr, 4 * c4);
      *reinterpret_cast<uint2*>(th + off) = make_uint2(h0, h1);
      *reinterpret_cast<uint2*>(tl + off) = make_uint2(l0, l1);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  const uint32_t idesc = idesc_f32acc(0, 128, 128);  // FP16 A and B, M 128, N 128
  bool ok = true;
  if (tid == 0) {
    const uint32_t qa = smem_u32(sm + kMtQ), ka = smem_u32(sm + kMtK);
#pragma unroll
    for (int pass = 0; pass < 3; ++pass) {
      const uint32_t aop = qa + (pass == 2 ? 16384u : 0u), bop = ka + (pass == 1 ? 16384u : 0u);
#pragma unroll
      for (int k = 0; k < kDqk / 16; ++k)
        umma_bf16(tmem + (pass == 0 ? 0u : 128u), sdesc_k_sw128(aop + 32 * k), sdesc_k_sw128(bop + 32 * k), idesc,
                  pass == 2 || k > 0 ? 1u : 0u);
    }
    umma_commit(mma_bar);
  }
  // v rows → Vᵀ split tiles while the MMA runs: thread = (stacked key tid % 128, dim half tid / 128), reading
  // 16 bytes of its row per step and writing 4 dims of its key column of atom key / 64
  cp_async_wait_group<0>();
  __syncthreads();
  {
    const int key = tid & 127, dh = tid >> 7;
    uint8_t* vh = sm + kMtV + (key >> 6) * 16384;
    uint8_t* vl = sm + kMtV + 32768 + (key >> 6) * 16384;
    const uint8_t* vr = sm + kMtVs + key * kMtVPitch + 256 * dh;
#pragma unroll 4
    for (int d4 = 0; d4 < 16; ++d4) {
      const float4 v = *reinterpret_cast<const float4*>(vr + 16 * d4);
      const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half h, l;
        sl_split(x[j], h, l);
        const int d = 64 * dh + 4 * d4 + j;
        *reinterpret_cast<__half*>(vh + mt_sw(d, key & 63)) = h;
        *reinterpret_cast<__half*>(vl + mt_sw(d, key & 63)) = l;
      }
    }
  }
  __syncthreads();  // the v buffer is read; the o rows go there
  {
    uint8_t* os = sm + kMtVs;
#pragma unroll 4
    for (int j = 0; j < 16; ++j) {
      const int cidx = tid + kMtThreads * j, rr = cidx >> 5, c = cidx & 31;
      bool okr;
      int hd;
      const float* rb = row_base(rr, okr, hd);
      cp_async16(os + rr * kMtVPitch + 16 * c, rb + o_off + hd * kDv + 4 * c, okr ? 16 : 0);
    }
    cp_async_commit();
  }
  if (!mbar_wait(mma_bar, 0)) ok = false;
  tc_fence_after();
  // C row half: C[t, s] = (q_t·k_s)/8 · exp(a[s] − M[t]) for keys s = 32·ch + j ≤ t of this pair; the row is
  // scaled by 2^e so its largest magnitude lies in [512, 1024) before the FP16 split (C hi/lo overlay Q and K,
  // which the MMA above has read)
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16);
  const double Mt = live ? mq[row] : 0.0;
  const double mt = live ? fq[row] + Mt : 0.0;
  float cv[32];
  float den = 0.0f, cmax = 0.0f;
  {
    uint32_t sv[32], sc[32];
    tmem_ld_32x32b_x32(lane_base + pr * 64 + 32 * ch, sv);
    tmem_ld_32x32b_x32(lane_base + 128 + pr * 64 + 32 * ch, sc);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int s_ = 32 * ch + j;
      float c = 0.0f;
      if (live && s_ <= t) {
        const float dot = fmaf(__uint_as_float(sc[j]), 1.0f / kSlLoScale, __uint_as_float(sv[j]));
        c = dot * 0.125f * expf(static_cast<float>(aa[pr * 64 + s_] - Mt));
      }
      cv[j] = c;
      den += c;
      cmax = fmaxf(cmax, fabsf(c));
    }
  }
  red[(0 * 2 + ch) * 128 + row] = den;
  red[(1 * 2 + ch) * 128 + row] = cmax;
  __syncthreads();
  den = red[(0 * 2 + 0) * 128 + row] + red[(0 * 2 + 1) * 128 + row];
  cmax = fmaxf(red[(1 * 2 + 0) * 128 + row], red[(1 * 2 + 1) * 128 + row]);
  int ex = 0;
  frexpf(cmax, &ex);
  const float cscale = ldexpf(1.0f, 10 - ex);  // exact; cmax·cscale in [512, 1024)
  {
    uint8_t* chh = sm + kMtC + pr * 16384;
    uint8_t* chl = sm + kMtC + 32768 + pr * 16384;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint32_t h[4], l[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sl_split2(cv[8 * c + 2 * u] * cscale, cv[8 * c + 2 * u + 1] * cscale, h[u], l[u]);
      const uint32_t off = mt_sw(row, 32 * ch + 8 * c);
      *reinterpret_cast<uint4*>(chh + off) = make_uint4(h[0], h[1], h[2], h[3]);
      *reinterpret_cast<uint4*>(chl + off) = make_uint4(l[0], l[1], l[2], l[3]);
      // the other pair's keys: zero
      *reinterpret_cast<uint4*>(sm + kMtC + (1 - pr) * 16384 + off) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(sm + kMtC + 32768 + (1 - pr) * 16384 + off) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) {
    const uint32_t ca = smem_u32(sm + kMtC), va = smem_u32(sm + kMtV);
#pragma unroll
    for (int pass = 0; pass < 3; ++pass) {
      const uint32_t aop = ca + (pass == 2 ? 32768u : 0u), bop = va + (pass == 1 ? 32768u : 0u);
#pragma unroll
      for (int k = 0; k < 128 / 16; ++k)
        umma_bf16(tmem + (pass == 0 ? 0u : 128u), sdesc_k_sw128(aop + (k >> 2) * 16384 + 32 * (k & 3)),
                  sdesc_k_sw128(bop + (k >> 2) * 16384 + 32 * (k & 3)), idesc, pass == 2 || k > 0 ? 1u : 0u);
    }
    umma_commit(mma_bar);
  }
  cp_async_wait_group<0>();  // this thread's o copies
  if (!mbar_wait(mma_bar, 1)) ok = false;
  tc_fence_after();
  __syncthreads();  // every thread's o copies have landed
  // h = O / (2^e · max(|den|, exp(−m)) + eps) over this thread's 64 dims; the head's LayerNorm with mean and
  // variance summed over both halves; then the σ(o) gate
  const float rnorm =
      1.0f / (static_cast<float>(fmax(fabs(static_cast<double>(den)), exp(-mt)) + static_cast<double>(kMlstmEps)) *
              cscale);
  auto chunk = [&](int c, float (&v)[32]) {  // dims 64·ch + 32·c ..
    uint32_t mv[32], cr[32];
    tmem_ld_32x32b_x32(lane_base + 64 * ch + 32 * c, mv);
    tmem_ld_32x32b_x32(lane_base + 128 + 64 * ch + 32 * c, cr);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fmaf(__uint_as_float(cr[j]), 1.0f / kSlLoScale, __uint_as_float(mv[j])) * rnorm;
  };
  float part = 0.0f;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    float v[32];
    chunk(c, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) part += v[j];
  }
  red[ch * 128 + row] = part;
  __syncthreads();
  const float mean = (red[row] + red[128 + row]) * (1.0f / kDv);
  part = 0.0f;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    float v[32];
    chunk(c, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) part = fmaf(v[j] - mean, v[j] - mean, part);
  }
  red[256 + ch * 128 + row] = part;
  __syncthreads();
  const float var = (red[256 + row] + red[256 + 128 + row]) * (1.0f / kDv);
  const float inv = rsqrtf(var + kNormEps);
  const long long orow = (static_cast<long long>(prow[pr]) * S + t) * ld_out + head * kDv + 64 * ch;
  const uint8_t* og = sm + kMtVs + row * kMtVPitch + 256 * ch;
#pragma unroll 1
  for (int c = 0; c < 2; ++c) {
    float v[32];
    chunk(c, v);  // warp-collective: every lane runs it, only live rows store
    if (!live) continue;
    const float4* wg = reinterpret_cast<const float4*>(norm_w + head * kDv + 64 * ch + 32 * c);
#pragma unroll
    for (int q4 = 0; q4 < 8; ++q4) {
      const float4 o4 = *reinterpret_cast<const float4*>(og + 128 * c + 16 * q4), w4 = __ldg(wg + q4);
      const float ov[4] = {o4.x, o4.y, o4.z, o4.w}, wv[4] = {w4.x, w4.y, w4.z, w4.w};
      float r4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) r4[e] = __fdividef((v[4 * q4 + e] - mean) * inv * wv[e], 1.0f + __expf(-ov[e]));
      put_op4(out_kind, out_hi, out_lo, orow + 32 * c + 4 * q4, make_float4(r4[0], r4[1], r4[2], r4[3]));
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kMtTmemCols);
  if (!ok && tid == 0) atomicOr(err, kErrTimeoutAcc);
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
  // every row starts as an empty series (nothing observed), in no known or kept list, so rows past a call's own
  // (bucket padding) compute harmlessly and never reach a real row
  if (ok)
    ok = cudaMemset(p->x, 0, sizeof(float) * rows * L) == cudaSuccess &&
         cudaMemset(p->present, 0, sizeof(float) * rows * L) == cudaSuccess;
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
  auto p = e.take_plan_failure() ? nullptr : make_plan(e, rows, nk, nv);
  if (!p && !dv.plans.empty()) {
    cudaStreamSynchronize(dv.stream);
    dv.plans.clear();
    p = e.take_plan_failure() ? nullptr : make_plan(e, rows, nk, nv);
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

// Independent GEMMs as one grouped launch (launch_gemm_group), timed as one launch under `name`.
cudaError_t gemm_group(TxDevice& dv, GemmArgs* g, int count, cudaStream_t s, const char* name) {
  double flops = 0.0;
  for (int i = 0; i < count; ++i) flops += 2.0 * g[i].M * g[i].N * g[i].K;
  dv.prof.begin(s, name, flops);
  cudaError_t r = launch_gemm_group(g, count, s, dv.err);
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
    prof.begin(s, "mlstm", 2.0 * rows * e.H * (0.5 * S * S) * (kDqk + kDv));
    if (S <= kMlT) {  // one 64-token block: the tensor-core kernel, two (row, head) pairs per CTA
      const unsigned blocks = static_cast<unsigned>((static_cast<long long>(rows) * e.H + 1) / 2);
      mlstm_tc_kernel<<<blocks, kMtThreads, kMtSmem, s>>>(p.proj, ldp, rows, S, e.H, B.head_norm, out_of_op(op),
                                                          p.hn.hi, p.hn.lo, p.hn.ld, dv.err);
    } else {
      dim3 grid(rows * e.H, (S + kMlT - 1) / kMlT);
      mlstm_kernel<<<grid, kMlThreads, mlstm_smem(S), s>>>(p.proj, ldp, rows, S, e.H, B.head_norm, out_of_op(op),
                                                           p.hn.hi, p.hn.lo, p.hn.ld);
    }
    prof.end(s);
    JC_TRY(cudaGetLastError());
    g = gemm_args(op, p.hn, T, B.out_proj);
    into_f32(g, dst, d, accumulate);
    JC_TRY(gemm(dv, g, s, "gemm.out_proj"));
  } else {
    // the headwise gate projections (Cells.headwiseGates): one K = 128 GEMM per head, all heads as one grouped
    // launch (kMaxGemmGroup heads at a time)
    const long long ldw = 4LL * d;
    for (int h0 = 0; h0 < e.SH; h0 += kMaxGemmGroup) {
      GemmArgs gh[kMaxGemmGroup];
      const int cnt = e.SH - h0 < kMaxGemmGroup ? e.SH - h0 : kMaxGemmGroup;
      for (int j = 0; j < cnt; ++j) {
        const int h = h0 + j;
        gh[j] = gemm_args(op, cols_of(in, op, static_cast<long long>(h) * kDh), T, B.gates[h]);
        into_f32(gh[j], p.proj + h * 4 * kDh, ldw, false);
      }
      JC_TRY(gemm_group(dv, gh, cnt, s, "gemm.gates"));
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kSlCta * ((rows + kSlRows - 1) / kSlRows), e.SH);
    cfg.blockDim = dim3(kSlThreads);
    cfg.dynamicSmemBytes = slstm_smem();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kSlCta;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    prof.begin(s, "slstm", 2.0 * T * e.SH * kDh * 4 * kDh);
    JC_TRY(cudaLaunchKernelEx(&cfg, slstm_kernel, static_cast<const float*>(p.proj), ldw, rows, S,
                              static_cast<const float*>(B.rec), static_cast<const float*>(B.sbias),
                              static_cast<const float*>(B.group_norm), dst, static_cast<long long>(d),
                              accumulate ? 1 : 0, dv.err));
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
  // input embedding: output(SiLU(hidden(tok))) + residual(tok). The two GEMMs of tok (hidden, and residual
  // stored into h) run as one grouped launch; output then adds into h, the same float sum as the reference's
  GemmArgs ge[2] = {gemm_args(op, p.tok, T, w.in_h), gemm_args(op, p.tok, T, w.in_r)};
  ge[0].ep.act = kActSilu;
  set_out(ge[0].ep, op, p.emb_h);
  into_f32(ge[1], p.h, d, false);
  JC_TRY(gemm_group(dv, ge, 2, s, "gemm.embed"));
  GemmArgs g = gemm_args(op, p.emb_h, T, w.in_o);
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
  // the output embedding: output(SiLU(hidden(xn))) + residual(xn); hidden and residual (stored into y) as one
  // grouped launch, then output adds into y
  const long long qp = static_cast<long long>(e.Q) * P;
  GemmArgs gh[2] = {gemm_args(op, p.xn, T, w.out_h), gemm_args(op, p.xn, T, w.out_r)};
  gh[0].ep.act = kActSilu;
  set_out(gh[0].ep, op, p.oh);
  into_f32(gh[1], p.y, qp, false);
  JC_TRY(gemm_group(dv, gh, 2, s, "gemm.head"));
  g = gemm_args(op, p.oh, T, w.out_o);
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
  if (e.take_slot_failure(dv.slot)) {  // injected (engine option fail_slot), before any device work
    *err = "injected shard failure (engine option fail_slot)";
    return JC_ERR_CUDA;
  }
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
  const int prows = e.buckets ? bucket_rows(rows) : rows;  // the plan's rows ≥ this shard's
  TxPlan* p = get_plan(e, dv, prows, nk, nv, err);
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
    // the mLSTM kernel's gate prefix lives in shared memory
    const size_t smem = mlstm_smem(e->S());
    if (smem > 227 * 1024)
      return fail(JC_ERR_UNSUPPORTED_SHAPE, "sequence of " + std::to_string(e->S()) +
                                                " patches is too long for the mLSTM kernel's shared-memory gate prefix");
    if (cudaFuncSetAttribute(mlstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess ||
        cudaFuncSetAttribute(slstm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(slstm_smem())) != cudaSuccess ||
        cudaFuncSetAttribute(mlstm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMtSmem) != cudaSuccess)
      return fail_cuda(cudaGetLastError(), "mLSTM / sLSTM kernel setup");
    std::string err;
    if (!upload(*e, hw, *dv, &err)) return fail(JC_ERR_OOM, err);
    dv->slot = static_cast<int>(e->devs.size());
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
    if (status[i] != JC_OK) return fail(status[i], "slot " + std::to_string(i) + " (GPU " + std::to_string(e->devs[i]->device) + "): " + errs[i]);
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

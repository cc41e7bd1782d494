// Attention companions of the Timestral forward (no GEMM-shaped work beyond n ≤ a few hundred
// keys per (row, head)): time attention with the BlockLayout masks, variate attention across the
// rows of one series, the sigmoid gate fused into the output, written in the operand format the
// following output-projection GEMM reads.
//
// Semantics: CpuTimestral.timeAttention / variateAttention (timestral/cpu/CpuTimestral.java:191-314)
// and the masks of BlockLayout.timeAllowed / variateAllowed (timestral/BlockLayout.java:209-243);
// the gate att · sigmoid(g) of CpuTimestral.java:156-161.
#include "attention.cuh"
#include "ptx.cuh"

namespace jc {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

__device__ __forceinline__ void put_op(int kind, void* hi, void* lo, long long i, float v) {
  switch (kind) {
    case kOutBF16: static_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v); break;
    case kOutTF32: static_cast<float*>(hi)[i] = round_tf32(v); break;
    case kOutSplit: {
      const float h = round_tf32(v);
      static_cast<float*>(hi)[i] = h;
      static_cast<float*>(lo)[i] = v - h;
      break;
    }
    default: static_cast<float*>(hi)[i] = v; break;
  }
}

// BlockLayout.timeAllowed for row `row`, query q, key k.
__device__ __forceinline__ bool time_allowed(const AttnArgs& a, int row, int q, int k) {
  if (q < a.enc) {
    if (k >= a.enc) return false;
    return k == q || (a.key_valid[(long long)row * a.enc + k] && (k <= q || a.known[row]));
  }
  if (k < a.enc) return k < a.ll && a.key_valid[(long long)row * a.enc + k];
  return k <= q;
}

constexpr int kQ = 128;    // queries per CTA (one per thread)
constexpr int kKeys = 64;  // keys staged per chunk

// One CTA per (row, head, 128-query tile); each thread owns one query and runs an online
// softmax over key chunks staged in shared memory. FP32 arithmetic throughout.
template <typename T, int DH>
__global__ void __launch_bounds__(kQ) time_attention_kernel(AttnArgs a) {
  __shared__ float ks[kKeys][DH + 1];
  __shared__ float vs[kKeys][DH + 1];
  const int tiles = (a.n + kQ - 1) / kQ;
  const int tile = blockIdx.x % tiles;
  const int hh = (blockIdx.x / tiles) % a.heads;
  const int row = blockIdx.x / (tiles * a.heads);
  const int t = tile * kQ + threadIdx.x;
  const bool live = t < a.n;
  const T* qkv = static_cast<const T*>(a.qkv);
  const long long ld = a.ld_qkv;
  float q[DH], acc[DH];
  if (live) {
    const T* qp = qkv + ((long long)row * a.n + t) * ld + hh * DH;
#pragma unroll
    for (int e = 0; e < DH; ++e) q[e] = ld_f(qp + e) * a.scale;
  }
#pragma unroll
  for (int e = 0; e < DH; ++e) acc[e] = 0.0f;
  float m = -INFINITY, l = 0.0f;
  // keys beyond the last query of the tile never matter for causal decoder queries, but
  // encoder/known rows may read forward keys, so every chunk is visited
  for (int k0 = 0; k0 < a.n; k0 += kKeys) {
    const int nk = min(kKeys, a.n - k0);
    __syncthreads();
    for (int i = threadIdx.x; i < nk * DH; i += kQ) {
      const int kk = i / DH, e = i % DH;
      const long long base = ((long long)row * a.n + k0 + kk) * ld + hh * DH + e;
      ks[kk][e] = ld_f(qkv + base + a.d);
      vs[kk][e] = ld_f(qkv + base + 2 * a.d);
    }
    __syncthreads();
    if (!live) continue;
    for (int kk = 0; kk < nk; ++kk) {
      if (!time_allowed(a, row, t, k0 + kk)) continue;
      float s = 0.0f;
#pragma unroll
      for (int e = 0; e < DH; ++e) s += q[e] * ks[kk][e];
      if (s > m) {
        const float corr = __expf(m - s);
        l *= corr;
#pragma unroll
        for (int e = 0; e < DH; ++e) acc[e] *= corr;
        m = s;
      }
      const float p = __expf(s - m);
      l += p;
#pragma unroll
      for (int e = 0; e < DH; ++e) acc[e] += p * vs[kk][e];
    }
  }
  if (!live) return;
  const float inv = 1.0f / l;  // every query attends at least itself
  const long long o = ((long long)row * a.n + t) * a.ld_out + hh * DH;
  const long long go = ((long long)row * a.n + t) * a.ld_gate + hh * DH;
#pragma unroll
  for (int e = 0; e < DH; ++e) {
    float v = acc[e] * inv;
    if (a.gate) v *= a.gate_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.gate)[go + e])
                                 : static_cast<const float*>(a.gate)[go + e];
    put_op(a.out_kind, a.out_hi, a.out_lo, o + e, v);
  }
}

// One thread per (row, slot, head): attention over the rows [group_start, group_end) of the
// row's series at the same token slot (BlockLayout.variateAllowed). Groups are small.
template <typename T, int DH>
__global__ void variate_attention_kernel(AttnArgs a) {
  const long long total = (long long)a.rows * a.n * a.heads;
  const T* qkv = static_cast<const T*>(a.qkv);
  for (long long id = blockIdx.x * (long long)blockDim.x + threadIdx.x; id < total;
       id += (long long)gridDim.x * blockDim.x) {
    const int hh = static_cast<int>(id % a.heads);
    const int t = static_cast<int>((id / a.heads) % a.n);
    const int i = static_cast<int>(id / ((long long)a.heads * a.n));
    const int gs = a.group_start[i], ge = a.group_end[i];
    float q[DH], acc[DH];
    const T* qp = qkv + ((long long)i * a.n + t) * a.ld_qkv + hh * DH;
#pragma unroll
    for (int e = 0; e < DH; ++e) {
      q[e] = ld_f(qp + e) * a.scale;
      acc[e] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    for (int j = gs; j < ge; ++j) {
      bool ok = true;
      if (j != i) {
        if (t < a.enc && !a.key_valid[(long long)j * a.enc + t]) ok = false;
        if (ok && a.covariates) {
          if (a.role[i] != 0 && a.role[j] == 0) ok = false;
          if (a.role[i] == 2 && a.role[j] != 2) ok = false;
        }
      }
      if (!ok) continue;
      const T* kp = qkv + ((long long)j * a.n + t) * a.ld_qkv + a.d + hh * DH;
      const T* vp = kp + a.d;
      float s = 0.0f;
#pragma unroll
      for (int e = 0; e < DH; ++e) s += q[e] * ld_f(kp + e);
      if (s > m) {
        const float corr = __expf(m - s);
        l *= corr;
#pragma unroll
        for (int e = 0; e < DH; ++e) acc[e] *= corr;
        m = s;
      }
      const float p = __expf(s - m);
      l += p;
#pragma unroll
      for (int e = 0; e < DH; ++e) acc[e] += p * ld_f(vp + e);
    }
    const float inv = 1.0f / l;
    const long long o = ((long long)i * a.n + t) * a.ld_out + hh * DH;
    const long long go = ((long long)i * a.n + t) * a.ld_gate + hh * DH;
#pragma unroll
    for (int e = 0; e < DH; ++e) {
      float v = acc[e] * inv;
      if (a.gate) v *= a.gate_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.gate)[go + e])
                                   : static_cast<const float*>(a.gate)[go + e];
      put_op(a.out_kind, a.out_hi, a.out_lo, o + e, v);
    }
  }
}

template <typename T>
cudaError_t launch_time_t(const AttnArgs& a, cudaStream_t s) {
  const int tiles = (a.n + kQ - 1) / kQ;
  const long long blocks = (long long)a.rows * a.heads * tiles;
  if (a.head_dim == 64) {
    time_attention_kernel<T, 64><<<static_cast<unsigned>(blocks), kQ, 0, s>>>(a);
  } else if (a.head_dim == 32) {
    time_attention_kernel<T, 32><<<static_cast<unsigned>(blocks), kQ, 0, s>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_variate_t(const AttnArgs& a, cudaStream_t s) {
  const long long total = (long long)a.rows * a.n * a.heads;
  long long blocks = (total + 127) / 128;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (a.head_dim == 64) {
    variate_attention_kernel<T, 64><<<static_cast<unsigned>(blocks), 128, 0, s>>>(a);
  } else if (a.head_dim == 32) {
    variate_attention_kernel<T, 32><<<static_cast<unsigned>(blocks), 128, 0, s>>>(a);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_time_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.rows <= 0) return cudaSuccess;
  return a.qkv_bf16 ? launch_time_t<__nv_bfloat16>(a, s) : launch_time_t<float>(a, s);
}

cudaError_t launch_variate_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.rows <= 0) return cudaSuccess;
  return a.qkv_bf16 ? launch_variate_t<__nv_bfloat16>(a, s) : launch_variate_t<float>(a, s);
}

}  // namespace jc

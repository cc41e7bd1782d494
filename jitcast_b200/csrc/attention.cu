// Attention companions of the Timestral forward (no GEMM-shaped work beyond n ≤ a few hundred
// keys per (row, head)): time attention with the BlockLayout masks, variate attention across the
// rows of one series, the sigmoid gate fused into the output, written in the operand format the
// following output-projection GEMM reads.
//
// Semantics: CpuTimestral.timeAttention / variateAttention (timestral/cpu/CpuTimestral.java:191-314)
// and the masks of BlockLayout.timeAllowed / variateAllowed (timestral/BlockLayout.java:209-243);
// the gate att · sigmoid(g) of CpuTimestral.java:156-161.
#include <type_traits>

#include "attention.cuh"
#include "mma_sync.cuh"
#include "ptx.cuh"

namespace jc {

namespace {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <>
__device__ __forceinline__ float ld_f<__half>(const __half* p) { return __half2float(*p); }

__device__ __forceinline__ float ld_gate(const AttnArgs& a, long long i) {
  if (a.gate_kind == kOutBF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(a.gate)[i]);
  if (a.gate_kind == kOutF16) return __half2float(static_cast<const __half*>(a.gate)[i]);
  return static_cast<const float*>(a.gate)[i];
}

template <typename T>
__device__ __forceinline__ float2 h2f2(uint32_t u);
template <>
__device__ __forceinline__ float2 h2f2<__half>(uint32_t u) { return __half22float2(*reinterpret_cast<__half2*>(&u)); }
template <>
__device__ __forceinline__ float2 h2f2<__nv_bfloat16>(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
}

template <typename T>
__device__ __forceinline__ uint32_t f22h(float a, float b);
template <>
__device__ __forceinline__ uint32_t f22h<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(fminf(fmaxf(a, -65504.0f), 65504.0f), fminf(fmaxf(b, -65504.0f), 65504.0f));
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t f22h<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void put_op(int kind, void* hi, void* lo, long long i, float v) {
  switch (kind) {
    case kOutBF16: static_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v); break;
    case kOutF16: static_cast<__half*>(hi)[i] = __float2half_rn(fminf(fmaxf(v, -65504.0f), 65504.0f)); break;
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

// BlockLayout.timeAllowed for row `row`, query q, key k (mask mode 0), or key liveness (mode 1,
// Chronos-2's time attention: every live key in both directions).
__device__ __forceinline__ bool time_allowed(const AttnArgs& a, int row, int q, int k) {
  if (a.mask_mode == 1) return a.live[(long long)row * a.n + k] != 0;
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
  // a query with no allowed key gets zeros (the layouts never make one: every Timestral query sees itself,
  // every Chronos-2 row has its live [REG] token)
  const float inv = l > 0.0f ? 1.0f / l : 0.0f;
  const long long o = ((long long)row * a.n + t) * a.ld_out + hh * DH;
  const long long go = ((long long)row * a.n + t) * a.ld_gate + hh * DH;
#pragma unroll
  for (int e = 0; e < DH; ++e) {
    float v = acc[e] * inv;
    if (a.gate) v *= ld_gate(a, go + e);
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
      if (a.mask_mode == 1) {
        ok = a.live[(long long)j * a.n + t] != 0;
      } else if (j != i) {
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
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;  // no live row in the group: zeros
    const long long o = ((long long)i * a.n + t) * a.ld_out + hh * DH;
    const long long go = ((long long)i * a.n + t) * a.ld_gate + hh * DH;
#pragma unroll
    for (int e = 0; e < DH; ++e) {
      float v = acc[e] * inv;
      if (a.gate) v *= ld_gate(a, go + e);
      put_op(a.out_kind, a.out_hi, a.out_lo, o + e, v);
    }
  }
}

// The same attention for 16-bit q/k/v/gate/output, vectorised: DH / 8 threads per (row, slot, head), each
// owning 8 dims read and written as one 16-byte vector, so an item's q, k, v and output rows are single
// coalesced 128-byte (DH 64) segments. Dot products are reduced across the item's threads with shuffles.
template <typename T, int DH>
__global__ void variate_attention_vec_kernel(AttnArgs a) {
  constexpr int TPI = DH / 8;  // threads per item: 8 (DH 64) or 4 (DH 32), a power of two dividing 32
  const long long items = (long long)a.rows * a.n * a.heads;
  const T* qkv = static_cast<const T*>(a.qkv);
  const int sub = threadIdx.x % TPI;
  const long long stride = (long long)gridDim.x * blockDim.x / TPI;
  for (long long id = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / TPI;; id += stride) {
    // the loop bound is per group of TPI lanes; whole warps leave together only at the end, so the
    // shuffles below always have every lane of the warp present
    const bool active = id < items;
    if (!__any_sync(0xffffffffu, active)) break;
    const long long item = active ? id : 0;
    const int hh = static_cast<int>(item % a.heads);
    const int t = static_cast<int>((item / a.heads) % a.n);
    const int i = static_cast<int>(item / ((long long)a.heads * a.n));
    const int gs = active ? a.group_start[i] : 0, ge = active ? a.group_end[i] : 0;
    const long long row_i = (long long)i * a.n + t;
    float q[8], acc[8];
    {
      const uint4 u = *reinterpret_cast<const uint4*>(qkv + row_i * a.ld_qkv + hh * DH + 8 * sub);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 f = h2f2<T>(w[c]);
        q[2 * c] = f.x * a.scale;
        q[2 * c + 1] = f.y * a.scale;
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    float m = -INFINITY, l = 0.0f;
    // every lane of the warp runs the same number of iterations (the longest group among its items)
    int gmax = ge - gs;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) gmax = max(gmax, __shfl_xor_sync(0xffffffffu, gmax, off));
    for (int jj = 0; jj < gmax; ++jj) {
      const int j = gs + jj;
      bool ok = active && j < ge;
      if (ok) {
        if (a.mask_mode == 1) {
          ok = a.live[(long long)j * a.n + t] != 0;
        } else if (j != i) {
          if (t < a.enc && !a.key_valid[(long long)j * a.enc + t]) ok = false;
          if (ok && a.covariates) {
            if (a.role[i] != 0 && a.role[j] == 0) ok = false;
            if (a.role[i] == 2 && a.role[j] != 2) ok = false;
          }
        }
      }
      float kv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, vv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (ok) {
        const T* kp = qkv + ((long long)j * a.n + t) * a.ld_qkv + a.d + hh * DH + 8 * sub;
        const uint4 uk = *reinterpret_cast<const uint4*>(kp);
        const uint4 uv = *reinterpret_cast<const uint4*>(kp + a.d);
        const uint32_t wk[4] = {uk.x, uk.y, uk.z, uk.w}, wv[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 fk = h2f2<T>(wk[c]), fv = h2f2<T>(wv[c]);
          kv[2 * c] = fk.x, kv[2 * c + 1] = fk.y, vv[2 * c] = fv.x, vv[2 * c + 1] = fv.y;
        }
      }
      float sdot = 0.0f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sdot = fmaf(q[e], kv[e], sdot);
#pragma unroll
      for (int off = TPI / 2; off > 0; off >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, off);
      if (!ok) continue;  // lanes of one item agree on ok (same i, j, t)
      if (sdot > m) {
        const float corr = __expf(m - sdot);
        l *= corr;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] *= corr;
        m = sdot;
      }
      const float p = __expf(sdot - m);
      l += p;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(p, vv[e], acc[e]);
    }
    if (!active) continue;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;  // no live row in the group: zeros
    float o[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = acc[e] * inv;
    if (a.gate) {
      const uint4 ug = *reinterpret_cast<const uint4*>(static_cast<const T*>(a.gate) + row_i * a.ld_gate + hh * DH +
                                                       8 * sub);
      const uint32_t wg[4] = {ug.x, ug.y, ug.z, ug.w};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const float2 g = h2f2<T>(wg[c]);
        o[2 * c] *= g.x;
        o[2 * c + 1] *= g.y;
      }
    }
    uint4 out;
    out.x = f22h<T>(o[0], o[1]);
    out.y = f22h<T>(o[2], o[3]);
    out.z = f22h<T>(o[4], o[5]);
    out.w = f22h<T>(o[6], o[7]);
    *reinterpret_cast<uint4*>(static_cast<T*>(a.out_hi) + row_i * a.ld_out + hh * DH + 8 * sub) = out;
  }
}

// ---- tensor-core time attention (16-bit q/k/v) ---------------------------------------------
// One CTA (4 warps) per (row, head). K and V of the row's n tokens are staged in shared memory as
// FP16 (a BF16 input converts exactly within FP16's range, so P·V keeps an 11-bit P in both modes)
// (rows padded to a multiple of 64, 72-element pitch so ldmatrix rows avoid bank conflicts). Each
// warp walks 16-query tiles; per 64-key block it forms S = Q·Kᵀ with mma.sync m16n8k16 (FP32
// accumulate), applies the BlockLayout mask and an online softmax in registers, converts P to the
// A-operand layout in place and accumulates O += P·V. Key blocks no query of the tile may read
// (beyond the last query of an all-encoder tile on a row that is not a known covariate) are skipped.
constexpr int kMmaWarps = 4;
constexpr int kPitch = 72;       // 64 + 8 halves
constexpr int kMaxTokens = 256;  // longer rows use the FP32 kernel

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t to_h2(__nv_bfloat162 v) {
  const float2 f = __bfloat1622float2(v);
  __half2 h = __floats2half2_rn(fminf(fmaxf(f.x, -65504.0f), 65504.0f), fminf(fmaxf(f.y, -65504.0f), 65504.0f));
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t to_h2(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

// Eight 16-bit values (one 16-byte vector) as FP16.
template <typename T>
__device__ __forceinline__ uint4 to_h8(uint4 u) {
  if constexpr (std::is_same<T, __half>::value) {
    return u;
  } else {
    uint4 r;
    r.x = to_h2(*reinterpret_cast<__nv_bfloat162*>(&u.x));
    r.y = to_h2(*reinterpret_cast<__nv_bfloat162*>(&u.y));
    r.z = to_h2(*reinterpret_cast<__nv_bfloat162*>(&u.z));
    r.w = to_h2(*reinterpret_cast<__nv_bfloat162*>(&u.w));
    return r;
  }
}

template <typename T>
__device__ __forceinline__ uint32_t ld_h2(const T* p) {
  if constexpr (std::is_same<T, __half>::value) {
    return *reinterpret_cast<const uint32_t*>(p);
  } else {
    return to_h2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
}

template <typename T>
__global__ void __launch_bounds__(kMmaWarps * 32) time_attention_mma_kernel(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int n = a.n, npad = (n + 63) & ~63;
  __half* ks = reinterpret_cast<__half*>(smem_raw);
  __half* vs = ks + npad * kPitch;
  int* kvalid = reinterpret_cast<int*>(vs + npad * kPitch);  // per key: may encoder queries read it
  const int hh = blockIdx.x % a.heads;
  const int row = blockIdx.x / a.heads;
  const T* qkv = static_cast<const T*>(a.qkv);
  const long long ld = a.ld_qkv;
  // stage K and V (16-byte vectors), zero rows past n
  for (int i = threadIdx.x; i < npad * 8; i += blockDim.x) {
    const int r = i >> 3, c = (i & 7) * 8;
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (r < n) {
      const T* base = qkv + ((long long)row * n + r) * ld + hh * 64 + c;
      kv = to_h8<T>(*reinterpret_cast<const uint4*>(base + a.d));
      vv = to_h8<T>(*reinterpret_cast<const uint4*>(base + 2 * a.d));
    }
    *reinterpret_cast<uint4*>(ks + r * kPitch + c) = kv;
    *reinterpret_cast<uint4*>(vs + r * kPitch + c) = vv;
  }
  for (int k = threadIdx.x; k < npad; k += blockDim.x) {
    if (a.mask_mode == 1)
      kvalid[k] = k < n ? a.live[(long long)row * n + k] : 0;
    else
      kvalid[k] = k < a.enc ? a.key_valid[(long long)row * a.enc + k] : 0;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;  // fragment row group and column pair
  const bool live_mode = a.mask_mode == 1;
  const bool known = !live_mode && a.known[row] != 0;
  const float sl2 = a.scale * 1.4426950408889634f;  // softmax in base 2
  const uint32_t ks_base = smem_u32(ks), vs_base = smem_u32(vs);
  const int qtiles = (n + 15) >> 4;
  for (int qt = warp; qt < qtiles; qt += kMmaWarps) {
    const int q0 = qt * 16;
    // Q fragments for the 4 k-steps of dh = 64, straight from global (rows past n read as 0)
    uint32_t qf[4][4];
    {
      const int ra = q0 + g, rb = q0 + g + 8;
      const T* pa = qkv + ((long long)row * n + ra) * ld + hh * 64;
      const T* pb = qkv + ((long long)row * n + rb) * ld + hh * 64;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int c = kk * 16 + tq * 2;
        qf[kk][0] = ra < n ? ld_h2(pa + c) : 0u;
        qf[kk][1] = rb < n ? ld_h2(pb + c) : 0u;
        qf[kk][2] = ra < n ? ld_h2(pa + c + 8) : 0u;
        qf[kk][3] = rb < n ? ld_h2(pb + c + 8) : 0u;
      }
    }
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.0f, 0.0f};
    // an all-encoder tile on a row that is not a known covariate reads no key past its last query
    int kend = npad;
    if (!live_mode && q0 + 15 < a.enc && !known) kend = min(npad, ((q0 + 15) / 64 + 1) * 64);
    for (int k0 = 0; k0 < kend; k0 += 64) {
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {  // two 8-key n-tiles per ldmatrix.x4
          const int krow = k0 + jp * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int kcol = kk * 16 + ((lane >> 3) & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm_x4(ks_base + (krow * kPitch + kcol) * 2, b0, b1, b2, b3);
          MmaT<__half>::mma(sc[2 * jp], qf[kk], b0, b1);
          MmaT<__half>::mma(sc[2 * jp + 1], qf[kk], b2, b3);
        }
      }
      // mask, scale, online softmax (rows g and g + 8 of the tile)
#pragma unroll
      for (int hr = 0; hr < 2; ++hr) {
        const int q = q0 + g + hr * 8;
        float mx = mrow[hr];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int k = k0 + j * 8 + tq * 2 + c;
            bool ok;
            if (live_mode) {
              ok = kvalid[k] != 0;
            } else if (q < a.enc) {
              ok = k < a.enc && (k == q || (kvalid[k] && (k <= q || known)));
            } else {
              ok = k < a.enc ? (k < a.ll && kvalid[k]) : (k <= q && k < n);
            }
            float v = ok ? sc[j][hr * 2 + c] * sl2 : -INFINITY;
            sc[j][hr * 2 + c] = v;
            mx = fmaxf(mx, v);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float corr = mx == -INFINITY ? 1.0f : ex2(mrow[hr] - mx);
        mrow[hr] = mx;
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float v = sc[j][hr * 2 + c];
            const float p = v == -INFINITY ? 0.0f : ex2(v - mx);
            sc[j][hr * 2 + c] = p;
            sum += p;
          }
        lrow[hr] = lrow[hr] * corr + sum;  // per-thread partial; reduced at the end
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j][hr * 2] *= corr;
          o[j][hr * 2 + 1] *= corr;
        }
      }
      // O += P·V: P's accumulator layout is the A-operand layout of the next MMA
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pf[4];
        pf[0] = MmaT<__half>::pack(sc[2 * kk][0], sc[2 * kk][1]);
        pf[1] = MmaT<__half>::pack(sc[2 * kk][2], sc[2 * kk][3]);
        pf[2] = MmaT<__half>::pack(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
        pf[3] = MmaT<__half>::pack(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {  // two 8-wide dh tiles per ldmatrix.x4.trans
          const int vrow = k0 + kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int vcol = jp * 16 + ((lane >> 4) << 3);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(vs_base + (vrow * kPitch + vcol) * 2, b0, b1, b2, b3);
          MmaT<__half>::mma(o[2 * jp], pf, b0, b1);
          MmaT<__half>::mma(o[2 * jp + 1], pf, b2, b3);
        }
      }
    }
    // finish: full row sums across the quad, normalise, gate, store in the operand format
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float l = lrow[hr];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
      const int q = q0 + g + hr * 8;
      if (q >= n) continue;
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const long long ob = ((long long)row * n + q) * a.ld_out + hh * 64;
      const long long gb = ((long long)row * n + q) * a.ld_gate + hh * 64;
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int e = j * 8 + tq * 2 + c;
          float v = o[j][hr * 2 + c] * inv;
          if (a.gate) v *= ld_gate(a, gb + e);
          put_op(a.out_kind, a.out_hi, a.out_lo, ob + e, v);
        }
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
  if constexpr (!std::is_same<T, float>::value) {
    const bool vec = !a.cuda_cores && a.out_kind == a.qkv_kind && (!a.gate || a.gate_kind == a.qkv_kind) &&
                     (a.head_dim == 64 || a.head_dim == 32) && a.ld_qkv % 8 == 0 && a.d % 8 == 0 &&
                     a.ld_out % 8 == 0 && (!a.gate || a.ld_gate % 8 == 0) &&
                     (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.out_hi) & 15) == 0 &&
                     (!a.gate || (reinterpret_cast<uintptr_t>(a.gate) & 15) == 0);
    if (vec) {
      const long long threads = (long long)a.rows * a.n * a.heads * (a.head_dim / 8);
      long long blocks = (threads + 255) / 256;
      if (blocks > 148 * 16) blocks = 148 * 16;
      if (a.head_dim == 64)
        variate_attention_vec_kernel<T, 64><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
      else
        variate_attention_vec_kernel<T, 32><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a);
      return cudaGetLastError();
    }
  }
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
  if (!a.cuda_cores && time_attention_tc_ok(a)) return launch_time_attention_tc(a, s);
  if (!a.cuda_cores && (a.qkv_kind == kOutBF16 || a.qkv_kind == kOutF16) && a.head_dim == 64 && a.n <= kMaxTokens &&
      a.ld_qkv % 8 == 0 && a.d % 8 == 0) {
    const int npad = (a.n + 63) & ~63;
    const size_t smem = 2 * static_cast<size_t>(npad) * kPitch * 2 + sizeof(int) * npad;
    const unsigned blocks = static_cast<unsigned>(static_cast<long long>(a.rows) * a.heads);
    // the shared-memory limit is raised once per device for the largest row (outside any capture:
    // the first forward of an engine runs eagerly)
    static bool raised[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!raised[dev & 63]) {
      const int most = static_cast<int>(2 * static_cast<size_t>(kMaxTokens) * kPitch * 2 + sizeof(int) * kMaxTokens);
      cudaFuncSetAttribute(time_attention_mma_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
      cudaFuncSetAttribute(time_attention_mma_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
      raised[dev & 63] = true;
    }
    if (a.qkv_kind == kOutBF16) {
      time_attention_mma_kernel<__nv_bfloat16><<<blocks, kMmaWarps * 32, smem, s>>>(a);
    } else {
      time_attention_mma_kernel<__half><<<blocks, kMmaWarps * 32, smem, s>>>(a);
    }
    return cudaGetLastError();
  }
  if (a.qkv_kind == kOutBF16) return launch_time_t<__nv_bfloat16>(a, s);
  if (a.qkv_kind == kOutF16) return launch_time_t<__half>(a, s);
  return launch_time_t<float>(a, s);
}

cudaError_t launch_variate_attention(const AttnArgs& a, cudaStream_t s) {
  if (a.rows <= 0) return cudaSuccess;
  if (a.qkv_kind == kOutBF16) return launch_variate_t<__nv_bfloat16>(a, s);
  if (a.qkv_kind == kOutF16) return launch_variate_t<__half>(a, s);
  return launch_variate_t<float>(a, s);
}

}  // namespace jc

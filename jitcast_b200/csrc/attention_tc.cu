// Time attention on the 5th-generation tensor cores (16-bit q/k/v, 64-wide heads, n ≤ 256 tokens).
//
// One CTA of 4 warps per (row, head). TMA brings the head's Q (the first 128 tokens) and K and V (the
// row's tokens, rounded up to 16) into 128-byte-swizzled shared memory; one thread issues
//
//   S[128 × nk] = Q · Kᵀ            tcgen05.mma kind::f16, A and B K-major, accumulator in TMEM
//   O[128 × 64] = P · V              A = P (K-major, written by the softmax), B = V read MN-major,
//                                    both FP16 (a BF16 V is converted in shared memory)
//
// and each thread owns one query row in between: it reads its row of S from TMEM twice (row max, then
// exp2), applies the row's mask, and writes P as 16-bit values straight into the swizzled A-operand
// layout. The row sums come from the tensor cores too (P times a 16-column tile of ones, beside the O MMA).
// The epilogue reads its row of O and its row sum from TMEM, divides by the sum,
// multiplies the gate (Timestral) and stores 16-byte vectors. Queries past the first 128 (the decoder
// tokens of a Timestral row, the [REG] and future tokens of a Chronos-2 row) run 8 at a time on the
// warp-level tensor cores (mma.sync) from the same shared-memory K and V, each warp a quarter of the keys.
//
// Masks: BlockLayout.timeAllowed (timestral/BlockLayout.java:209-221; mask mode 0) or per-key
// liveness in both directions (Chronos-2 ModelLayout; mask mode 1). Semantics: CpuTimestral.java:191-262
// and CpuChronos2.timeAttention; softmax(scale · q·k) over the allowed keys, times the gate if any.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "attention.cuh"
#include "mma_sync.cuh"
#include "ptx.cuh"

namespace jc {

namespace {

constexpr int kTcThreads = 128;
constexpr int kTcQ = 128;        // queries per MMA tile (TMEM lanes)
constexpr int kTcMaxTokens = 256;
constexpr int kTcExtraKeys = 8;  // keys past a 128-key S MMA the main rows may score on the CUDA cores

struct TcShape {
  int nkl;        // K/V rows staged (round_up(n, 16))
  int nkm;        // keys in the S = Q·Kᵀ MMA (multiple of 16, ≤ nkl)
  int nx;         // live keys past the MMA's 128 (mode 1, at most kTcExtraKeys): CUDA-core scores and P·V
  int o_col;      // first TMEM column of O
  int tmem_cols;  // TMEM columns allocated (power of two)
  int k_off, v_off, p_off, bar_off, ones_off;  // byte offsets into the 1024-aligned dynamic shared memory
};

__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __half>::value) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  if constexpr (std::is_same<T, __half>::value) {
    return __half22float2(*reinterpret_cast<__half2*>(&u));
  } else {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&u));
  }
}

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Byte offset of element (r, c), c < 64, of a 16-bit tile of 128-byte rows stored with the 128-byte
// swizzle (the layout TMA writes and the UMMA descriptors read; the tile is 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((((c >> 3) ^ r) & 7) << 4) + ((c & 7) << 1));
}

// Bits of the keys in [lo, hi) that fall in 32-key word w.
__device__ __forceinline__ uint32_t range_bits(int w, int lo, int hi) {
  const int a = max(lo - 32 * w, 0), b = min(hi - 32 * w, 32);
  if (a >= b) return 0u;
  return static_cast<uint32_t>((1ull << b) - 1ull) & ~static_cast<uint32_t>((1ull << a) - 1ull);
}

// Word w of the keys query q may read: BlockLayout.timeAllowed (mode 0) or the live keys (mode 1);
// `bits` holds the row's key_valid (mode 0, keys < enc) or live (mode 1, keys < n) flags.
__device__ __forceinline__ uint32_t allowed_word(const AttnArgs& a, const uint32_t* bits, bool known, int q, int w) {
  const uint32_t f = bits[w];
  if (a.mask_mode == 1) return f;
  if (q < a.enc) return (known ? f : (f & range_bits(w, 0, q + 1))) | range_bits(w, q, q + 1);
  return (f & range_bits(w, 0, a.ll)) | range_bits(w, a.enc, min(q, a.n - 1) + 1);
}

constexpr int kTailQ = 8;  // queries past the MMA tile handled per round
constexpr int kTailPitch = 68;  // floats per query row of the partial P·V scratch (64 + 4: no bank conflicts)

// Lane (g, t) = (lane / 4, lane % 4) of a warp's m16n8k16 tile: rows 0..7 are a round's queries (rows 8..15
// zero); the lane holds query g's A fragments (dims 16k + 2t, +1 and 16k + 8 + 2t, +1 of k-step k), its keys
// 8j + 2t, +1 of each 8-key n-tile of S and its output dims 8j + 2t, +1.
template <typename T>
__device__ __forceinline__ void tail_q(const AttnArgs& a, long long row0, int hh, int t0, int nt, int lane,
                                       uint32_t (&qa)[4][2]) {
  const int g = lane >> 2, t = lane & 3;
  const bool live = g < nt;
  const uint32_t* qr = reinterpret_cast<const uint32_t*>(static_cast<const T*>(a.qkv) +
                                                         (row0 + t0 + (live ? g : 0)) * a.ld_qkv + hh * 64);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    qa[k][0] = live ? __ldg(qr + 8 * k + t) : 0u;
    qa[k][1] = live ? __ldg(qr + 8 * k + 4 + t) : 0u;
  }
}

// The gate values thread tid applies in a tail round (query tid / 16, dims 4·(tid % 16) .. + 3), loaded before the
// round so that their latency is not on its path; zeros where the thread has no query or there is no gate.
template <typename T>
__device__ __forceinline__ uint2 tail_gate(const AttnArgs& a, long long row0, int hh, int t0, int nt, int tid) {
  const int qg = tid >> 4, d4 = 4 * (tid & 15);
  if (!a.gate || qg >= nt) return make_uint2(0u, 0u);
  return __ldg(reinterpret_cast<const uint2*>(static_cast<const T*>(a.gate) + (row0 + t0 + qg) * a.ld_gate + hh * 64 + d4));
}

// One round of up to kTailQ queries past the MMA tile (tokens t0 .. t0 + nt), on the four warps' warp-level tensor
// cores (mma.sync m16n8k16, FP32 accumulation): warp w owns the 16-key steps w, w + 4, .. of the row's keys. It
// forms S = q·Kᵀ for them (B = the K tile by ldmatrix), applies the mask and publishes its per-query max; after a
// barrier each warp takes the row max, forms P = 2^(S − max) as FP16 A fragments, publishes its partial sum and
// its partial O = P·V (B = the FP16 V tile by ldmatrix.trans); after a second barrier a thread per (query, 4 dims)
// adds the four partials, divides by the row sum, multiplies the gate (`tg`, from tail_gate before the round) and
// stores. Keys the query may not read get
// probability 0; the K/V rows staged past the row's n tokens hold finite values (the next row's tokens or TMA's
// zero fill), so they add nothing. The caller orders the scratch against later writes to Q's tile.
template <typename T>
__device__ __forceinline__ void tail_round(const AttnArgs& a, const TcShape& sh, const uint32_t* bits, bool known,
                                           const uint8_t* ks, const uint8_t* vs, long long row0, int hh, int t0,
                                           int nt, float sl2, int warp, int lane, int tid, const uint32_t (&qa)[4][2],
                                           uint2 tg, float* tmax, float* tsum, float* tpart) {
  constexpr int KW = kTcMaxTokens / 64;  // k-steps per warp at most
  const int g = lane >> 2, t = lane & 3;
  const bool live = g < nt;
  const int tok = t0 + g;
  const uint32_t ks_a = smem_u32(ks), vs_a = smem_u32(vs);
  const int steps = sh.nkl / 16;
  float s[KW][4];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < KW; ++i) {
    s[i][0] = s[i][1] = s[i][2] = s[i][3] = -INFINITY;
    const int kk = warp + 4 * i;
    if (kk >= steps) continue;  // warp-uniform
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // the step's two 8-key n-tiles
      const int key0 = 16 * kk + 8 * h;
      uint32_t b[8];
      const int kr = key0 + (lane & 7);
      ldsm_x4(ks_a + sw128(kr, 8 * (lane >> 3)), b[0], b[1], b[2], b[3]);
      ldsm_x4(ks_a + sw128(kr, 32 + 8 * (lane >> 3)), b[4], b[5], b[6], b[7]);
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t av[4] = {qa[k][0], 0u, qa[k][1], 0u};
        MmaT<T>::mma(c, av, b[2 * k], b[2 * k + 1]);
      }
      const int key = key0 + 2 * t;
      const uint32_t w = live ? allowed_word(a, bits, known, tok, key >> 5) : 0u;
      if ((w >> (key & 31)) & 1u) s[i][2 * h] = c[0] * sl2;
      if ((w >> ((key + 1) & 31)) & 1u) s[i][2 * h + 1] = c[1] * sl2;
    }
    mx = fmax3(mx, fmax3(s[i][0], s[i][1], s[i][2]), s[i][3]);
  }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  if (t == 0) tmax[warp * kTailQ + g] = mx;
  __syncthreads();
  mx = fmaxf(fmaxf(tmax[g], tmax[kTailQ + g]), fmaxf(tmax[2 * kTailQ + g], tmax[3 * kTailQ + g]));
  const float base = mx == -INFINITY ? 0.0f : mx;
  float l = 0.0f;
  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
#pragma unroll
  for (int i = 0; i < KW; ++i) {
    const int kk = warp + 4 * i;
    if (kk >= steps) continue;  // warp-uniform
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      p[e] = s[i][e] == -INFINITY ? 0.0f : ex2f(s[i][e] - base);
      l += p[e];
    }
    const uint32_t av[4] = {pack2<__half>(p[0], p[1]), 0u, pack2<__half>(p[2], p[3]), 0u};
    const int vr = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
    for (int d = 0; d < 4; ++d) {  // dims 16d .. 16d + 15: two 8-dim n-tiles
      uint32_t b0, b1, b2, b3;
      ldsm_x4_t(vs_a + sw128(vr, 16 * d + 8 * (lane >> 4)), b0, b1, b2, b3);
      MmaT<__half>::mma(o[2 * d], av, b0, b1);
      MmaT<__half>::mma(o[2 * d + 1], av, b2, b3);
    }
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  if (t == 0) tsum[warp * kTailQ + g] = l;
  float* part = tpart + (warp * kTailQ + g) * kTailPitch;
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<float2*>(part + 8 * j + 2 * t) = make_float2(o[j][0], o[j][1]);
  __syncthreads();
  // a thread per (query, 4 dims): the partials in warp order, 1/l, the gate, one 8-byte store
  const int qg = tid >> 4, d4 = 4 * (tid & 15);
  if (qg < nt) {
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float sum = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(tpart + (w * kTailQ + qg) * kTailPitch + d4);
      acc.x += v.x, acc.y += v.y, acc.z += v.z, acc.w += v.w;
      sum += tsum[w * kTailQ + qg];
    }
    const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
    float x[4] = {acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv};
    const long long tk = row0 + t0 + qg;
    if (a.gate) {
      const float2 g0 = unpack2<T>(tg.x), g1 = unpack2<T>(tg.y);
      x[0] *= g0.x, x[1] *= g0.y, x[2] *= g1.x, x[3] *= g1.y;
    }
    if constexpr (std::is_same<T, __half>::value) {
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = fminf(fmaxf(x[e], -65504.0f), 65504.0f);
    }
    *reinterpret_cast<uint2*>(static_cast<T*>(a.out_hi) + tk * a.ld_out + hh * 64 + d4) =
        make_uint2(pack2<T>(x[0], x[1]), pack2<T>(x[2], x[3]));
  }
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 4) attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                                                                  const __grid_constant__ CUtensorMap tmKV,
                                                                  AttnArgs a, TcShape sh) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* ks = smem + sh.k_off;
  uint8_t* vs = smem + sh.v_off;
  uint8_t* ps = smem + sh.p_off;  // over Q and K when they are large enough (both dead by then)
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + sh.bar_off);  // [0] TMA, [1] S, [2] O
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3);
  uint32_t* abort_flag = tmem_slot + 1;
  uint32_t* bits = tmem_slot + 2;  // [8]: one bit per key
  // tail-round scratch in Q's tile once the S MMA has read it: per warp and query the partial max, sum and P·V
  float* tmax = reinterpret_cast<float*>(qs);         // [4][kTailQ]
  float* tsum = tmax + 4 * kTailQ;                     // [4][kTailQ]
  float* tpart = tsum + 4 * kTailQ;                    // [4][kTailQ][kTailPitch]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hh = blockIdx.x % a.heads;
  const int row = blockIdx.x / a.heads;
  const int n = a.n;
  const bool known = a.mask_mode == 0 && a.known[row] != 0;

  const long long row0 = static_cast<long long>(row) * n;
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    mbar_init(&bars[2], 1);
    *abort_flag = 0;
    fence_mbar_init();
    // the head's Q, K and V in flight from the start, under the TMEM allocation and the key-flag loads
    mbar_arrive_expect_tx(&bars[0], static_cast<uint32_t>(kTcQ * 128 + 2 * sh.nkl * 128));
    tma_load_2d(qs, &tmQ, &bars[0], hh * 64, static_cast<int>(row0));
    tma_load_2d(ks, &tmKV, &bars[0], a.d + hh * 64, static_cast<int>(row0));
    tma_load_2d(vs, &tmKV, &bars[0], 2 * a.d + hh * 64, static_cast<int>(row0));
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(tmem_slot, static_cast<uint32_t>(sh.tmem_cols));
    tmem_relinquish();
    tc_fence_before();
  }
  // the row's key flags as bit words (keys ≥ the flag array's length read as 0)
  for (int k0 = 0; k0 < kTcMaxTokens; k0 += kTcThreads) {
    const int k = k0 + tid;
    int f = 0;
    if (a.mask_mode == 1) {
      f = k < n ? a.live[static_cast<long long>(row) * n + k] : 0;
    } else {
      f = k < a.enc ? a.key_valid[static_cast<long long>(row) * a.enc + k] : 0;
    }
    const uint32_t word = __ballot_sync(0xffffffffu, f != 0);
    if (lane == 0) bits[k >> 5] = word;
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the first tail round's q fragments (queries past the MMA tile), in flight during the TMA wait
  uint32_t tqa[4][2];
  uint2 tg = make_uint2(0u, 0u);
  if (n > kTcQ) {
    tail_q<T>(a, row0, hh, kTcQ, min(kTailQ, n - kTcQ), lane, tqa);
    tg = tail_gate<T>(a, row0, hh, kTcQ, min(kTailQ, n - kTcQ), tid);
  }
  // this thread's gate row on its way into L2 for the epilogue
  if (a.gate && tid < n) prefetch_l2(static_cast<const T*>(a.gate) + (row0 + tid) * a.ld_gate + hh * 64);
  // this thread's query and its allowed keys as bit words
  const int q = tid;
  const bool my_row = q < n;
  if (!mbar_wait(&bars[0], 0)) atomicOr(abort_flag, 1u);
  __syncthreads();
  const bool ok = *abort_flag == 0;
  const uint32_t fmt = std::is_same<T, __half>::value ? 0u : 1u;
  if (ok && tid == 0) {
    tc_fence_after();
    const uint32_t idesc = idesc_f32acc(fmt, kTcQ, static_cast<uint32_t>(sh.nkm));
    const uint32_t qa = smem_u32(qs), ka = smem_u32(ks);
#pragma unroll
    for (int k = 0; k < 4; ++k) umma_bf16(tmem, sdesc_k_sw128(qa + 32 * k), sdesc_k_sw128(ka + 32 * k), idesc, k > 0);
    umma_commit(&bars[1]);
  }

  // P·V runs in FP16 in both modes (an 11-bit P): a BF16 V tile is converted in place, saturating at
  // ±65504, while the S MMA reads Q and K
  if (ok && !std::is_same<T, __half>::value) {
    uint4* v4 = reinterpret_cast<uint4*>(vs);
    for (int i = tid; i < sh.nkl * 8; i += kTcThreads) {
      uint4 u = v4[i];
      u.x = pack2<__half>(fminf(fmaxf(unpack2<__nv_bfloat16>(u.x).x, -65504.0f), 65504.0f),
                          fminf(fmaxf(unpack2<__nv_bfloat16>(u.x).y, -65504.0f), 65504.0f));
      u.y = pack2<__half>(fminf(fmaxf(unpack2<__nv_bfloat16>(u.y).x, -65504.0f), 65504.0f),
                          fminf(fmaxf(unpack2<__nv_bfloat16>(u.y).y, -65504.0f), 65504.0f));
      u.z = pack2<__half>(fminf(fmaxf(unpack2<__nv_bfloat16>(u.z).x, -65504.0f), 65504.0f),
                          fminf(fmaxf(unpack2<__nv_bfloat16>(u.z).y, -65504.0f), 65504.0f));
      u.w = pack2<__half>(fminf(fmaxf(unpack2<__nv_bfloat16>(u.w).x, -65504.0f), 65504.0f),
                          fminf(fmaxf(unpack2<__nv_bfloat16>(u.w).y, -65504.0f), 65504.0f));
      v4[i] = u;
    }
    fence_proxy_async_smem();
  }
  // the S MMA must have read Q before its tile holds the tail scratch
  if (ok && !mbar_wait(&bars[1], 0)) atomicOr(abort_flag, 2u);
  __syncthreads();
  tc_fence_after();
  const bool ok1 = *abort_flag == 0;
  const float sl2 = a.scale * 1.4426950408889634f;

  // keys past a 128-key S MMA (Chronos-2's [REG] and future tokens, mode 1): raw scores from this thread's
  // Q row, taken before the tail rounds reuse Q's tile; they join the softmax's max and sum, and their P·V
  // is added on the CUDA cores in the epilogue
  float xs[kTcExtraKeys];  // scores, then probabilities
#pragma unroll
  for (int i = 0; i < kTcExtraKeys; ++i) xs[i] = -INFINITY;
  if (ok1 && sh.nx > 0) {
    float xa[kTcExtraKeys];
#pragma unroll
    for (int i = 0; i < kTcExtraKeys; ++i) xa[i] = 0.0f;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 qu = *reinterpret_cast<const uint4*>(qs + sw128(tid, 8 * c));
      const float2 q0 = unpack2<T>(qu.x), q1 = unpack2<T>(qu.y), q2 = unpack2<T>(qu.z), q3 = unpack2<T>(qu.w);
#pragma unroll
      for (int i = 0; i < kTcExtraKeys; ++i) {
        if (i >= sh.nx) break;
        const uint4 ku = *reinterpret_cast<const uint4*>(ks + sw128(kTcQ + i, 8 * c));
        const float2 k0 = unpack2<T>(ku.x), k1 = unpack2<T>(ku.y), k2 = unpack2<T>(ku.z), k3 = unpack2<T>(ku.w);
        xa[i] = fmaf(q0.x, k0.x, fmaf(q0.y, k0.y, fmaf(q1.x, k1.x, fmaf(q1.y, k1.y, xa[i]))));
        xa[i] = fmaf(q2.x, k2.x, fmaf(q2.y, k2.y, fmaf(q3.x, k3.x, fmaf(q3.y, k3.y, xa[i]))));
      }
    }
    const uint32_t xw = bits[kTcQ / 32];
#pragma unroll
    for (int i = 0; i < kTcExtraKeys; ++i) xs[i] = i < sh.nx && ((xw >> i) & 1u) ? xa[i] : -INFINITY;
  }
  if (sh.nx > 0) __syncthreads();  // every Q row read before the tail rounds overwrite Q's tile

  // queries past the MMA tile, kTailQ per round over all four warps (scratch in Q's tile)
  if (ok1) {
    for (int t0 = kTcQ; t0 < n; t0 += kTailQ) {
      const int nt = min(kTailQ, n - t0);
      if (t0 != kTcQ) {
        tail_q<T>(a, row0, hh, t0, nt, lane, tqa);
        tg = tail_gate<T>(a, row0, hh, t0, nt, tid);
      }
      tail_round<T>(a, sh, bits, known, ks, vs, row0, hh, t0, nt, sl2, warp, lane, tid, tqa, tg, tmax, tsum, tpart);
    }
  }

  // softmax of this thread's row of S into the swizzled FP16 A-operand tile of P. A 32-key chunk no
  // query of the warp may read (past the diagonal of a causal row) is skipped by the whole warp.
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float l = 0.0f;  // the extra keys' share of the row sum; the tile keys' share comes from the row-sum MMA
  if (ok1) {
    float mx = -INFINITY;
#pragma unroll 1  // one copy of each chunk body: the unrolled chunk loops overflowed the instruction cache
    for (int c = 0; c < kTcMaxTokens / 32; ++c) {
      const uint32_t mw = allowed_word(a, bits, known, q, c);
      if (32 * c >= sh.nkm || !__any_sync(0xffffffffu, mw != 0u)) continue;
      uint32_t r[32];
      tmem_ld_32x32b_x32(lane_base + 32 * c, r);
      tmem_ld_wait();
      if (__all_sync(0xffffffffu, mw == ~0u)) {  // every key of the chunk open to every query of the warp
#pragma unroll
        for (int j = 0; j < 32; j += 2) mx = fmax3(mx, __uint_as_float(r[j]), __uint_as_float(r[j + 1]));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if ((mw >> j) & 1u) mx = fmaxf(mx, __uint_as_float(r[j]));
      }
    }
    if (sh.nx > 0) {
#pragma unroll
      for (int i = 0; i < kTcExtraKeys; ++i) mx = fmaxf(mx, xs[i]);
    }
    // the last tail round's reads of its scratch end before P is written over Q's tile
    if (n > kTcQ) __syncthreads();
    const float mo = mx == -INFINITY ? 0.0f : mx * sl2;
    if (sh.nx > 0) {
#pragma unroll
      for (int i = 0; i < kTcExtraKeys; ++i) {
        xs[i] = xs[i] == -INFINITY ? 0.0f : ex2f(fmaf(xs[i], sl2, -mo));
        l += xs[i];
      }
    }
#pragma unroll 1
    for (int c = 0; c < kTcMaxTokens / 32; ++c) {
      if (32 * c >= sh.nkm) continue;
      uint32_t pk[16];
      const uint32_t mw = allowed_word(a, bits, known, q, c);
      if (__any_sync(0xffffffffu, mw != 0u)) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(lane_base + 32 * c, r);
        tmem_ld_wait();
        if (__all_sync(0xffffffffu, mw == ~0u)) {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float p0 = ex2f(fmaf(__uint_as_float(r[j]), sl2, -mo));
            const float p1 = ex2f(fmaf(__uint_as_float(r[j + 1]), sl2, -mo));
            pk[j >> 1] = pack2<__half>(p0, p1);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const float p0 = (mw >> j) & 1u ? ex2f(fmaf(__uint_as_float(r[j]), sl2, -mo)) : 0.0f;
            const float p1 = (mw >> (j + 1)) & 1u ? ex2f(fmaf(__uint_as_float(r[j + 1]), sl2, -mo)) : 0.0f;
            pk[j >> 1] = pack2<__half>(p0, p1);
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) pk[j] = 0u;
      }
      // 32 keys = 4 chunks of 16 bytes within the 64-key swizzle atom c / 2
      uint8_t* atom = ps + (c >> 1) * (kTcQ * 128);
      const int cc = (c & 1) * 4;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(atom + sw128(q, 8 * (cc + u))) =
            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
    }
  }
  // the B operand of the row-sum MMA: 16 rows of FP16 ones (2 KB; every 16-key step reads the same atom)
  reinterpret_cast<uint4*>(smem + sh.ones_off)[tid] = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  const bool ok2 = *abort_flag == 0;
  if (ok2 && tid == 0) {
    tc_fence_after();
    // O into TMEM columns [0, 64) (S is consumed); V read MN-major: instruction descriptor bit 16
    const uint32_t idesc = idesc_f32acc(0u, kTcQ, 64) | (1u << 16);  // FP16 P and V
    const uint32_t pa = smem_u32(ps), va = smem_u32(vs);
    // and the row sums Σ P into TMEM columns [64, 80): P times 16 columns of ones (B K-major), FP32 accumulation
    // of the FP16 P that the O MMA reads
    const uint32_t isum = idesc_f32acc(0u, kTcQ, 16);
    const uint32_t oa = smem_u32(smem + sh.ones_off);
    for (int j = 0; j < sh.nkm / 16; ++j) {
      const uint64_t pd = sdesc_k_sw128(pa + (j >> 2) * (kTcQ * 128) + 32 * (j & 3));
      umma_bf16(tmem, pd, sdesc_k_sw128(va + 2048 * j), idesc, j > 0);
      umma_bf16(tmem + 64, pd, sdesc_k_sw128(oa + 32 * (j & 3)), isum, j > 0);
    }
    umma_commit(&bars[2]);
  }
  // this thread's gate row, fetched while the O MMA runs
  uint4 gate[8];
  if (a.gate && my_row) {
    const uint4* gp = reinterpret_cast<const uint4*>(static_cast<const T*>(a.gate) + (row0 + q) * a.ld_gate + hh * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) gate[i] = __ldg(gp + i);
  }
  if (ok2 && !mbar_wait(&bars[2], 0)) atomicOr(abort_flag, 4u);
  __syncthreads();
  tc_fence_after();
  const bool ok3 = *abort_flag == 0;
  // tcgen05.ld and its wait are warp-collective: every lane runs them, only rows < n store
  if (ok3) {
    l += __uint_as_float(tmem_ld_32x32b_x1(lane_base + 64));
    tmem_ld_wait();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    T* op = static_cast<T*>(a.out_hi) + (row0 + q) * a.ld_out + hh * 64;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t r[32];
      tmem_ld_32x32b_x32(lane_base + static_cast<uint32_t>(32 * half), r);
      tmem_ld_wait();
      if (!my_row) continue;
      if (sh.nx > 0) {  // P·V of the keys past the S MMA, from the (FP16) V tile
#pragma unroll
        for (int i = 0; i < kTcExtraKeys; ++i) {
          if (i >= sh.nx || xs[i] == 0.0f) continue;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 vv = *reinterpret_cast<const uint4*>(vs + sw128(kTcQ + i, 32 * half + 8 * u));
            const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const float2 v2 = unpack2<__half>(vw[w]);
              r[8 * u + 2 * w] = __float_as_uint(fmaf(xs[i], v2.x, __uint_as_float(r[8 * u + 2 * w])));
              r[8 * u + 2 * w + 1] = __float_as_uint(fmaf(xs[i], v2.y, __uint_as_float(r[8 * u + 2 * w + 1])));
            }
          }
        }
      }
      uint32_t pk[16];
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float v0 = __uint_as_float(r[j]) * inv, v1 = __uint_as_float(r[j + 1]) * inv;
        if (a.gate) {
          const float2 g = unpack2<T>(word_of(gate[(16 * half + (j >> 1)) >> 2], (j >> 1) & 3));
          v0 *= g.x;
          v1 *= g.y;
        }
        pk[j >> 1] = pack2<T>(v0, v1);
      }
      uint4* dst = reinterpret_cast<uint4*>(op + 32 * half);
#pragma unroll
      for (int u = 0; u < 4; ++u) dst[u] = make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, static_cast<uint32_t>(sh.tmem_cols));
  if (tid == 0 && *abort_flag != 0 && a.err) atomicOr(a.err, kErrAttnWait);
}

}  // namespace

// Whether the tensor-core kernel takes this attention (16-bit operands of 64-wide heads, ≤ 256 tokens,
// 16-byte aligned rows, 16-bit output).
bool time_attention_tc_ok(const AttnArgs& a) {
  const bool k16 = a.qkv_kind == kOutBF16 || a.qkv_kind == kOutF16;
  return k16 && a.out_kind == a.qkv_kind && (!a.gate || a.gate_kind == a.qkv_kind) && a.head_dim == 64 &&
         a.n >= 1 && a.n <= kTcMaxTokens && a.ld_qkv % 8 == 0 && a.d % 64 == 0 && a.ld_out % 8 == 0 &&
         (!a.gate || a.ld_gate % 8 == 0) && (reinterpret_cast<uintptr_t>(a.qkv) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(a.out_hi) & 15) == 0 && (!a.gate || (reinterpret_cast<uintptr_t>(a.gate) & 15) == 0);
}

cudaError_t launch_time_attention_tc(const AttnArgs& a, cudaStream_t s) {
  TcShape sh{};
  sh.nkl = (a.n + 15) & ~15;
  const int first = a.n < kTcQ ? a.n : kTcQ;
  // encoder queries of mask mode 0 read encoder keys only
  sh.nkm = (a.mask_mode == 0 && a.enc >= first) ? ((a.enc + 15) & ~15) : sh.nkl;
  if (sh.nkm > sh.nkl) sh.nkm = sh.nkl;
  // mode 1 rows a few keys past 128 (Chronos-2: 128 context + [REG] + 4 future tokens): a 128-key S MMA and
  // the rest on the CUDA cores keep TMEM at 128 columns, i.e. four CTAs per SM instead of two
  sh.nx = 0;
  if (a.mask_mode == 1 && a.n > kTcQ && a.n <= kTcQ + kTcExtraKeys) {
    sh.nkm = kTcQ;
    sh.nx = a.n - kTcQ;
  }
  sh.o_col = 0;  // O reuses S's columns once the softmax has read S
  sh.tmem_cols = sh.nkm <= 128 ? 128 : 256;
  sh.k_off = kTcQ * 128;
  sh.v_off = sh.k_off + sh.nkl * 128;
  const int p_bytes = ((sh.nkm + 63) / 64) * kTcQ * 128;
  const int qkv_end = (sh.v_off + sh.nkl * 128 + 1023) & ~1023;
  // P over the Q and K tiles when it fits there (both are dead once the S MMA and the tail queries are
  // done), else after V
  sh.p_off = p_bytes <= sh.v_off ? 0 : qkv_end;
  sh.bar_off = sh.p_off == 0 ? qkv_end : qkv_end + p_bytes;
  sh.ones_off = (sh.bar_off + 3 * 8 + 4 * 10 + 1023) & ~1023;
  int smem = sh.ones_off + 2048 + 1024;
  // never more CTAs on an SM than its 512 TMEM columns hold, so no tcgen05.alloc has to wait: ask for
  // enough shared memory that one more CTA would not fit in the SM's 228 KB (1 KB reserved per CTA)
  const int fit = 512 / sh.tmem_cols;
  const int floor_smem = 233472 / (fit + 1) - 1024 + 16;
  if (smem < floor_smem) smem = floor_smem;
  const int op = a.qkv_kind == kOutBF16 ? kOpBF16 : kOpF16;
  const long long tokens = static_cast<long long>(a.rows) * a.n;
  CUtensorMap mq, mkv;
  if (!make_operand_map(&mq, a.qkv, op, tokens, a.ld_qkv, a.ld_qkv, kTcQ) ||
      !make_operand_map(&mkv, a.qkv, op, tokens, a.ld_qkv, a.ld_qkv, sh.nkl))
    return cudaErrorInvalidValue;
  static bool raised[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!raised[dev & 63]) {
    const int most = 200 * 1024;
    cudaFuncSetAttribute(attention_tc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(attention_tc_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    raised[dev & 63] = true;
  }
  const unsigned blocks = static_cast<unsigned>(static_cast<long long>(a.rows) * a.heads);
  if (a.qkv_kind == kOutBF16)
    attention_tc_kernel<__nv_bfloat16><<<blocks, kTcThreads, smem, s>>>(mq, mkv, a, sh);
  else
    attention_tc_kernel<__half><<<blocks, kTcThreads, smem, s>>>(mq, mkv, a, sh);
  return cudaGetLastError();
}

}  // namespace jc

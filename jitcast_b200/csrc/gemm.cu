// Persistent, warp-specialised tcgen05 GEMM for sm_100a with a fused epilogue.
//
//   C[m, n] (+)= act(rs[m]·(A[m, :]·W[n, :]) + b[n])      A [M, K], W [N, K], both K-major
//
// One CTA per SM walks output tiles of 128 × BN. Warp 0 streams A and W K-slices into a
// ring of shared-memory stages with TMA (128-byte swizzle); warp 1 issues tcgen05.mma into
// one of two TMEM accumulators (128 lanes × BN fp32 columns each); warps 2-5 drain the
// other accumulator with tcgen05.ld and run the epilogue (bias, activation, residual add,
// FP32 store, operand-typed copy for the next GEMM, SwiGLU pairing, RoPE, sigmoid gate)
// straight from registers to HBM, so no separate elementwise kernel touches C.
//
// The semantics follow the reference's shared GEMM kernel (Kernels.gemm, Kernels.java:59-102):
// bias, then SiLU or ReLU, then the accumulate of C; and its CPU operator Ops.linear
// (Ops.java:33-51) for y = x·Wᵀ + b.
#include "gemm.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <type_traits>

namespace jc {

template <int BN_, int OPK_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr int OPK = OPK_;
  static constexpr int BM = 128;
  static constexpr int ESZ = (OPK == kOpBF16 || OPK == kOpF16) ? 2 : 4;
  static constexpr int BK = 128 / ESZ;   // K elements per 128-byte swizzled row
  static constexpr int UK = 32 / ESZ;    // K per tcgen05.mma (32 bytes)
  static constexpr int NSUB = BK / UK;   // MMAs per stage per product
  static constexpr int NOP = OPK == kOpSplit ? 2 : 1;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = NOP * (A_BYTES + B_BYTES);
  static constexpr int STAGES_RAW = (200 * 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  // The split FP32 mode drains every stage's partial product (K = 32) out of TMEM and sums the partials in
  // FP32 with round-to-nearest (a "slab" accumulation): NACC rotating partial buffers plus one sum buffer.
  // The tensor cores' own accumulation truncates, and over a long K that bias grows with the number of
  // accumulate steps; drained per stage it is bounded by 16 steps.
  static constexpr bool SLAB = OPK == kOpSplit;
  static constexpr int NACC = SLAB ? 3 : 2;
  static constexpr int TMEM_COLS = SLAB ? 4 * BN : 2 * BN;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = idesc_f32acc(OPK == kOpBF16 ? 1u : OPK == kOpF16 ? 0u : 2u, BM, BN);
  static_assert(STAGES >= 2, "too few stages");
  static_assert(TMEM_COLS >= 32 && TMEM_COLS <= 512, "TMEM columns");
  static_assert(!SLAB || BN <= 128, "the split mode's slab buffers need BN <= 128");
};

constexpr int kEpiWarps = 8;                    // two warps per TMEM lane quarter, splitting the columns
constexpr int kThreads = 32 * (2 + kEpiWarps);  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue

// ---- epilogue helpers ---------------------------------------------------------------------
// vec_ok levels: 2 = every pointer and pitch 32-byte aligned (256-bit accesses, whole 32-byte
// sectors), 1 = 16-byte aligned, 0 = scalar.

__device__ __forceinline__ void st8_f32(float* p, const float* v) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(v[0]), "f"(v[1]), "f"(v[2]),
               "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

__device__ __forceinline__ void st8_b32(void* p, const uint32_t* u) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(u[0]), "r"(u[1]), "r"(u[2]),
               "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7])
               : "memory");
}

__device__ __forceinline__ void ld8_f32(const float* p, float* v) {
  asm volatile("ld.global.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}

__device__ __forceinline__ void ld8_f32_nc(const float* p, float* v) {
  asm volatile("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
               : "l"(p));
}

// 32 (or nv) fp32 values starting at src: read-only data (bias, tables).
__device__ __forceinline__ void load_ro(const float* src, int nv, int vec, float (&v)[32]) {
  if (nv == 32 && vec == 2) {
#pragma unroll
    for (int q = 0; q < 4; ++q) ld8_f32_nc(src + 8 * q, v + 8 * q);
  } else if (nv == 32 && vec == 1) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + q);
      v[4 * q] = b.x;
      v[4 * q + 1] = b.y;
      v[4 * q + 2] = b.z;
      v[4 * q + 3] = b.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = j < nv ? __ldg(src + j) : 0.0f;
  }
}

__device__ __forceinline__ void add_bias(const EpiParams& p, int col0, int nv, float (&v)[32]) {
  float b[32];
  load_ro(p.bias + col0, nv, p.vec_ok, b);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] += b[j];
}

// Writes 32 (or nv) fp32 values of one row to an fp32 buffer.
__device__ __forceinline__ void store_f32(float* dst, int nv, int vec, const float (&v)[32]) {
  if (nv == 32 && vec == 2) {
#pragma unroll
    for (int q = 0; q < 4; ++q) st8_f32(dst + 8 * q, v + 8 * q);
  } else if (nv == 32 && vec == 1) {
    float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int q = 0; q < 8; ++q) d4[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) dst[j] = v[j];
  }
}

constexpr float kHalfMax = 65504.0f;

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

__device__ __forceinline__ uint32_t pack_f16(float a, float b) {
  __half2 t = __floats2half2_rn(fminf(fmaxf(a, -kHalfMax), kHalfMax), fminf(fmaxf(b, -kHalfMax), kHalfMax));
  return *reinterpret_cast<uint32_t*>(&t);
}

// 32 values as 16-bit (bf16 or saturated f16) to dst.
template <bool F16>
__device__ __forceinline__ void store_16(void* dst, int nv, int vec, const float (&v)[32]) {
  if (nv == 32 && vec >= 1) {
    uint32_t u[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) u[j] = F16 ? pack_f16(v[2 * j], v[2 * j + 1]) : pack_bf16(v[2 * j], v[2 * j + 1]);
    if (vec == 2) {
      st8_b32(dst, u);
      st8_b32(static_cast<uint32_t*>(dst) + 8, u + 8);
    } else {
      uint4* d4 = static_cast<uint4*>(dst);
#pragma unroll
      for (int q = 0; q < 4; ++q) d4[q] = make_uint4(u[4 * q], u[4 * q + 1], u[4 * q + 2], u[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) {
        if (F16)
          static_cast<__half*>(dst)[j] = __float2half_rn(fminf(fmaxf(v[j], -kHalfMax), kHalfMax));
        else
          static_cast<__nv_bfloat16*>(dst)[j] = __float2bfloat16_rn(v[j]);
      }
  }
}

// The operand-typed copy of a row chunk (for the next GEMM's A).
__device__ __forceinline__ void store_operand(const EpiParams& p, long long off, int nv, const float (&v)[32]) {
  const int vec = p.vec_ok;
  switch (p.o_kind) {
    case kOutBF16:
      store_16<false>(static_cast<__nv_bfloat16*>(p.o_hi) + off, nv, vec, v);
      break;
    case kOutF16:
      store_16<true>(static_cast<__half*>(p.o_hi) + off, nv, vec, v);
      break;
    case kOutF32:
      store_f32(static_cast<float*>(p.o_hi) + off, nv, vec, v);
      break;
    case kOutTF32: {
      float t[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) t[j] = round_tf32(v[j]);
      store_f32(static_cast<float*>(p.o_hi) + off, nv, vec, t);
      break;
    }
    case kOutSplit: {
      float hi[32], lo[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        hi[j] = round_tf32(v[j]);
        lo[j] = v[j] - hi[j];
      }
      store_f32(static_cast<float*>(p.o_hi) + off, nv, vec, hi);
      store_f32(static_cast<float*>(p.o_lo) + off, nv, vec, lo);
      break;
    }
    default:
      break;
  }
}

// A folded RMSNorm's scale of GEMM row `row`: 1 / sqrt(Σ_u norm_sq[row · units + u] / d + eps), the partial sums
// added in unit order.
__device__ __forceinline__ float norm_scale(const EpiParams& p, int row) {
  const float* q = p.norm_sq + (long long)row * p.norm_units;
  float ss = 0.0f;
  if ((p.norm_units & 3) == 0) {
    for (int u = 0; u < p.norm_units; u += 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(q + u));
      ss += v.x;
      ss += v.y;
      ss += v.z;
      ss += v.w;
    }
  } else {
    for (int u = 0; u < p.norm_units; ++u) ss += __ldg(q + u);
  }
  return 1.0f / sqrtf(ss * p.norm_inv_d + p.norm_eps);
}

// The folded norm's scale of row row0 + lane (1 for rows ≥ M), for a warp whose lanes own rows row0 .. row0 + 31.
// With a unit count that is a multiple of 4 the warp reads its rows' partial sums as one contiguous block of
// 16-byte vectors (coalesced, instead of a 32-row gather per vector), sums each vector, adds the vectors of a row
// across lanes by shuffles and hands each lane its row's sum. Every epilogue uses it, so their results agree.
__device__ __forceinline__ float norm_scale_warp(const EpiParams& p, int row0, int lane, int M) {
  const int U = p.norm_units, F = U >> 2;  // F: vectors per row
  if ((U & 3) != 0 || (F & (F - 1)) != 0 || F > 32) return row0 + lane < M ? norm_scale(p, row0 + lane) : 1.0f;
  const float4* blk = reinterpret_cast<const float4*>(p.norm_sq + (long long)row0 * U);
  const int per = 32 / F;                        // rows per 32 vectors
  const int valid = max(0, min(32, M - row0)) * F;  // vectors of rows < M
  float mine = 0.0f;
  for (int k = 0; k < F; ++k) {
    const int i = lane + 32 * k;  // vector i: row i / F
    float s = 0.0f;
    if (i < valid) {
      const float4 v = __ldg(blk + i);
      s = ((v.x + v.y) + v.z) + v.w;
    }
    for (int o = 1; o < F; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float t = __shfl_sync(0xffffffffu, s, (lane % per) * F);
    if (lane / per == k) mine = t;
  }
  return row0 + lane < M ? 1.0f / sqrtf(mine * p.norm_inv_d + p.norm_eps) : 1.0f;
}

__device__ __forceinline__ void scale32(float (&v)[32], float s) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] *= s;
}

// Norm scale → bias → activation, for one row's 32-column chunk (rs: the row's norm scale, if the GEMM folds one).
__device__ __forceinline__ void epi_act_chunk(const EpiParams& p, float rs, int col0, int nv, float (&v)[32]) {
  if (p.norm_sq) scale32(v, rs);
  if (p.bias_on) add_bias(p, col0, nv, v);
  switch (p.act) {  // one branch per chunk, not per element
    case kActSilu:
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = silu_f(v[j]);
      break;
    case kActRelu:
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
      break;
    case kActGelu:
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_f(v[j]);
      break;
    case kActSigmoid:
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = sigmoid_f(v[j]);
      break;
    case kActSiluRelu:
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(silu_f(v[j]), 0.0f);
      break;
    default:
      break;
  }
}

// 32 (or nv) fp32 values of a row from src: every pointer and pitch of the epilogue allows `vec` (2: 32-byte, 1:
// 16-byte vectors, 0: scalar).
__device__ __forceinline__ void load_row32(const float* src, int nv, int vec, float (&c)[32]) {
  if (nv == 32 && vec == 2) {
#pragma unroll
    for (int q = 0; q < 4; ++q) ld8_f32(src + 8 * q, c + 8 * q);
  } else if (nv == 32 && vec == 1) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 x = s4[q];
      c[4 * q] = x.x, c[4 * q + 1] = x.y, c[4 * q + 2] = x.z, c[4 * q + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) c[j] = j < nv ? src[j] : 0.0f;
  }
}

// The FP32 store, the operand-typed copy and Σv², for one row's 32-column chunk.
__device__ __forceinline__ void epi_store_chunk(const EpiParams& p, int orow, int col0, int nv, const float (&v)[32],
                                                float& sq) {
  if (p.c) store_f32(p.c + (long long)orow * p.ldc + col0, nv, p.vec_ok, v);
  if (p.o_kind != kOutNone) store_operand(p, (long long)orow * p.ldo + col0, nv, v);
  if (p.rowsq) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nv) sq += v[j] * v[j];
  }
}

// Bias → activation → accumulate → stores, for one row's 32-column chunk.
__device__ __forceinline__ void epi_plain_chunk(const EpiParams& p, float rs, int orow, int col0, int nv,
                                                float (&v)[32], float& sq) {
  epi_act_chunk(p, rs, col0, nv, v);
  if (p.accumulate) {
    float c[32];
    load_row32(p.cin + (long long)orow * p.ldcin + col0, nv, p.vec_ok, c);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] += c[j];
  }
  epi_store_chunk(p, orow, col0, nv, v, sq);
}

// Two 32-column chunks of the thread's accumulator row with a single wait, so their TMEM latencies overlap.
__device__ __forceinline__ void load_chunk_pair(uint32_t ta, uint32_t tb, float (&a)[32], float (&b)[32]) {
  uint32_t ra[32], rb[32];
  tmem_ld_32x32b_x32(ta, ra);
  tmem_ld_32x32b_x32(tb, rb);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    a[j] = __uint_as_float(ra[j]);
    b[j] = __uint_as_float(rb[j]);
  }
}

__device__ __forceinline__ void load_chunk(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld_32x32b_x32(taddr, r);
  tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// The residual epilogue (plain mode, += C) with the residual read early: each thread's residual for the first
// 64-column unit of its row in a tile goes into registers BEFORE the epilogue waits for the tile's accumulator, so
// those reads overlap the tile's MMAs; a later unit's residual is read together with its accumulator chunks,
// instead of after them.
struct ResidualPre {
  float a[32], b[32];  // the thread's row in its first 64-column unit of the tile
};

// The residual-preloading epilogue covers the residual GEMMs (a layer's output projection into the residual
// stream): plain mode, += C into an FP32 C, an optional bias, no activation, no operand-typed copy, no row scale or
// Σv². Their only registers are the accumulator and residual chunks (the 10-warp CTA gives each thread 168).
__host__ __device__ __forceinline__ bool residual_preloaded(const EpiParams& p) {
  return p.mode == kEpiPlain && p.accumulate && p.c && p.act == kActNone && p.o_kind == kOutNone && !p.norm_sq &&
         !p.rowsq;
}

__device__ __forceinline__ int out_row(const EpiParams& p, int row) {
  const int rr = row % p.rg;
  return (row / p.rg) * p.rg_stride + rr + p.rg_off + (rr >= p.rg_split ? p.rg_shift : 0);
}

// The residual of the thread's first unit (columns n0 + 64·half ..), into registers.
__device__ __forceinline__ void residual_preload(const EpiParams& p, int M, int N, int m0, int n0, int row_in_tile,
                                                 int half, ResidualPre& r) {
  const int row = m0 + row_in_tile;
  const int col0 = n0 + 64 * half;
  if (row >= M || col0 >= N) return;
  const float* src = p.cin + (long long)out_row(p, row) * p.ldcin + col0;
  load_row32(src, min(32, N - col0), p.vec_ok, r.a);
  load_row32(src + 32, col0 + 32 < N ? min(32, N - col0 - 32) : 0, p.vec_ok, r.b);
}

// One 32-column chunk of the residual epilogue: + bias, += the residual, the FP32 store.
__device__ __forceinline__ void residual_chunk(const EpiParams& p, int orow, int col0, int nv, float (&v)[32],
                                               const float (&r)[32]) {
  if (p.bias_on) add_bias(p, col0, nv, v);
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] += r[k];
  store_f32(p.c + (long long)orow * p.ldc + col0, nv, p.vec_ok, v);
}

// epilogue_tile for the residual epilogue, a 32-column chunk at a time: the first unit's residual is already in
// registers; each later chunk's residual is read together with its accumulator chunk rather than after it.
template <int BN>
__device__ __forceinline__ void epilogue_tile_residual(const EpiParams& p, int M, int N, int m0, int n0,
                                                       uint32_t tbase, int row_in_tile, int half,
                                                       const ResidualPre& r) {
  const int row = m0 + row_in_tile;
  const bool live = row < M;
  const int orow = live ? out_row(p, row) : 0;
  const int c0 = n0 + 64 * half;
  if (64 * half < BN && c0 < N) {  // warp-uniform
    float v[32];
    load_chunk(tbase + 64 * half, v);
    if (live) residual_chunk(p, orow, c0, min(32, N - c0), v, r.a);
    if (c0 + 32 < N) {
      load_chunk(tbase + 64 * half + 32, v);
      if (live) residual_chunk(p, orow, c0 + 32, min(32, N - c0 - 32), v, r.b);
    }
  }
#pragma unroll 1
  for (int u = half + 2; u < BN / 64; u += 2) {
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int col0 = n0 + 64 * u + 32 * c;
      if (col0 >= N) break;  // warp-uniform
      const int nv = min(32, N - col0);
      float rv[32];
      if (live) load_row32(p.cin + (long long)orow * p.ldcin + col0, nv, p.vec_ok, rv);
      float v[32];
      load_chunk(tbase + 64 * u + 32 * c, v);
      if (live) residual_chunk(p, orow, col0, nv, v, rv);
    }
  }
}

// Pulls what the thread's epilogue of a tile will read from memory into L2 — the residual input (the 128-byte
// lines of its row in the tile's columns it will add) or its row's RoPE table entries — issued before the
// epilogue waits for the tile's accumulator so that those reads overlap the tile's MMAs.
template <int BN>
__device__ __forceinline__ void prefetch_residual(const EpiParams& p, int M, int N, int m0, int n0, int row_in_tile,
                                                  int half) {
  const int row = m0 + row_in_tile;
  if (row >= M) return;
  if (p.mode == kEpiQKV && n0 < p.rope_cols) {
    // the row's RoPE table entries (cos and sin halves), fetched into L2 while the tile's MMAs run
    const float* tc = p.rope_table + (long long)p.pos[row] * p.head_dim;
    for (int off = 0; off < p.head_dim; off += 32) asm volatile("prefetch.global.L2 [%0];" ::"l"(tc + off));
    return;
  }
  if (!p.accumulate || p.mode != kEpiPlain) return;
  const int rr = row % p.rg;
  const int orow = (row / p.rg) * p.rg_stride + rr + p.rg_off + (rr >= p.rg_split ? p.rg_shift : 0);
  const float* base = p.cin + (long long)orow * p.ldcin;
#pragma unroll 1
  for (int u = half; u < BN / 64; u += 2)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int col0 = n0 + 64 * u + 32 * c;
      if (col0 < N) asm volatile("prefetch.global.L2 [%0];" ::"l"(base + col0));
    }
}

// Bias and RoPE of one q|k|v head chunk pair: a = the head's columns ca .. ca + 31 (relative to n0), b = the
// columns hd / 2 further (cb), s = the pair index of a's first column. Pairs from rope_pairs on, and heads past
// rope_cols (v), keep their values.
template <int NC>
__device__ __forceinline__ void rope_rotate(float (&a)[32], float (&b)[32], const float (&cs)[NC],
                                            const float (&sn)[NC], int nr) {
  // pair j: (a, b) ← (a cos − b sin, b cos + a sin), each product rounded once, the same in every epilogue
#pragma unroll
  for (int j = 0; j < NC; ++j) {
    if (j < nr) {
      const float x = a[j], y = b[j];
      a[j] = fmaf(x, cs[j], __fmul_rn(-y, sn[j]));
      b[j] = fmaf(y, cs[j], __fmul_rn(x, sn[j]));
    }
  }
}

__device__ __forceinline__ void qkv_bias_rope(const EpiParams& p, int n0, int ca, int cb, int s, int pos,
                                              float (&a)[32], float (&b)[32]) {
  const int hd = p.head_dim, hh = hd / 2;
  if (p.bias_on) {
    add_bias(p, n0 + ca, 32, a);
    add_bias(p, n0 + cb, 32, b);
  }
  // the pairs of this chunk that rotate (a partial rotary factor leaves the rest as they are)
  const int nr = min(32, (p.rope_pairs > 0 ? p.rope_pairs : hh) - s);
  if (n0 + ca < p.rope_cols && nr > 0) {
    float cs[32], sn[32];
    const float* tc = p.rope_table + (long long)pos * hd + s;
    if (nr == 16 && p.vec_ok >= 1) {  // a half-rotary head: 16 cos and 16 sin in 16-byte vectors
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 c4 = __ldg(reinterpret_cast<const float4*>(tc) + q);
        const float4 s4 = __ldg(reinterpret_cast<const float4*>(tc + hh) + q);
        cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
        sn[4 * q] = s4.x, sn[4 * q + 1] = s4.y, sn[4 * q + 2] = s4.z, sn[4 * q + 3] = s4.w;
      }
    } else {
      load_ro(tc, nr, p.vec_ok, cs);
      load_ro(tc + hh, nr, p.vec_ok, sn);
    }
    rope_rotate(a, b, cs, sn, nr);
  }
}

// One accumulator tile (rows m0.., columns n0..) → HBM, for the thread's row. The tile's columns are
// split into 64-column units (a head of q|k|v in the RoPE mode); `half` (0 or 1) takes every other unit.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const EpiParams& p, int M, int N, int m0, int n0, uint32_t tbase,
                                              int row_in_tile, int half) {
  const int row = m0 + row_in_tile;
  const bool live = row < M;
  const int rr = row % p.rg;
  const int orow = live ? (row / p.rg) * p.rg_stride + rr + p.rg_off + (rr >= p.rg_split ? p.rg_shift : 0) : 0;
  const float rs = p.norm_sq ? norm_scale_warp(p, row - (row_in_tile & 31), row_in_tile & 31, M) : 1.0f;
  if (p.mode == kEpiPlain || (p.mode == kEpiQKV && n0 >= p.n_split)) {
    const bool gate = p.mode == kEpiQKV;
#pragma unroll 1
    for (int u = half; u < BN / 64; u += 2) {
      float sq = 0.0f;  // Σv² of the unit, for a folded norm's producer
#pragma unroll 1
      for (int c = 2 * u; c < 2 * u + 2; ++c) {
        const int col0 = n0 + 32 * c;
        if (col0 >= N) break;  // warp-uniform
        float v[32];
        load_chunk(tbase + 32 * c, v);
        if (!live) continue;
        const int nv = min(32, N - col0);
        if (!gate) {
          epi_plain_chunk(p, rs, orow, col0, nv, v, sq);
          continue;
        }
        if (p.norm_sq) scale32(v, rs);
        if (p.bias_on) add_bias(p, col0, nv, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = sigmoid_f(v[j]);
        const long long off = (long long)orow * p.ldg + (col0 - p.n_split);
        if (p.g_kind == kOutBF16)
          store_16<false>(static_cast<__nv_bfloat16*>(p.g_out) + off, nv, p.vec_ok, v);
        else if (p.g_kind == kOutF16)
          store_16<true>(static_cast<__half*>(p.g_out) + off, nv, p.vec_ok, v);
        else
          store_f32(static_cast<float*>(p.g_out) + off, nv, p.vec_ok, v);
      }
      if (p.rowsq && live && n0 + 64 * u < N) p.rowsq[(long long)orow * p.rowsq_units + (n0 >> 6) + u] = sq;
    }
  } else if (p.mode == kEpiSwiGLU) {
    // tile columns (64u .. 64u+31) are the SiLU half of output columns (n0/2 + 32u ..), (64u+32 ..) the linear half
#pragma unroll 1
    for (int u = half; u < BN / 64; u += 2) {
      const int col0 = n0 + 64 * u;
      if (col0 >= N) break;
      float a[32], b[32];
      load_chunk_pair(tbase + 64 * u, tbase + 64 * u + 32, a, b);
      if (!live) continue;
      if (p.norm_sq) {
        scale32(a, rs);
        scale32(b, rs);
      }
      if (p.bias_on) {
        add_bias(p, col0, 32, a);
        add_bias(p, col0 + 32, 32, b);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] = silu_f(a[j]) * b[j];
      const int ocol = col0 / 2;
      store_operand(p, (long long)orow * p.ldo + ocol, min(32, N / 2 - ocol), a);
    }
  } else {  // kEpiQKV, q|k|v columns: one head (head_dim columns) at a time, RoPE on q and k
    const int hd = p.head_dim, hh = hd / 2;
    const int pos = live ? p.pos[row] : 0;
#pragma unroll 1
    for (int h0 = half * hd; h0 < BN; h0 += 2 * hd) {
#pragma unroll 1
      for (int s = 0; s < hh; s += 32) {
        const int ca = h0 + s, cb = h0 + hh + s;
        if (n0 + ca >= N) break;
        float a[32], b[32];
        load_chunk_pair(tbase + ca, tbase + cb, a, b);
        if (!live) continue;
        if (p.norm_sq) {
          scale32(a, rs);
          scale32(b, rs);
        }
        qkv_bias_rope(p, n0, ca, cb, s, pos, a, b);
        store_operand(p, (long long)orow * p.ldo + n0 + ca, 32, a);
        store_operand(p, (long long)orow * p.ldo + n0 + cb, 32, b);
      }
    }
  }
}

// Which epilogue warp half (0 or 1) of a TMEM lane quarter reads the tile's 32-column chunk `c` in
// epilogue_tile: 64-column units alternate between the halves, or, for the q|k|v columns of the RoPE mode,
// whole heads do.
__device__ __forceinline__ int chunk_owner(const EpiParams& p, int n0, int c) {
  if (p.mode == kEpiQKV && n0 < p.n_split) return ((32 * c) / p.head_dim) & 1;
  return (c >> 1) & 1;
}

// The split mode's drain of one stage's partial product: for every chunk this thread's epilogue will read,
// sum += partial (FP32, round-to-nearest), or sum = partial for the tile's first stage. The sum buffer stays
// with this thread from the first stage to the epilogue, so only its own tcgen05.ld/st order it.
template <int BN>
__device__ __forceinline__ void drain_partial(const EpiParams& p, int N, int n0, int half, uint32_t part,
                                              uint32_t sum, bool first) {
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    if (n0 + 32 * c >= N) break;  // warp-uniform
    if (chunk_owner(p, n0, c) != half) continue;
    uint32_t r[32];
    tmem_ld_32x32b_x32(part + 32 * c, r);
    if (!first) {
      uint32_t q[32];
      tmem_ld_32x32b_x32(sum + 32 * c, q);
      tmem_ld_wait();
#pragma unroll
      for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(q[j])));
    } else {
      tmem_ld_wait();
    }
    tmem_st_32x32b_x32(sum + 32 * c, r);
  }
  tmem_st_wait();
}

// ---- problems and groups ----------------------------------------------------------------------
// One GEMM of a launch: its operands' tensor maps, shape, epilogue and the first tile it owns in the launch's
// tile walk. A grouped launch walks the tiles of up to kMaxGemmGroup problems one after another, so GEMMs
// that are independent of each other (the heads of a headwise projection, two projections of one input) share
// one persistent grid. G = 1 is the plain single GEMM.
struct alignas(64) GemmProblem {
  CUtensorMap a, w;    // A [M, K] and W [N, K]
  CUtensorMap a2, w2;  // the split mode's lo parts; the staged epilogues' maps of their outputs and residual
  CUtensorMap o2;      // the staged residual epilogue's 16-bit copy of its output (a folded norm's producer)
  EpiParams ep;
  int M, N, kblks, n_blks, tile0;
};

template <int G>
struct GemmGroup {
  GemmProblem p[G];
  int count, tiles;
  // The problem that owns tile t of the walk, and t's index within that problem's tiles.
  __device__ __forceinline__ const GemmProblem& of(int t, int& local) const {
    int i = 0;
    if constexpr (G > 1) {
      while (i + 1 < count && t >= p[i + 1].tile0) ++i;
    }
    local = t - p[i].tile0;
    return p[i];
  }
};

// ---- the kernel -----------------------------------------------------------------------------
// RESID: the launch's one problem is a residual GEMM (residual_preloaded): its epilogue loop reads the residual
// early. A separate instantiation, so the other kernels keep their register allocation.
template <int BN, int OPK, int G, bool RESID>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ GemmGroup<G> grp, uint32_t* err) {
  using C = Cfg<BN, OPK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + C::NACC;
  uint64_t* drain = acc_empty + C::NACC;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = grp.tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    for (int i = 0; i < grp.count; ++i) {
      prefetch_tmap(&grp.p[i].a);
      prefetch_tmap(&grp.p[i].w);
      if (OPK == kOpSplit) {
        prefetch_tmap(&grp.p[i].a2);
        prefetch_tmap(&grp.p[i].w2);
      }
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        int lt;
        const GemmProblem& P = grp.of(t, lt);
        const int m0 = (lt / P.n_blks) * C::BM, n0 = (lt % P.n_blks) * BN;
        for (int kb = 0; kb < P.kblks; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1) || *abort_flag) {
            atomicOr(err, kErrTimeoutEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          uint8_t* sb = sa + C::A_BYTES;
          mbar_arrive_expect_tx(full + stage, C::STAGE_BYTES);
          tma_load_2d(sa, &P.a, full + stage, kb * C::BK, m0);
          tma_load_2d(sb, &P.w, full + stage, kb * C::BK, n0);
          if (OPK == kOpSplit) {
            tma_load_2d(sb + C::B_BYTES, &P.a2, full + stage, kb * C::BK, m0);
            tma_load_2d(sb + C::B_BYTES + C::A_BYTES, &P.w2, full + stage, kb * C::BK, n0);
          }
          ++issued;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // let the copies still in flight land before the CTA's shared memory goes away
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < C::STAGES && i < issued; ++i) {
          if (--s < 0) {
            s = C::STAGES - 1;
            ph ^= 1;
          }
          mbar_wait(full + s, ph);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      int slab = 0;  // split mode: stages issued so far, each into partial buffer slab % NACC
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++it) {
        int lt;
        const int kblks = grp.of(t, lt).kblks;
        const int buf = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!C::SLAB && (!mbar_wait(acc_empty + buf, aph ^ 1) || *abort_flag)) {
          atomicOr(err, kErrTimeoutAccFree);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < kblks; ++kb) {
          if (C::SLAB) {
            const int pb = slab % C::NACC;
            if (!mbar_wait(acc_empty + pb, ((slab / C::NACC) & 1) ^ 1) || *abort_flag) {
              atomicOr(err, kErrTimeoutAccFree);
              *abort_flag = 1;
              ok = false;
              break;
            }
            tc_fence_after();
            d = tmem + pb * BN;
          }
          if (!mbar_wait(full + stage, phase) || *abort_flag) {
            atomicOr(err, kErrTimeoutFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::NSUB; ++k) {
            const uint64_t ad = sdesc_k_sw128(sa + 32 * k);
            const uint64_t bd = sdesc_k_sw128(sb + 32 * k);
            const uint32_t acc = ((kb > 0 && !C::SLAB) || k > 0) ? 1u : 0u;
            if (OPK == kOpBF16 || OPK == kOpF16) {
              umma_bf16(d, ad, bd, C::IDESC, acc);
            } else if (OPK == kOpTF32) {
              umma_tf32(d, ad, bd, C::IDESC, acc);
            } else {
              const uint64_t ad2 = sdesc_k_sw128(sb + C::B_BYTES + 32 * k);
              const uint64_t bd2 = sdesc_k_sw128(sb + C::B_BYTES + C::A_BYTES + 32 * k);
              // smallest terms first; lo·lo halves the split's error against an FP32 product
              umma_tf32(d, ad2, bd2, C::IDESC, acc);  // lo·lo
              umma_tf32(d, ad2, bd, C::IDESC, 1u);    // lo·hi
              umma_tf32(d, ad, bd2, C::IDESC, 1u);    // hi·lo
              umma_tf32(d, ad, bd, C::IDESC, 1u);    // hi·hi
            }
          }
          umma_commit(empty + stage);
          if (C::SLAB) umma_commit(acc_full + (slab++ % C::NACC));
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (!C::SLAB) umma_commit(acc_full + buf);
      }
      // every MMA this thread issued has completed once `drain` flips
      umma_commit(drain);
      mbar_wait(drain, 0);
    }
  } else if (C::SLAB) {
    // ---- split-mode epilogue: drain each stage's partial into the sum buffer, then the tile's epilogue ----
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t sum = tmem + lanes + C::NACC * BN;
    int slab = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      int lt;
      const GemmProblem& P = grp.of(t, lt);
      const int m0 = (lt / P.n_blks) * C::BM, n0 = (lt % P.n_blks) * BN;
      for (int kb = 0; kb < P.kblks; ++kb, ++slab) {
        const int pb = slab % C::NACC;
        const bool got = mbar_wait(acc_full + pb, (slab / C::NACC) & 1);
        if (!(__all_sync(0xffffffffu, got) && !*abort_flag)) {
          if (lane == 0) atomicOr(err, kErrTimeoutAcc);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        drain_partial<BN>(P.ep, P.N, n0, half, tmem + lanes + pb * BN, sum, kb == 0);
        tc_fence_before();
        mbar_arrive(acc_empty + pb);
      }
      if (!ok) break;
      epilogue_tile<BN>(P.ep, P.M, P.N, m0, n0, sum, row_in_tile, half);
    }
  } else {
    // ---- epilogue: warps 2..9; TMEM lane quarter = warp % 4, column half = (warp - 2) / 4 ----
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    // the residual-preloading loop for a residual GEMM (RESID), else the general one
    auto loop = [&](auto pre_tag) {
      constexpr bool PRE = decltype(pre_tag)::value;
      int it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        int lt;
        const GemmProblem& P = grp.of(t, lt);
        const int m0 = (lt / P.n_blks) * C::BM, n0 = (lt % P.n_blks) * BN;
        ResidualPre rp;
        if constexpr (PRE)
          residual_preload(P.ep, P.M, P.N, m0, n0, row_in_tile, half, rp);
        else
          prefetch_residual<BN>(P.ep, P.M, P.N, m0, n0, row_in_tile, half);
        const bool got = mbar_wait(acc_full + buf, aph);
        const bool all = __all_sync(0xffffffffu, got) && !*abort_flag;
        if (!all) {
          if (lane == 0) atomicOr(err, kErrTimeoutAcc);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        // the next tile's residual / table lines, a whole epilogue ahead of their use
        const int tn = t + gridDim.x;
        if (tn < tiles) {
          int ln;
          const GemmProblem& Q = grp.of(tn, ln);
          prefetch_residual<BN>(Q.ep, Q.M, Q.N, (ln / Q.n_blks) * C::BM, (ln % Q.n_blks) * BN, row_in_tile, half);
        }
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
        if constexpr (PRE)
          epilogue_tile_residual<BN>(P.ep, P.M, P.N, m0, n0, tbase, row_in_tile, half, rp);
        else
          epilogue_tile<BN>(P.ep, P.M, P.N, m0, n0, tbase, row_in_tile, half);
        tc_fence_before();
        mbar_arrive(acc_empty + buf);
      }
    };
    if constexpr (RESID)
      loop(std::true_type{});
    else
      loop(std::false_type{});
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---- the CTA-pair kernel --------------------------------------------------------------------
// The same GEMM over 256 × 256 tiles shared by a cluster of two CTAs on neighbouring SMs: each CTA stages
// its own 128 rows of A and its own 128 rows (half of the tile's N) of W, and one thread of CTA 0 issues
// tcgen05.mma.cta_group::2 (M 256 × N 256) that reads both CTAs' tiles and leaves each CTA's 128 rows of
// the accumulator in its own TMEM. Per SM that halves the W bytes per MMA, so six 32 KB stages stay in
// flight instead of four 48 KB ones. Both CTAs' TMA loads complete on CTA 0's stage barrier (armed by CTA
// 0 for both CTAs' bytes); CTA 0's commits arrive on both CTAs' stage-free and accumulator-ready barriers;
// each CTA's epilogue warps release an accumulator with one arrive on CTA 0's barrier. No TMA multicast.
// WIDE: 256 × 512 tiles, two N = 256 MMAs per K step into one 512-column accumulator. A row block is then read
// from L2 once per 512 output columns instead of once per 256, 25 % fewer operand bytes per FLOP on the L2 → SM
// path that bounds this kernel; with TMEM full, the next tile's MMAs wait for the epilogue, while the TMA
// producer keeps filling the stages. Otherwise 256 × 256 tiles with two accumulators.
// RS > 0: the staged epilogues (EPI 2 and 3 below) give each epilogue warp a ring of RS shared-memory slots of
// 4 KB (32 rows × 128 bytes, 128-byte swizzle); the operand stages shrink to make room.
template <int OPK_, bool WIDE_ = false, int RS_ = 0>
struct CfgPair {
  static constexpr int OPK = OPK_;
  static constexpr bool WIDE = WIDE_;
  static constexpr int RS = RS_;
  static constexpr int BN = WIDE ? 512 : 256;  // tile N; each CTA stages BN / 2 rows of W, in 128-row chunks
  static constexpr int BM = 128;               // rows per CTA; the tile is 2 · BM rows
  static constexpr int MMA_N = 256;            // N of one tcgen05.mma; BN / MMA_N of them per K step
  static constexpr int NMMA = BN / MMA_N;
  static constexpr int ESZ = (OPK == kOpBF16 || OPK == kOpF16) ? 2 : 4;
  static constexpr int BK = 128 / ESZ;
  static constexpr int UK = 32 / ESZ;
  static constexpr int NSUB = BK / UK;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_CHUNK = (MMA_N / 2) * 128;  // this CTA's 128 W rows of one MMA
  static constexpr int B_BYTES = NMMA * B_CHUNK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = WIDE ? (RS ? 3 : 4) : (RS ? 4 : 6);
  static constexpr int NACC = WIDE ? 1 : 2;  // accumulators of BN columns in the 512 TMEM columns
  static constexpr int TMEM_COLS = 512;
  static constexpr int SLOT_BYTES = 32 * 32 * 4;
  static constexpr int RING_BYTES = kEpiWarps * RS * SLOT_BYTES;
  static constexpr int BAR_BYTES = 256 + kEpiWarps * RS * 8;
  static constexpr int SMEM = STAGES * STAGE_BYTES + RING_BYTES + BAR_BYTES + 1024;
  static constexpr uint32_t IDESC = idesc_f32acc(OPK == kOpBF16 ? 1u : OPK == kOpF16 ? 0u : 2u, 2 * BM, MMA_N);
  static_assert(OPK != kOpSplit, "the split FP32 mode runs on the single-CTA kernel");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(NACC * BN == TMEM_COLS, "TMEM columns");
};

// The thread's 32 values as 16-bit into 16-byte chunks q0 .. q0 + 3 of its 128-byte slot row (128-byte swizzle).
__device__ __forceinline__ void slot_row16(uint32_t rowp, int lane, int q0, bool f16, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = f16 ? pack_f16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]) : pack_bf16(v[8 * q + 2 * e], v[8 * q + 2 * e + 1]);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(rowp + (((q0 + q) ^ (lane & 7)) << 4)), "r"(w[0]),
                 "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  }
}

// One epilogue warp of the staged residual epilogue (EPI 2, or EPI 4 with NORM) over the pair's tiles. The warp's chunks form
// one sequence over its tiles: chunk k of a tile covers the warp's 32 rows (TMEM lanes 32·quarter ..) and the
// columns n0 + 64·(half + 2·(k / 2)) + 32·(k % 2), k < BN / 64, as in the general epilogue. Chunk j lives in slot
// j % RS; lane 0 loads chunk j + RS − 1 after chunk j has been stored, once chunk j − 1's store has read its slot
// (one bulk group per chunk). A chunk outside the output (columns ≥ N or rows ≥ M) moves nothing: lane 0 completes
// its slot's barrier phase with a plain arrival. P.a2 maps the residual C_in and P.w2 the output C, 32 × 32 boxes.
// NORM (a folded RMSNorm's producer): the last of the warp's RS slots instead collects each 64-column unit's 16-bit
// copy of the output, stored by one box of 64 × 32 through P.o2, and each thread stores its row's Σv² over the
// unit to rowsq. Bulk groups then go FP16 unit store (an empty group when there is none), FP32 chunk store at the
// end of a unit, FP32 chunk store alone otherwise.
template <class C, bool NORM>
__device__ __forceinline__ void staged_residual_epilogue(const GemmProblem& P, int pair, int pairs, int tiles,
                                                         uint32_t rank, uint32_t tmem, uint64_t* acc_full,
                                                         uint32_t acc_empty0, volatile uint32_t* abort_flag,
                                                         uint32_t* err, uint8_t* ring, uint64_t* rbar, int quarter,
                                                         int half, int lane) {
  constexpr int BN = C::BN, RS = NORM ? C::RS - 1 : C::RS, KPT = BN / 64;  // RS: the FP32 slots
  static_assert(RS >= 2, "the FP32 ring needs two slots");
  const int my_tiles = pair < tiles ? (tiles - pair + pairs - 1) / pairs : 0;
  const int jobs = my_tiles * KPT;
  const EpiParams& ep = P.ep;
  // the chunk's column and row origin; false if it lies outside the output
  auto where = [&](int j, int& col0, int& row0) {
    const int t = pair + (j / KPT) * pairs, k = j % KPT;
    row0 = (t / P.n_blks) * 2 * C::BM + static_cast<int>(rank) * C::BM + quarter * 32;
    col0 = (t % P.n_blks) * BN + 64 * (half + 2 * (k >> 1)) + 32 * (k & 1);
    return col0 < P.N && row0 < P.M;
  };
  auto issue = [&](int j) {  // lane 0
    uint64_t* bar = rbar + j % RS;
    int col0, row0;
    if (where(j, col0, row0)) {
      mbar_arrive_expect_tx(bar, C::SLOT_BYTES);
      tma_load_2d(ring + (j % RS) * C::SLOT_BYTES, &P.a2, bar, col0, row0);
    } else {
      mbar_arrive(bar);
    }
  };
  int issued = 0;
  if (lane == 0)
    for (; issued < RS - 1 && issued < jobs; ++issued) issue(issued);
  const bool f16 = ep.o_kind == kOutF16;
  const uint32_t hrow = smem_u32(ring + RS * C::SLOT_BYTES) + lane * 128;  // NORM: this thread's row of the unit slot
  float sq = 0.0f;
  bool ok = true;
  int j = 0;
  for (int it = 0; it < my_tiles && ok; ++it) {
    const int buf = it % C::NACC;
    const bool got = mbar_wait(acc_full + buf, (it / C::NACC) & 1);
    if (!(__all_sync(0xffffffffu, got) && !*abort_flag)) {
      if (lane == 0) atomicOr(err, kErrTimeoutAcc);
      *abort_flag = 1;
      ok = false;
      break;
    }
    tc_fence_after();
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
#pragma unroll 1
    for (int k = 0; k < KPT; ++k, ++j) {
      int col0, row0;
      const bool live = where(j, col0, row0);
      const uint32_t slot = smem_u32(ring + (j % RS) * C::SLOT_BYTES);
      uint32_t acc[32];
      if (live) tmem_ld_32x32b_x32(tbase + 64 * (half + 2 * (k >> 1)) + 32 * (k & 1), acc);
      const bool have = mbar_wait(rbar + j % RS, (j / RS) & 1);
      if (!__all_sync(0xffffffffu, have)) {
        if (live) tmem_ld_wait();
        if (lane == 0) atomicOr(err, kErrTimeoutResidual);
        *abort_flag = 1;
        ok = false;
        break;
      }
      if (NORM && (k & 1) == 0) {
        if (lane == 0) bulk_wait_read<1>();  // the last unit's 16-bit store has read the unit slot
        __syncwarp();
      }
      if (live) {
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(acc[q]);
        if (ep.bias_on) add_bias(ep, col0, min(32, P.N - col0), v);
        // the thread's row of the slot: 16-byte chunk q at q ^ (row % 8), the 128-byte swizzle
        const uint32_t rowp = slot + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t a = rowp + ((q ^ (lane & 7)) << 4);
          const float4 r = lds_f32x4(a);
          v[4 * q] += r.x, v[4 * q + 1] += r.y, v[4 * q + 2] += r.z, v[4 * q + 3] += r.w;
          sts_f32x4(a, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
        }
        if constexpr (NORM) {
#pragma unroll
          for (int q = 0; q < 32; ++q) sq += v[q] * v[q];
          slot_row16(hrow, lane, 4 * (k & 1), f16, v);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      const bool unit_end = NORM && (k & 1) == 1;
      if (unit_end) {
        const int row = row0 + lane;
        if (live && row < P.M) ep.rowsq[(long long)row * ep.rowsq_units + (col0 >> 6)] = sq;
        sq = 0.0f;
      }
      if (lane == 0) {
        if (unit_end) {
          if (live) tma_store_2d(&P.o2, ring + RS * C::SLOT_BYTES, col0 - 32, row0);
          bulk_commit();
        }
        if (live) tma_store_2d(&P.w2, ring + (j % RS) * C::SLOT_BYTES, col0, row0);
        bulk_commit();
        if (issued < jobs) {
          // chunk j − 1's store has read the slot chunk j + RS − 1 reuses (the unit's 16-bit store may be pending too)
          if (unit_end)
            bulk_wait_read<2>();
          else
            bulk_wait_read<1>();
          issue(issued++);
        }
      }
    }
    if (!ok) break;
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * buf);
  }
  if (lane == 0) {
    // loads still in flight after an abort land before the CTA's shared memory is released
    for (int q = j; q < issued; ++q) mbar_wait(rbar + q % RS, (q / RS) & 1);
    bulk_wait<0>();
  }
  __syncwarp();
}


// One epilogue warp of the staged 16-bit epilogue (EPI 3 or 5) over the pair's tiles, for the q|k|v|gate, the
// SwiGLU and the plain 16-bit-output GEMMs: each 64-column block of 16-bit output — a head of q|k|v with its bias
// and RoPE, 64 gate columns with bias and sigmoid, the SwiGLU products of two 64-column tile units, or 64 columns
// with bias and activation — goes through a slot of the warp's
// ring (32 rows × 64 16-bit columns, 4 KB, 128-byte swizzle) and out by one bulk-tensor store (P.a2 maps the
// q|k|v or SwiGLU output, P.w2 the gate output, boxes of 64 × 32). Block j lives in slot j % RS; lane 0 reuses a
// slot once the store that last read it has done so (one bulk group per block).
template <class C>
__device__ __forceinline__ void staged_16bit_epilogue(const GemmProblem& P, int pair, int pairs, int tiles,
                                                    uint32_t rank, uint32_t tmem, uint64_t* acc_full,
                                                    uint32_t acc_empty0, volatile uint32_t* abort_flag,
                                                    uint32_t* err, uint8_t* ring, int quarter, int half, int lane) {
  constexpr int BN = C::BN;
  // two output slots; a third, where the ring has one, holds the warp's rows of the packed RoPE table
  constexpr int RS = 2;
  constexpr bool TSLOT = C::RS >= 3;
  const EpiParams& ep = P.ep;
  const bool f16 = ep.o_kind == kOutF16;
  const uint32_t tslot = smem_u32(ring + 2 * C::SLOT_BYTES) + lane * 128;  // this thread's row of the table slot
  int j = 0;
  int it = 0;
  for (int t = pair; t < tiles; t += pairs, ++it) {
    const int buf = it % C::NACC;
    const int m0 = (t / P.n_blks) * 2 * C::BM + static_cast<int>(rank) * C::BM, n0 = (t % P.n_blks) * BN;
    const int row0 = m0 + quarter * 32, row = row0 + lane;
    const bool rows_live = row0 < P.M;  // warp-uniform
    const bool swiglu = ep.mode == kEpiSwiGLU;
    const bool plain = ep.mode == kEpiPlain;
    const bool heads = !swiglu && !plain && n0 < ep.n_split;
    // what the tile's epilogue reads from memory, before it waits for the accumulator: the rows' norm scales, their
    // positions and (packed table) their RoPE table rows
    const float rs = ep.norm_sq ? norm_scale_warp(ep, row0, lane, P.M) : 1.0f;
    const int pos = heads && row < P.M ? ep.pos[row] : 0;
    const bool packed = TSLOT && heads && ep.rope_pack && n0 < ep.rope_cols && ep.rope_pairs > 0 &&
                        ep.rope_pairs <= 16;  // warp-uniform
    if (packed) {
      __syncwarp();  // the last tile's reads of the table slot are done
      const int pos0 = __shfl_sync(0xffffffffu, pos, 0);
      const float4* src = reinterpret_cast<const float4*>(ep.rope_pack);
      const uint32_t tbase0 = tslot - lane * 128;
      if (__all_sync(0xffffffffu, row < P.M && pos == pos0 + lane)) {
        // consecutive positions: one contiguous 4 KB block, read coalesced and spread over the rows
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int i = lane + 32 * k, r = i >> 3, c = i & 7;
          sts_f32x4(tbase0 + r * 128 + ((c ^ (r & 7)) << 4), __ldg(src + (long long)(pos0 + r) * 8 + c));
        }
      } else if (row < P.M) {
#pragma unroll
        for (int c = 0; c < 8; ++c) sts_f32x4(tslot + ((c ^ (lane & 7)) << 4), __ldg(src + (long long)pos * 8 + c));
      }
      __syncwarp();
    }
    const bool got = mbar_wait(acc_full + buf, (it / C::NACC) & 1);
    if (!(__all_sync(0xffffffffu, got) && !*abort_flag)) {
      if (lane == 0) atomicOr(err, kErrTimeoutAcc);
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
    // SwiGLU: block i = tile units 2i, 2i + 1 → output columns n0 / 2 + 64 i ..; otherwise block i = unit i
#pragma unroll 1
    for (int i = half; i < (swiglu ? BN / 128 : BN / 64); i += 2, ++j) {
      const int c0 = n0 + 64 * (swiglu ? 2 * i : i);
      if (c0 >= P.N) break;  // warp-uniform
      uint8_t* slot = ring + (j % RS) * C::SLOT_BYTES;
      const uint32_t rowp = smem_u32(slot) + lane * 128;
      if (lane == 0) bulk_wait_read<RS - 1>();  // the store that last read this slot has read it
      __syncwarp();
      if (swiglu) {
        // tile columns 64u .. 64u + 31 are the SiLU half of output columns n0 / 2 + 32u .., 64u + 32 .. the linear one
#pragma unroll 1
        for (int h = 0; h < 2; ++h) {
          const int u = 2 * i + h;
          float a[32], b[32];
          load_chunk_pair(tbase + 64 * u, tbase + 64 * u + 32, a, b);
          if (ep.norm_sq) {
            scale32(a, rs);
            scale32(b, rs);
          }
          if (ep.bias_on) {
            add_bias(ep, n0 + 64 * u, 32, a);
            add_bias(ep, n0 + 64 * u + 32, 32, b);
          }
#pragma unroll
          for (int q = 0; q < 32; ++q) a[q] = silu_f(a[q]) * b[q];
          slot_row16(rowp, lane, 4 * h, f16, a);
        }
      } else {
        float a[32], b[32];
        load_chunk_pair(tbase + 64 * i, tbase + 64 * i + 32, a, b);
        if (ep.norm_sq) {
          scale32(a, rs);
          scale32(b, rs);
        }
        if (heads && packed) {
          if (ep.bias_on) {
            add_bias(ep, c0, 32, a);
            add_bias(ep, c0 + 32, 32, b);
          }
          if (c0 < ep.rope_cols) {
            float cs[16], sn[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float4 cv = lds_f32x4(tslot + ((q ^ (lane & 7)) << 4));
              const float4 sv = lds_f32x4(tslot + (((q + 4) ^ (lane & 7)) << 4));
              cs[4 * q] = cv.x, cs[4 * q + 1] = cv.y, cs[4 * q + 2] = cv.z, cs[4 * q + 3] = cv.w;
              sn[4 * q] = sv.x, sn[4 * q + 1] = sv.y, sn[4 * q + 2] = sv.z, sn[4 * q + 3] = sv.w;
            }
            rope_rotate(a, b, cs, sn, ep.rope_pairs);
          }
        } else if (heads) {
          qkv_bias_rope(ep, n0, 64 * i, 64 * i + 32, 0, pos, a, b);
        } else if (plain) {
          // bias → activation as in the general epilogue (the norm scale is applied above; 1 leaves it exact)
          epi_act_chunk(ep, 1.0f, c0, 32, a);
          epi_act_chunk(ep, 1.0f, c0 + 32, 32, b);
        } else {
          if (ep.bias_on) {
            add_bias(ep, c0, 32, a);
            add_bias(ep, c0 + 32, 32, b);
          }
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            a[q] = sigmoid_f(a[q]);
            b[q] = sigmoid_f(b[q]);
          }
        }
        slot_row16(rowp, lane, 0, f16, a);
        slot_row16(rowp, lane, 4, f16, b);
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if (rows_live) {
          if (swiglu)
            tma_store_2d(&P.a2, slot, c0 / 2, row0);
          else if (heads || plain)
            tma_store_2d(&P.a2, slot, c0, row0);
          else
            tma_store_2d(&P.w2, slot, c0 - ep.n_split, row0);
        }
        bulk_commit();
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * buf);
  }
  if (lane == 0) bulk_wait<0>();
  __syncwarp();
}

// Slots per epilogue warp of the staged epilogues' rings: the residual epilogue three with 256-wide tiles and two
// beside the wide tiles' 48 KB stages; the 16-bit epilogue two output slots, plus a slot for the packed RoPE table
// rows with 256-wide tiles; the residual epilogue of a folded norm's producer three (two FP32 slots and the unit
// slot of its 16-bit copy; 256-wide tiles only).
template <bool WIDE, int EPI>
constexpr int epi_slots() {
  return EPI == 2 ? (WIDE ? 2 : 3) : EPI == 3 ? (WIDE ? 2 : 3) : EPI == 4 ? 3 : EPI == 5 ? 2 : 0;
}

// EPI: 0 the general epilogue; 1 a residual GEMM with the register-preloading epilogue; 2 a residual GEMM with
// the staged epilogue; 3 the staged 16-bit epilogue of a q|k|v|gate GEMM (with a slot for the packed RoPE rows);
// 4 the staged residual epilogue of a folded norm's producer; 5 the staged 16-bit epilogue of a SwiGLU GEMM or of
// a plain GEMM with only a 16-bit output. The
// staged epilogues move their outputs (and the
// residual GEMM its FP32 residual) by TMA through shared memory: each epilogue warp
// loads its 32 rows × 32 columns of the residual into a slot of its ring two chunks ahead (the next tile's first
// chunks while the MMAs of that tile still run), adds the accumulator chunk and the bias in place, and stores the
// slot back with one bulk-tensor store. The residual and the result thereby bypass the per-thread load and store
// path, whose uncoalesced 32-row requests (one row per thread) kept the SM's L1 busy for most of the epilogue.
template <int OPK, int G, bool WIDE, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_pair_kernel(const __grid_constant__ GemmGroup<G> grp, uint32_t* err) {
  using C = CfgPair<OPK, WIDE, epi_slots<WIDE, EPI>()>;
  constexpr int BN = C::BN;
  static_assert(EPI < 2 || G == 1, "the staged epilogues serve single GEMMs");
  static_assert(EPI != 4 || !WIDE, "a folded norm's producer runs 256-wide tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + C::RING_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;
  uint64_t* acc_empty = acc_full + C::NACC;
  uint64_t* drain = acc_empty + C::NACC;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile uint32_t* abort_flag = tmem_holder + 1;
  uint64_t* rbar = drain + 2;  // kEpiWarps × RS residual-slot barriers

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int tiles = grp.tiles;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < C::NACC; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, 2 * kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kEpiWarps * C::RS; ++i) mbar_init(rbar + i, 1);
    *abort_flag = 0;
    fence_mbar_init();
    for (int i = 0; i < grp.count; ++i) {
      prefetch_tmap(&grp.p[i].a);
      prefetch_tmap(&grp.p[i].w);
      if constexpr (EPI >= 2) {
        prefetch_tmap(&grp.p[i].a2);
        prefetch_tmap(&grp.p[i].w2);
      }
      if constexpr (EPI == 4) prefetch_tmap(&grp.p[i].o2);
    }
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // both CTAs' barriers exist and their TMEM is allocated before any cross-CTA arrival or load
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs): this CTA's A rows and W half, counted on CTA 0's stage barrier ----
      const uint32_t full0 = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs) {
        int lt;
        const GemmProblem& P = grp.of(t, lt);
        const int m0 = (lt / P.n_blks) * 2 * C::BM + static_cast<int>(rank) * C::BM;
        // this CTA's 128 W rows of each MMA: rows n_tile + 256·j + 128·rank
        const int n0 = (lt % P.n_blks) * BN + static_cast<int>(rank) * (C::MMA_N / 2);
        for (int kb = 0; kb < P.kblks; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1) || *abort_flag) {
            atomicOr(err, kErrTimeoutEmpty);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * C::STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(full + stage, 2 * C::STAGE_BYTES);
          tma_load_2d_pair(sa, &P.a, full0 + 8 * stage, kb * C::BK, m0);
#pragma unroll
          for (int j = 0; j < C::NMMA; ++j)
            tma_load_2d_pair(sa + C::A_BYTES + j * C::B_CHUNK, &P.w, full0 + 8 * stage, kb * C::BK,
                             n0 + j * C::MMA_N);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (CTA 0 only) ----
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < tiles && ok; t += pairs, ++it) {
        int lt;
        const int kblks = grp.of(t, lt).kblks;
        const int buf = it % C::NACC;
        const uint32_t aph = (it / C::NACC) & 1;
        if (!mbar_wait(acc_empty + buf, aph ^ 1) || *abort_flag) {
          atomicOr(err, kErrTimeoutAccFree);
          *abort_flag = 1;
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < kblks; ++kb) {
          if (!mbar_wait(full + stage, phase) || *abort_flag) {
            atomicOr(err, kErrTimeoutFull);
            *abort_flag = 1;
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * C::STAGE_BYTES);
          const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
          for (int k = 0; k < C::NSUB; ++k) {
            const uint64_t ad = sdesc_k_sw128(sa + 32 * k);
            const uint32_t acc = (kb > 0 || k > 0) ? 1u : 0u;
#pragma unroll
            for (int j = 0; j < C::NMMA; ++j) {
              const uint64_t bd = sdesc_k_sw128(sb + j * C::B_CHUNK + 32 * k);
              if (OPK == kOpTF32)
                umma_tf32_pair(d + j * C::MMA_N, ad, bd, C::IDESC, acc);
              else
                umma_f16_pair(d + j * C::MMA_N, ad, bd, C::IDESC, acc);
            }
          }
          umma_commit_pair_multicast(empty + stage, 0x3);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_multicast(acc_full + buf, 0x3);
      }
      // every MMA this thread issued has completed once `drain` flips
      umma_commit_pair(smem_u32(drain));
      mbar_wait(drain, 0);
    }
  } else {
    // ---- epilogue (both CTAs): warps 2..9; this CTA's 128 rows of each tile ----
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t acc_empty0 = mapa_shared(smem_u32(acc_empty), 0);
    // as in the single-CTA kernel: the residual-preloading loop for a residual GEMM (EPI 1), else the general one
    auto loop = [&](auto pre_tag) {
      constexpr bool PRE = decltype(pre_tag)::value;
      int it = 0;
      for (int t = pair; t < tiles; t += pairs, ++it) {
        const int buf = it % C::NACC;
        const uint32_t aph = (it / C::NACC) & 1;
        int lt;
        const GemmProblem& P = grp.of(t, lt);
        const int m0 = (lt / P.n_blks) * 2 * C::BM + static_cast<int>(rank) * C::BM, n0 = (lt % P.n_blks) * BN;
        ResidualPre rp;
        if constexpr (PRE)
          residual_preload(P.ep, P.M, P.N, m0, n0, row_in_tile, half, rp);
        else
          prefetch_residual<BN>(P.ep, P.M, P.N, m0, n0, row_in_tile, half);
        const bool got = mbar_wait(acc_full + buf, aph);
        const bool all = __all_sync(0xffffffffu, got) && !*abort_flag;
        if (!all) {
          if (lane == 0) atomicOr(err, kErrTimeoutAcc);
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const int tn = t + pairs;
        if (tn < tiles) {
          int ln;
          const GemmProblem& Q = grp.of(tn, ln);
          prefetch_residual<BN>(Q.ep, Q.M, Q.N, (ln / Q.n_blks) * 2 * C::BM + static_cast<int>(rank) * C::BM,
                                (ln % Q.n_blks) * BN, row_in_tile, half);
        }
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + buf * BN;
        if constexpr (PRE)
          epilogue_tile_residual<BN>(P.ep, P.M, P.N, m0, n0, tbase, row_in_tile, half, rp);
        else
          epilogue_tile<BN>(P.ep, P.M, P.N, m0, n0, tbase, row_in_tile, half);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acc_empty0 + 8 * buf);
      }
    };
    if constexpr (EPI == 3 || EPI == 5)
      staged_16bit_epilogue<C>(grp.p[0], pair, pairs, tiles, rank, tmem, acc_full, acc_empty0, abort_flag, err,
                               ring + (warp - 2) * C::RS * C::SLOT_BYTES, quarter, half, lane);
    else if constexpr (EPI == 2 || EPI == 4)
      staged_residual_epilogue<C, EPI == 4>(grp.p[0], pair, pairs, tiles, rank, tmem, acc_full, acc_empty0, abort_flag,
                                            err, ring + (warp - 2) * C::RS * C::SLOT_BYTES, rbar + (warp - 2) * C::RS,
                                            quarter, half, lane);
    else if constexpr (EPI == 1)
      loop(std::true_type{});
    else
      loop(std::false_type{});
  }
  tc_fence_before();
  __syncthreads();
  // neither CTA frees its TMEM or exits while the other's MMAs, loads or arrivals may still target it
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, C::TMEM_COLS);
  }
}

// ---- host side ---------------------------------------------------------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A 2-D K-major tensor map: `rows` rows of `k` elements, `ld` elements apart; box = 128 bytes × box_rows.
static bool make_map(CUtensorMap* map, const void* base, int op, long long rows, long long k, long long ld,
                     int box_rows) {
  auto enc = get_encode();
  if (!enc) return false;
  const int esz = (op == kOpBF16 || op == kOpF16) ? 2 : 4;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * esz)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType dt = op == kOpBF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : op == kOpF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUresult r = enc(map, dt, 2,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_operand_map(CUtensorMap* map, const void* base, int op, long long rows, long long k, long long ld,
                      int box_rows) {
  return make_map(map, base, op, rows, k, ld, box_rows);
}

EpiParams epi_default() {
  EpiParams p{};
  p.rg = 1 << 30;
  p.rg_stride = 1 << 30;
  p.rg_off = 0;
  p.rg_split = 1 << 30;
  p.rg_shift = 0;
  p.vec_ok = 0;
  return p;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Tile widths (bit 0: 64, bit 1: 128, bit 2: 256, bit 3: 512) that keep heads and the gate split whole.
static int qkv_tile_choices(const EpiParams& e) {
  int bits = 0, i = 0;
  for (int bn : {64, 128, 256, 512}) {
    const bool heads_ok = e.rope_cols == 0 || bn % e.head_dim == 0;
    if (heads_ok && e.n_split % bn == 0) bits |= 1 << i;
    ++i;
  }
  return bits;
}

const char* check_gemm(const GemmArgs& g) {
  if (g.M < 1 || g.N < 1 || g.K < 1) return "M, N and K must be positive";
  if (g.op < kOpBF16 || g.op > kOpF16) return "unknown operand kind";
  const int esz = (g.op == kOpBF16 || g.op == kOpF16) ? 2 : 4;
  if (!g.a_hi || !g.w_hi) return "null operand";
  if (g.op == kOpSplit && (!g.a_lo || !g.w_lo)) return "split operands need hi and lo buffers";
  if (!aligned16(g.a_hi) || !aligned16(g.w_hi) || (g.a_lo && !aligned16(g.a_lo)) || (g.w_lo && !aligned16(g.w_lo)))
    return "operand base addresses must be 16-byte aligned";
  if ((g.lda * esz) % 16 != 0 || (g.ldw * esz) % 16 != 0) return "operand row pitch must be a multiple of 16 bytes";
  if (g.lda < g.K || g.ldw < g.K) return "leading dimension smaller than K";
  const EpiParams& e = g.ep;
  if (e.mode == kEpiSwiGLU && (g.N % 64 != 0)) return "SwiGLU GEMM needs N % 64 == 0";
  if (e.mode == kEpiQKV) {
    if (e.rope_cols > 0 && (e.head_dim % 64 != 0 || e.rope_cols % e.head_dim != 0))
      return "fused RoPE needs head_dim % 64 == 0 and whole heads";
    if (e.rope_cols > 0 && (!e.pos || !e.rope_table)) return "fused RoPE needs positions and a table";
    if (e.n_split % 64 != 0) return "the gate columns must start on a 64-column boundary";
    if (g.N > e.n_split && !e.g_out) return "gate columns without a gate output";
    if ((qkv_tile_choices(e) & 7) == 0) return "no tile width fits the q|k|v|gate layout";
  }
  if (e.accumulate && !e.cin) return "accumulate without C input";
  if (e.rowsq && e.rowsq_units < (g.N + 63) / 64) return "rowsq needs a partial sum per 64-column unit";
  if (e.norm_sq && (e.norm_units < 1 || !(e.norm_inv_d > 0.0f))) return "a folded norm needs its unit sums and 1/d";
  if (e.bias_on && !e.bias) return "bias flag without bias";
  if (e.rg < 1) return "row group must be positive";
  return nullptr;
}

// Fills grp's problems for tiles of bm rows × bn columns (the W box: w_rows rows); false if a map fails.
template <int G>
static bool build_group(GemmGroup<G>& grp, const GemmArgs* g, int count, int bm, int bn, int a_rows, int w_rows) {
  int tile = 0;
  for (int i = 0; i < count; ++i) {
    const GemmArgs& x = g[i];
    GemmProblem& P = grp.p[i];
    if (!make_map(&P.a, x.a_hi, x.op, x.M, x.K, x.lda, a_rows) || !make_map(&P.w, x.w_hi, x.op, x.N, x.K, x.ldw, w_rows))
      return false;
    if (x.op == kOpSplit) {
      if (!make_map(&P.a2, x.a_lo, x.op, x.M, x.K, x.lda, a_rows) ||
          !make_map(&P.w2, x.w_lo, x.op, x.N, x.K, x.ldw, w_rows))
        return false;
    } else {
      P.a2 = P.a;
      P.w2 = P.w;
    }
    const int esz = (x.op == kOpBF16 || x.op == kOpF16) ? 2 : 4;
    const int bk = 128 / esz;
    P.ep = x.ep;
    P.M = x.M;
    P.N = x.N;
    P.kblks = (x.K + bk - 1) / bk;
    P.n_blks = (x.N + bn - 1) / bn;
    P.tile0 = tile;
    tile += ((x.M + bm - 1) / bm) * P.n_blks;
  }
  grp.count = count;
  grp.tiles = tile;
  return true;
}

template <int BN, int OPK, int G, bool RESID>
static cudaError_t launch_cfg_r(const GemmArgs* g, int count, cudaStream_t stream, uint32_t* err, int num_sms) {
  using C = Cfg<BN, OPK>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<BN, OPK, G, RESID>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  GemmGroup<G> grp;
  if (!build_group(grp, g, count, C::BM, BN, C::BM, BN)) return cudaErrorInvalidValue;
  const int grid = grp.tiles < num_sms ? grp.tiles : num_sms;
  gemm_tc_kernel<BN, OPK, G, RESID><<<grid, kThreads, C::SMEM, stream>>>(grp, err);
  return cudaGetLastError();
}

// A single residual GEMM (not the split mode, whose epilogue drains K slabs) runs the RESID instantiation.
template <int BN, int OPK, int G>
static cudaError_t launch_cfg(const GemmArgs* g, int count, cudaStream_t stream, uint32_t* err, int num_sms) {
  if constexpr (G == 1 && OPK != kOpSplit) {
    if (residual_preloaded(g[0].ep)) return launch_cfg_r<BN, OPK, G, true>(g, count, stream, err, num_sms);
  }
  return launch_cfg_r<BN, OPK, G, false>(g, count, stream, err, num_sms);
}

template <int OPK, int G, bool WIDE, int EPI>
static cudaError_t launch_pair_r(const GemmArgs* g, int count, cudaStream_t stream, uint32_t* err, int num_sms) {
  using C = CfgPair<OPK, WIDE, epi_slots<WIDE, EPI>()>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev & 63]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_pair_kernel<OPK, G, WIDE, EPI>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev & 63] = true;
  }
  GemmGroup<G> grp;
  if (!build_group(grp, g, count, 2 * C::BM, C::BN, C::BM, C::MMA_N / 2)) return cudaErrorInvalidValue;
  if constexpr (EPI == 2 || EPI == 4) {
    // the staged residual epilogue's 32 × 32 FP32 boxes of C_in (a2) and C (w2), and the 64 × 32 16-bit boxes of
    // a norm producer's copy of C (o2)
    const GemmArgs& x = g[0];
    if (!make_map(&grp.p[0].a2, x.ep.cin, kOpTF32, x.M, x.N, x.ep.ldcin, 32) ||
        !make_map(&grp.p[0].w2, x.ep.c, kOpTF32, x.M, x.N, x.ep.ldc, 32))
      return cudaErrorInvalidValue;
    if (EPI == 4 &&
        !make_map(&grp.p[0].o2, x.ep.o_hi, x.ep.o_kind == kOutF16 ? kOpF16 : kOpBF16, x.M, x.N, x.ep.ldo, 32))
      return cudaErrorInvalidValue;
  }
  if constexpr (EPI == 3 || EPI == 5) {
    // the staged 16-bit epilogue's 64 × 32 boxes of the q|k|v or SwiGLU output (a2) and the gate output (w2)
    const GemmArgs& x = g[0];
    const int ok = x.ep.o_kind == kOutF16 ? kOpF16 : kOpBF16;
    const int o_cols = x.ep.mode == kEpiSwiGLU ? x.N / 2 : x.ep.mode == kEpiPlain ? x.N : x.ep.n_split;
    if (!make_map(&grp.p[0].a2, x.ep.o_hi, ok, x.M, o_cols, x.ep.ldo, 32)) return cudaErrorInvalidValue;
    if (x.ep.mode == kEpiQKV && x.N > x.ep.n_split) {
      if (!make_map(&grp.p[0].w2, x.ep.g_out, ok, x.M, x.N - x.ep.n_split, x.ep.ldg, 32)) return cudaErrorInvalidValue;
    } else {
      grp.p[0].w2 = grp.p[0].a2;
    }
  }
  const int pairs = grp.tiles < num_sms / 2 ? grp.tiles : num_sms / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemm_pair_kernel<OPK, G, WIDE, EPI>, grp, err);
}

// JC_GEMM_STAGED=0 in the environment keeps residual GEMMs on the register-preloading epilogue and q|k|v|gate GEMMs
// on the general one (for comparisons).
static bool staged_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = std::getenv("JC_GEMM_STAGED");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// A residual GEMM whose C_in and C the staged epilogue can move by TMA: rows in place (no remap), 16-byte aligned
// bases and pitches.
static bool residual_staged_ok(const GemmArgs& g) {
  const EpiParams& e = g.ep;
  return staged_enabled() && residual_preloaded(e) && e.rg >= g.M && e.rg_split >= g.M && e.rg_off == 0 &&
         aligned16(e.cin) && aligned16(e.c) && e.ldcin % 4 == 0 && e.ldc % 4 == 0 && e.ldcin >= g.N &&
         e.ldc >= g.N;
}

// A q|k|v|gate GEMM whose 16-bit outputs the staged epilogue can store by TMA: 64-wide heads, the gate (if any)
// in the same 16-bit kind, rows in place, no other output, 16-byte aligned bases and pitches.
static bool qkv_staged_ok(const GemmArgs& g) {
  const EpiParams& e = g.ep;
  const bool o16 = e.o_kind == kOutF16 || e.o_kind == kOutBF16;
  const bool gate_ok = g.N == e.n_split || (e.g_out && e.g_kind == e.o_kind && aligned16(e.g_out) && e.ldg % 8 == 0);
  return staged_enabled() && e.mode == kEpiQKV && o16 && gate_ok && e.head_dim == 64 && e.n_split % 64 == 0 &&
         (g.N - e.n_split) % 64 == 0 && e.o_hi && aligned16(e.o_hi) && e.ldo % 8 == 0 && e.ldo >= e.n_split &&
         !e.c && !e.rowsq && !e.accumulate && e.rg >= g.M && e.rg_split >= g.M && e.rg_off == 0;
}

// A SwiGLU GEMM whose 16-bit output the staged epilogue can store by TMA: whole 128-column unit pairs, rows in
// place, no other output, a 16-byte aligned base and pitch.
static bool swiglu_staged_ok(const GemmArgs& g) {
  const EpiParams& e = g.ep;
  return staged_enabled() && e.mode == kEpiSwiGLU && (e.o_kind == kOutF16 || e.o_kind == kOutBF16) &&
         g.N % 128 == 0 && e.o_hi && aligned16(e.o_hi) && e.ldo % 8 == 0 && e.ldo >= g.N / 2 && !e.c && !e.rowsq &&
         !e.accumulate && e.rg >= g.M && e.rg_split >= g.M && e.rg_off == 0;
}

// A folded norm's producer the staged residual epilogue can run: a residual GEMM as above that also writes a
// 16-bit copy of C (whole 64-column units) and the per-unit Σv².
static bool residual_norm_ok(const GemmArgs& g) {
  const EpiParams& e = g.ep;
  return staged_enabled() && e.mode == kEpiPlain && e.accumulate && e.c && e.act == kActNone && !e.norm_sq &&
         e.rowsq && e.rowsq_units == g.N / 64 && g.N % 64 == 0 && (e.o_kind == kOutF16 || e.o_kind == kOutBF16) &&
         e.o_hi && aligned16(e.o_hi) && e.ldo % 8 == 0 && e.ldo >= g.N && e.rg >= g.M && e.rg_split >= g.M &&
         e.rg_off == 0 && aligned16(e.cin) && aligned16(e.c) && e.ldcin % 4 == 0 && e.ldc % 4 == 0 && e.ldcin >= g.N &&
         e.ldc >= g.N;
}

// A plain GEMM whose only output is 16-bit (an activation's output, such as an FFN's hidden layer) the staged
// epilogue can store by TMA: whole 64-column units, rows in place, a 16-byte aligned base and pitch.
static bool plain16_staged_ok(const GemmArgs& g) {
  const EpiParams& e = g.ep;
  return staged_enabled() && e.mode == kEpiPlain && (e.o_kind == kOutF16 || e.o_kind == kOutBF16) && g.N % 64 == 0 &&
         e.o_hi && aligned16(e.o_hi) && e.ldo % 8 == 0 && e.ldo >= g.N && !e.c && !e.rowsq && !e.accumulate &&
         e.rg >= g.M && e.rg_split >= g.M && e.rg_off == 0;
}

template <int OPK, int G, bool WIDE>
static cudaError_t launch_pair(const GemmArgs* g, int count, cudaStream_t stream, uint32_t* err, int num_sms) {
  if constexpr (G == 1 && !WIDE) {
    if (residual_norm_ok(g[0])) return launch_pair_r<OPK, G, WIDE, 4>(g, count, stream, err, num_sms);
  }
  if constexpr (G == 1 && OPK != kOpTF32) {
    if (qkv_staged_ok(g[0])) return launch_pair_r<OPK, G, WIDE, 3>(g, count, stream, err, num_sms);
    if (swiglu_staged_ok(g[0]) || plain16_staged_ok(g[0]))
      return launch_pair_r<OPK, G, WIDE, 5>(g, count, stream, err, num_sms);
  }
  if constexpr (G == 1) {
    if (residual_staged_ok(g[0])) return launch_pair_r<OPK, G, WIDE, 2>(g, count, stream, err, num_sms);
    if (residual_preloaded(g[0].ep)) return launch_pair_r<OPK, G, WIDE, 1>(g, count, stream, err, num_sms);
  }
  return launch_pair_r<OPK, G, WIDE, 0>(g, count, stream, err, num_sms);
}

// JC_GEMM_WIDE=0 in the environment keeps the CTA-pair kernel on 256 × 256 tiles (for comparisons).
static bool wide_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = std::getenv("JC_GEMM_WIDE");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

// JC_GEMM_PAIR=0 in the environment keeps every GEMM on the single-CTA kernel (for comparisons).
static bool pair_enabled() {
  static int on = -1;
  if (on < 0) {
    const char* v = std::getenv("JC_GEMM_PAIR");
    on = (v && v[0] == '0') ? 0 : 1;
  }
  return on == 1;
}

static int sm_count() {
  static int count[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!count[dev & 63]) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    count[dev & 63] = c > 0 ? c : 148;
  }
  return count[dev & 63];
}

// Tile widths every problem of a launch allows (bit 0: 64, bit 1: 128, bit 2: 256).
static int allowed_widths(const GemmArgs* g, int count) {
  int allowed = 15;
  for (int i = 0; i < count; ++i)
    if (g[i].ep.mode == kEpiQKV) allowed &= qkv_tile_choices(g[i].ep);
  return allowed;
}

// The widest allowed tile that still gives every SM a tile, else the narrowest (all problems of a launch
// share the tile width).
static int choose_bn(const GemmArgs* g, int count, int num_sms) {
  if (g[0].bn) return g[0].bn;
  const int allowed = allowed_widths(g, count);
  const int widths[3] = {64, 128, 256};
  for (int i = 2; i >= 0; --i)
    if ((allowed >> i) & 1) {
      long long tiles = 0;
      for (int j = 0; j < count; ++j)
        tiles += (long long)((g[j].M + 127) / 128) * ((g[j].N + widths[i] - 1) / widths[i]);
      if (tiles >= num_sms) return widths[i];
    }
  // too few tiles for the grid: the narrowest allowed tile, unless N fits one 128-wide tile
  int max_n = 0;
  for (int j = 0; j < count; ++j) max_n = g[j].N > max_n ? g[j].N : max_n;
  if (max_n <= 128 && max_n > 64 && (allowed & 2)) return 128;
  for (int i = 0; i < 3; ++i)
    if ((allowed >> i) & 1) return widths[i];
  return 256;
}

// The widest access every epilogue pointer and pitch allows: 2 = 32 bytes, 1 = 16 bytes, 0 = scalar.
static int vector_ok(const EpiParams& e) {
  auto ok = [](const void* p, long long ld, int esz, unsigned align) {
    return p == nullptr || ((reinterpret_cast<uintptr_t>(p) % align) == 0 && (ld * esz) % align == 0);
  };
  const int oesz = (e.o_kind == kOutBF16 || e.o_kind == kOutF16) ? 2 : 4;
  const int gesz = (e.g_kind == kOutBF16 || e.g_kind == kOutF16) ? 2 : 4;
  for (unsigned align : {32u, 16u}) {
    const bool all = ok(e.c, e.ldc, 4, align) && ok(e.cin, e.ldcin, 4, align) && ok(e.bias, 0, 4, align) &&
                     ok(e.o_hi, e.ldo, oesz, align) && ok(e.o_lo, e.ldo, oesz, align) &&
                     ok(e.g_out, e.ldg, gesz, align) && ok(e.rope_table, e.head_dim, 4, align);
    if (all) return align == 32u ? 2 : 1;
  }
  return 0;
}

template <int G>
static cudaError_t launch_group(GemmArgs* g, int count, cudaStream_t stream, uint32_t* err) {
  const int op = g[0].op;
  const int sms = sm_count();
  // CTA pairs for the 16-bit and TF32 modes when the 256 × 256 tiles still give every SM pair work and the
  // tile width keeps the q|k|v|gate layout whole
  const int allowed = allowed_widths(g, count);
  // 256 × 512 pair tiles for long K (≥ 2,048: the un-overlapped epilogue is then a small share of a tile; at
  // K = 1,024 it costs more than the saved operand bytes) where every problem's N is a multiple of 512 and the
  // tiles still give every SM pair one
  if (pair_enabled() && wide_enabled() && op != kOpSplit && g[0].bn == 0 && ((allowed >> 3) & 1)) {
    long long wtiles = 0;
    bool fits = true;
    for (int i = 0; i < count; ++i) {
      // (a folded norm's producer keeps 256-wide tiles, whose staged epilogue writes its 16-bit copy)
      fits = fits && g[i].N % 512 == 0 && g[i].K >= 2048 && !g[i].ep.rowsq;
      wtiles += (long long)((g[i].M + 255) / 256) * (g[i].N / 512);
    }
    if (fits && wtiles >= sms / 2) {
      switch (op) {
        case kOpBF16: return launch_pair<kOpBF16, G, true>(g, count, stream, err, sms);
        case kOpF16: return launch_pair<kOpF16, G, true>(g, count, stream, err, sms);
        default: return launch_pair<kOpTF32, G, true>(g, count, stream, err, sms);
      }
    }
  }
  if (pair_enabled() && op != kOpSplit && (g[0].bn == 0 || g[0].bn == 256) && ((allowed >> 2) & 1)) {
    long long ptiles = 0;
    for (int i = 0; i < count; ++i) ptiles += (long long)((g[i].M + 255) / 256) * ((g[i].N + 255) / 256);
    if (ptiles >= sms / 2) {
      switch (op) {
        case kOpBF16: return launch_pair<kOpBF16, G, false>(g, count, stream, err, sms);
        case kOpF16: return launch_pair<kOpF16, G, false>(g, count, stream, err, sms);
        default: return launch_pair<kOpTF32, G, false>(g, count, stream, err, sms);
      }
    }
  }
  int bn = choose_bn(g, count, sms);
  if (op == kOpSplit && bn > 128) {  // the split mode's slab buffers: 4 · BN TMEM columns
    bn = (allowed & 2) ? 128 : (allowed & 1) ? 64 : 0;
    if (!bn) return cudaErrorInvalidValue;
  }
  if (bn == 256) {
    switch (op) {
      case kOpBF16: return launch_cfg<256, kOpBF16, G>(g, count, stream, err, sms);
      case kOpTF32: return launch_cfg<256, kOpTF32, G>(g, count, stream, err, sms);
      default: return launch_cfg<256, kOpF16, G>(g, count, stream, err, sms);
    }
  }
#define JC_LAUNCH(BN_)                                                              \
  switch (op) {                                                                     \
    case kOpBF16: return launch_cfg<BN_, kOpBF16, G>(g, count, stream, err, sms);   \
    case kOpTF32: return launch_cfg<BN_, kOpTF32, G>(g, count, stream, err, sms);   \
    case kOpF16: return launch_cfg<BN_, kOpF16, G>(g, count, stream, err, sms);     \
    default: return launch_cfg<BN_, kOpSplit, G>(g, count, stream, err, sms);       \
  }
  if (bn == 128) {
    JC_LAUNCH(128)
  } else {
    JC_LAUNCH(64)
  }
#undef JC_LAUNCH
}

cudaError_t launch_gemm(const GemmArgs& gin, cudaStream_t stream, uint32_t* err) {
  if (check_gemm(gin)) return cudaErrorInvalidValue;
  GemmArgs g = gin;
  g.ep.vec_ok = vector_ok(g.ep);
  return launch_group<1>(&g, 1, stream, err);
}

const char* check_gemm_group(const GemmArgs* g, int count) {
  if (count < 1 || count > kMaxGemmGroup) return "a GEMM group holds 1 to kMaxGemmGroup problems";
  for (int i = 0; i < count; ++i) {
    if (const char* m = check_gemm(g[i])) return m;
    if (g[i].op != g[0].op) return "the problems of a GEMM group must share the operand kind";
    if (g[i].bn != g[0].bn) return "the problems of a GEMM group must share the tile width request";
  }
  return nullptr;
}

cudaError_t launch_gemm_group(const GemmArgs* gin, int count, cudaStream_t stream, uint32_t* err) {
  if (check_gemm_group(gin, count)) return cudaErrorInvalidValue;
  GemmArgs g[kMaxGemmGroup];
  for (int i = 0; i < count; ++i) {
    g[i] = gin[i];
    g[i].ep.vec_ok = vector_ok(g[i].ep);
  }
  if (count == 1) return launch_group<1>(g, 1, stream, err);
  return launch_group<kMaxGemmGroup>(g, count, stream, err);
}

}  // namespace jc

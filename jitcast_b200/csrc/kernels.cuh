// Launchers for the non-GEMM device kernels: operand conversion and packing, RMSNorm,
// token assembly, attention and the small per-family companions.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "gemm.h"

namespace jc {

// dst[r, c] (operand kind `op`, row pitch ldd) = src[r, c] for c < cols, 0 for cols <= c < ldd.
// src is fp32 with row pitch lds. For kOpSplit dst_lo receives the TF32 residual.
void launch_convert(int op, const float* src, long long lds, void* dst_hi, void* dst_lo, long long ldd, long long rows,
                    int cols, cudaStream_t s);
// The same conversion into columns 0 .. cols − 1 of each destination row only, leaving the rest of the row (the
// destination is a column block of a wider buffer).
void launch_convert_cols(int op, const float* src, long long lds, void* dst_hi, void* dst_lo, long long ldd,
                         long long rows, int cols, cudaStream_t s);

// y[r, :] = x[r, :] · rsqrt(mean(x[r, :]²) + eps) · w  for rows r, written as operand kind `op`
// (or fp32 for kOutF32). If gather_* is set, source row = (r / gather_rows) * gather_stride +
// gather_off + r % gather_rows (selects the decoder tokens of each series row).
void launch_rmsnorm(const float* x, long long ldx, const float* w, int cols, float eps, int out_kind, void* y_hi,
                    void* y_lo, long long ldy, long long rows, int gather_rows, int gather_stride, int gather_off,
                    cudaStream_t s);

// A folded RMSNorm's producer for rows t0 .. t1 − 1 of every group of n rows of x [.., cols] (cols % 64 == 0, 16-byte
// aligned rows): their 16-bit copy (kind kOutF16 or kOutBF16) into xh and their Σv² per 64-column unit into
// rowsq[row · cols / 64 + u].
void launch_norm_copy_rows(const float* x, long long ldx, int cols, int kind, void* xh, long long ldh, float* rowsq,
                           int rows, int t0, int t1, int n, cudaStream_t s);

// x[(r·n + t), :] = q for every row r and token t in [t0, t1) (the decoder tokens, a [REG] token).
void launch_fill_rows(float* x, long long ldx, const float* q, int cols, int rows, int t0, int t1, int n,
                      cudaStream_t s);

// Blocks of `threads` for `work` grid-stride items: enough to cover it, at most 16 per SM of the 148.
int grid_for(long long work, int threads);

// out[i] = in[i] + add for i < n (integer index rebasing on the device).
void launch_add_i32(const int* in, int* out, long long n, int add, cudaStream_t s);

// ---- the Timestral host ends on the device (timestral_ends.cu) ----

constexpr int kMaxQuantiles = 64;

// What the scaler, the token assembly and the quantile finish need of one shard: rows of `enc`
// patches of P steps (window W = enc·P), the context's `ll` patches, Q levels with the median at
// `median` and Quantiles.scale() in `qscale`.
struct TsEnds {
  int rows = 0, enc = 0, P = 0, ll = 0, Q = 0, median = 0, use_asinh = 0;
  float min_scale = 0.0f;
  float qscale[kMaxQuantiles] = {};
};

// Scaler.causalPatchLocScale (Scaler.instanceNorm on known rows) of every row of win/obs
// [rows · W]: frame [rows · enc] (loc, scale) per patch, row_asinh [rows] whether the row's
// affine transform takes the asinh.
void launch_ts_scaler(const float* win, const uint8_t* obs, const int* known, const TsEnds& ep, float2* frame,
                      uint8_t* row_asinh, cudaStream_t s);

// BlockPrep.tokens [rows · enc · 2P]: each patch's scaled values, then its missing flags.
void launch_ts_tokens(const float* win, const uint8_t* obs, const float2* frame, const uint8_t* row_asinh,
                      const TsEnds& ep, float* tok, cudaStream_t s);

// BlockPrep.finish in place on raw [rows · steps · Q] (steps = horizon · P): monotone levels,
// denormalised with each row's last context frame, infinities clamped.
void launch_ts_finish(float* raw, const float2* frame, const TsEnds& ep, int steps, cudaStream_t s);

// ---- the Chronos-2 host ends on the device (chronos2_ends.cu) ----

// One shard's ModelPrep / finish shape: rows of nc context and h output patches of P steps, Q levels.
struct C2Ends {
  int rows = 0, nc = 0, h = 0, P = 0, Q = 0, use_arcsinh = 0;
  float time_scale = 1.0f;
};

// InstanceNorm of every row of window [rows · nc·P] (NaN = missing): norm [rows] (loc, scale).
void launch_c2_norm(const float* window, const C2Ends& ep, float2* norm, cudaStream_t s);

// ModelPrep.tokens [rows · (nc + h) · 3P] from the window and future [rows · h·P].
void launch_c2_tokens(const float* window, const float* future, const float2* norm, const C2Ends& ep, float* tok,
                      cudaStream_t s);

// ModelPrep.finish: out [rows · Q · h·P] = sinh(raw)·scale + loc, raw [rows · h · Q · P].
void launch_c2_finish(const float* raw, const float2* norm, const C2Ends& ep, float* out, cudaStream_t s);

}  // namespace jc

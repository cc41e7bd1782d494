// Memory-bound companion kernels: operand conversion (fp32 → bf16 / TF32 / TF32 hi-lo with
// K padding), RMSNorm (optionally gathering the decoder tokens), and decoder-token fill.
// Each is a grid-stride loop sized to the SM count; one warp owns one row where a row
// reduction is needed.
#include "kernels.cuh"
#include "ptx.cuh"

namespace jc {

namespace {

__device__ __forceinline__ void put(int kind, void* hi, void* lo, long long i, float v) {
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

int out_kind_of(int op) {
  return op == kOpBF16 ? kOutBF16 : op == kOpF16 ? kOutF16 : op == kOpTF32 ? kOutTF32 : kOutSplit;
}

__global__ void convert_kernel(int kind, const float* __restrict__ src, long long lds, void* hi, void* lo,
                               long long ldd, long long rows, int cols) {
  const long long total = rows * ldd;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / ldd;
    const int c = static_cast<int>(i - r * ldd);
    put(kind, hi, lo, i, c < cols ? src[r * lds + c] : 0.0f);
  }
}

// Columns 0 .. cols − 1 of each destination row only (the destination is a column block of a wider buffer).
__global__ void convert_cols_kernel(int kind, const float* __restrict__ src, long long lds, void* hi, void* lo,
                                    long long ldd, long long rows, int cols) {
  const long long total = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / cols;
    const int c = static_cast<int>(i - r * cols);
    put(kind, hi, lo, r * ldd + c, src[r * lds + c]);
  }
}

// One warp per output row.
__global__ void rmsnorm_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w, int cols,
                               float eps, int kind, void* hi, void* lo, long long ldy, long long rows, int grows,
                               int gstride, int goff) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const long long src = grows > 0 ? (r / grows) * gstride + goff + r % grows : r;
    const float* xr = x + src * ldx;
    float ss = 0.0f;
    for (int c = lane; c < cols; c += 32) ss += xr[c] * xr[c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(ss) / cols + eps));
    for (int c = lane; c < cols; c += 32) put(kind, hi, lo, r * ldy + c, xr[c] * inv * (w ? w[c] : 1.0f));
  }
}

// One warp per row held in registers: NV float4 per lane (cols = 128·NV), one read of x, 16-byte loads.
template <int NV>
__global__ void rmsnorm_vec_kernel(const float* __restrict__ x, long long ldx, const float* __restrict__ w, float eps,
                                   int kind, void* hi, void* lo, long long ldy, long long rows, int grows, int gstride,
                                   int goff) {
  constexpr int cols = 128 * NV;
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long r = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
    const long long src = grows > 0 ? (r / grows) * gstride + goff + r % grows : r;
    const float4* xr = reinterpret_cast<const float4*>(x + src * ldx);
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = static_cast<float>(1.0 / sqrt(static_cast<double>(ss) / cols + eps));
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int c = 4 * (lane + 32 * i);
      float4 g = w ? __ldg(reinterpret_cast<const float4*>(w + c)) : make_float4(1.0f, 1.0f, 1.0f, 1.0f);
      const float y0 = v[i].x * inv * g.x, y1 = v[i].y * inv * g.y, y2 = v[i].z * inv * g.z, y3 = v[i].w * inv * g.w;
      const long long o = r * ldy + c;
      if (kind == kOutBF16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(y0, y1), b = __floats2bfloat162_rn(y2, y3);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(hi) + o) = u;
      } else if (kind == kOutF16) {
        __half2 a = __floats2half2_rn(fminf(fmaxf(y0, -65504.0f), 65504.0f), fminf(fmaxf(y1, -65504.0f), 65504.0f));
        __half2 b = __floats2half2_rn(fminf(fmaxf(y2, -65504.0f), 65504.0f), fminf(fmaxf(y3, -65504.0f), 65504.0f));
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&a);
        u.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__half*>(hi) + o) = u;
      } else {
        put(kind, hi, lo, o, y0);
        put(kind, hi, lo, o + 1, y1);
        put(kind, hi, lo, o + 2, y2);
        put(kind, hi, lo, o + 3, y3);
      }
    }
  }
}

__global__ void fill_rows_kernel(float* x, long long ldx, const float* __restrict__ q, int cols, int rows, int t0,
                                 int t1, int n) {
  const int h = t1 - t0;
  const long long total = (long long)rows * h * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int c = static_cast<int>(i % cols);
    const long long t = i / cols;
    const long long r = t / h;
    const int tok = t0 + static_cast<int>(t % h);
    x[(r * n + tok) * ldx + c] = q[c];
  }
}

// The 16-bit copy and the per-64-column-unit Σv² of rows t0 .. t1 − 1 of every group of n rows of x (a folded
// RMSNorm's producer for rows no GEMM writes): a thread per (row, unit).
__global__ void norm_copy_rows_kernel(const float* __restrict__ x, long long ldx, int units, int kind, void* xh,
                                      long long ldh, float* rowsq, int rows, int t0, int t1, int n) {
  const int h = t1 - t0;
  const long long total = (long long)rows * h * units;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int u = static_cast<int>(i % units);
    const long long t = i / units;
    const long long row = (t / h) * n + t0 + t % h;
    const float4* src = reinterpret_cast<const float4*>(x + row * ldx + 64 * u);
    float ss = 0.0f;
#pragma unroll 4
    for (int q = 0; q < 16; ++q) {
      const float4 v = src[q];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      const long long o = row * ldh + 64 * u + 4 * q;
      uint2 w;
      if (kind == kOutBF16) {
        __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
        w.x = *reinterpret_cast<uint32_t*>(&a);
        w.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(xh) + o) = w;
      } else {
        __half2 a = __floats2half2_rn(fminf(fmaxf(v.x, -65504.0f), 65504.0f), fminf(fmaxf(v.y, -65504.0f), 65504.0f));
        __half2 b = __floats2half2_rn(fminf(fmaxf(v.z, -65504.0f), 65504.0f), fminf(fmaxf(v.w, -65504.0f), 65504.0f));
        w.x = *reinterpret_cast<uint32_t*>(&a);
        w.y = *reinterpret_cast<uint32_t*>(&b);
        *reinterpret_cast<uint2*>(static_cast<__half*>(xh) + o) = w;
      }
    }
    rowsq[row * units + u] = ss;
  }
}

__global__ void add_i32_kernel(const int* __restrict__ in, int* __restrict__ out, long long n, int add) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = in[i] + add;
}

}  // namespace

int grid_for(long long work, int threads) {
  long long b = (work + threads - 1) / threads;
  const long long cap = 148LL * 16;  // 16 CTAs on each of the 148 SMs, grid-stride beyond
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

void launch_convert(int op, const float* src, long long lds, void* dst_hi, void* dst_lo, long long ldd,
                    long long rows, int cols, cudaStream_t s) {
  if (rows <= 0) return;
  convert_kernel<<<grid_for(rows * ldd, 256), 256, 0, s>>>(out_kind_of(op), src, lds, dst_hi, dst_lo, ldd, rows,
                                                           cols);
}

void launch_convert_cols(int op, const float* src, long long lds, void* dst_hi, void* dst_lo, long long ldd,
                         long long rows, int cols, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return;
  convert_cols_kernel<<<grid_for(rows * cols, 256), 256, 0, s>>>(out_kind_of(op), src, lds, dst_hi, dst_lo, ldd, rows,
                                                                 cols);
}

void launch_rmsnorm(const float* x, long long ldx, const float* w, int cols, float eps, int out_kind, void* y_hi,
                    void* y_lo, long long ldy, long long rows, int gather_rows, int gather_stride, int gather_off,
                    cudaStream_t s) {
  if (rows <= 0) return;
  // the register-resident kernel when the row is a whole number of 128-column groups and every row and the
  // weight start on a 16-byte boundary (8 bytes for the 16-bit output)
  const bool vec = cols % 128 == 0 && cols <= 1024 && ldx % 4 == 0 && ldy % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (!w || (reinterpret_cast<uintptr_t>(w) & 15) == 0) &&
                   (reinterpret_cast<uintptr_t>(y_hi) & 7) == 0;
  const int blocks = grid_for(rows * 32, 256);
  if (vec) {
    switch (cols / 128) {
#define JC_RMS_CASE(NV)                                                                                          \
  case NV:                                                                                                       \
    rmsnorm_vec_kernel<NV><<<blocks, 256, 0, s>>>(x, ldx, w, eps, out_kind, y_hi, y_lo, ldy, rows, gather_rows, \
                                                  gather_stride, gather_off);                                    \
    return;
      JC_RMS_CASE(1)
      JC_RMS_CASE(2)
      JC_RMS_CASE(3)
      JC_RMS_CASE(4)
      JC_RMS_CASE(5)
      JC_RMS_CASE(6)
      JC_RMS_CASE(7)
      JC_RMS_CASE(8)
#undef JC_RMS_CASE
      default:
        break;
    }
  }
  rmsnorm_kernel<<<blocks, 256, 0, s>>>(x, ldx, w, cols, eps, out_kind, y_hi, y_lo, ldy, rows, gather_rows,
                                        gather_stride, gather_off);
}

void launch_norm_copy_rows(const float* x, long long ldx, int cols, int kind, void* xh, long long ldh, float* rowsq,
                           int rows, int t0, int t1, int n, cudaStream_t s) {
  const long long total = (long long)rows * (t1 - t0) * (cols / 64);
  if (total <= 0) return;
  norm_copy_rows_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, ldx, cols / 64, kind, xh, ldh, rowsq, rows, t0, t1, n);
}

void launch_fill_rows(float* x, long long ldx, const float* q, int cols, int rows, int t0, int t1, int n,
                      cudaStream_t s) {
  const long long total = (long long)rows * (t1 - t0) * cols;
  if (total <= 0) return;
  fill_rows_kernel<<<grid_for(total, 256), 256, 0, s>>>(x, ldx, q, cols, rows, t0, t1, n);
}

void launch_add_i32(const int* in, int* out, long long n, int add, cudaStream_t s) {
  if (n <= 0) return;
  add_i32_kernel<<<grid_for(n, 256), 256, 0, s>>>(in, out, n, add);
}

}  // namespace jc

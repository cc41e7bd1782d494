// Element stores in a GEMM operand format (OutKind), for companion kernels whose output is the
// next GEMM's A operand: bf16, saturated f16, TF32-rounded fp32, TF32 hi + fp32 lo, or plain fp32.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "gemm.h"
#include "ptx.cuh"

namespace jc {

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

// Elements i .. i + 3 in one vector store per plane (i a multiple of 4 in a buffer whose rows are 16-byte
// aligned), rounded exactly as put_op rounds each.
__device__ __forceinline__ void put_op4(int kind, void* hi, void* lo, long long i, float4 v) {
  switch (kind) {
    case kOutBF16: {
      __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(hi) + i) =
          make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
      break;
    }
    case kOutF16: {
      auto sat = [](float x) { return fminf(fmaxf(x, -65504.0f), 65504.0f); };
      __half2 a = __floats2half2_rn(sat(v.x), sat(v.y)), b = __floats2half2_rn(sat(v.z), sat(v.w));
      *reinterpret_cast<uint2*>(static_cast<__half*>(hi) + i) =
          make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
      break;
    }
    case kOutTF32:
      *reinterpret_cast<float4*>(static_cast<float*>(hi) + i) =
          make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
      break;
    case kOutSplit: {
      const float4 h = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
      *reinterpret_cast<float4*>(static_cast<float*>(hi) + i) = h;
      *reinterpret_cast<float4*>(static_cast<float*>(lo) + i) = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      break;
    }
    default: *reinterpret_cast<float4*>(static_cast<float*>(hi) + i) = v; break;
  }
}

}  // namespace jc

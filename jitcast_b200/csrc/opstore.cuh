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

}  // namespace jc

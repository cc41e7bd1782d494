// C-ABI entry point of the op-level time attention (the companion kernel of the Timestral and Chronos-2
// forwards): TimestralKernels.timeAttention (timestral/tornado/TimestralKernels.java:114) with the
// BlockLayout masks, and Chronos2Kernels.timeAttention (chronos2/tornado/Chronos2Kernels.java:130) over
// live keys, on device buffers.
#include <string>

#include "attention.cuh"
#include "runtime.h"

using namespace jc;

extern "C" {

jc_status jc_time_attention_device(int device, jc_precision precision, const void* qkv, long long ld_qkv,
                                   const void* gate, long long ld_gate, void* out, long long ld_out, int rows, int n,
                                   int heads, int head_dim, int d, float scale, int mask_mode, int enc, int ll,
                                   const int32_t* key_valid, const int32_t* known, const int32_t* live, int flags,
                                   void* stream) {
  clear_error();
  if (precision != JC_FP32 && precision != JC_TF32 && precision != JC_BF16 && precision != JC_FP16)
    return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (rows < 0 || n < 1 || heads < 1 || d != heads * head_dim || ld_qkv < 3LL * d || ld_out < d ||
      (gate && ld_gate < d))
    return fail(JC_ERR_INVALID_ARG, "inconsistent attention shape");
  if (head_dim != 32 && head_dim != 64) return fail(JC_ERR_UNSUPPORTED_SHAPE, "head_dim must be 32 or 64");
  if (!qkv || !out) return fail(JC_ERR_INVALID_ARG, "null qkv or output");
  if (flags & ~JC_ATTN_CUDA_CORES) return fail(JC_ERR_INVALID_ARG, "unknown attention flags");
  if (mask_mode == 0) {
    if (enc < 0 || enc > n || ll < 0 || ll > enc || (enc > 0 && !key_valid) || !known)
      return fail(JC_ERR_INVALID_ARG, "mask mode 0 needs 0 <= ll <= enc <= n, key_valid and known");
  } else if (mask_mode == 1) {
    if (!live) return fail(JC_ERR_INVALID_ARG, "mask mode 1 needs live");
  } else {
    return fail(JC_ERR_INVALID_ARG, "mask_mode must be 0 or 1");
  }
  std::string why;
  DeviceRt* rt = device_rt(device, &why);
  if (!rt) return fail(JC_ERR_NO_DEVICE, why);
  std::lock_guard<std::mutex> lk(rt->mu);
  if (cudaSetDevice(device) != cudaSuccess) return fail(JC_ERR_CUDA, "cannot select the device");
  const int kind = precision == JC_BF16 ? kOutBF16 : precision == JC_FP16 ? kOutF16 : kOutF32;
  AttnArgs a{};
  a.qkv = qkv;
  a.qkv_kind = kind;
  a.ld_qkv = ld_qkv;
  a.gate = gate;
  a.gate_kind = kind;
  a.ld_gate = ld_gate;
  a.out_hi = out;
  a.ld_out = ld_out;
  a.out_kind = kind;
  a.rows = rows;
  a.n = n;
  a.enc = mask_mode == 0 ? enc : n;
  a.ll = mask_mode == 0 ? ll : n;
  a.heads = heads;
  a.head_dim = head_dim;
  a.d = d;
  a.scale = scale;
  a.key_valid = key_valid;
  a.known = known;
  a.mask_mode = mask_mode;
  a.live = live;
  a.err = rt->err;
  a.cuda_cores = (flags & JC_ATTN_CUDA_CORES) ? 1 : 0;
  const cudaError_t e = launch_time_attention(a, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail_cuda(e, "time attention launch");
  return JC_OK;
}

}  // extern "C"

// Attention companion kernels (time and variate attention with the block-layout masks).
#pragma once

#include <cuda_runtime.h>

#include "gemm.h"

namespace jc {

struct AttnArgs {
  const void* qkv;  // [rows·n, ld_qkv]: q | k | v, heads-major (head h at columns h·dh within each part)
  int qkv_kind;     // qkv element type: kOutF32, kOutBF16 or kOutF16
  long long ld_qkv;
  const void* gate;  // [rows·n, ld_gate] sigmoid gate multiplied into the output, or null
  int gate_kind;    // kOutF32, kOutBF16 or kOutF16
  long long ld_gate;
  void* out_hi;  // [rows·n, ld_out] in OutKind out_kind
  void* out_lo;
  long long ld_out;
  int out_kind;
  int rows, n, enc, ll, heads, head_dim, d;
  float scale;  // applied to q·k
  const int* key_valid;  // [rows·enc]
  const int* known;      // [rows]
  const int* role;       // [rows]
  const int* group_start;
  const int* group_end;
  int covariates;
  // 0: the Timestral block layout (key_valid, known, enc, ll; variate rows always read themselves);
  // 1: per-token liveness (live [rows·n]): every live key of the row in time attention, the live
  //    rows of the group in group attention, zeros when a group has none (Chronos-2's ModelLayout).
  int mask_mode;
  const int* live;
  uint32_t* err;  // device error word: bounded waits of the tensor-core kernel that gave up, or null
  int cuda_cores;  // 1: the FP32-math CUDA-core kernel even where the tensor-core kernels apply
};

cudaError_t launch_time_attention(const AttnArgs& a, cudaStream_t s);

// The tcgen05 time attention (attention_tc.cu): 16-bit q/k/v of 64-wide heads, ≤ 256 tokens per row.
bool time_attention_tc_ok(const AttnArgs& a);
cudaError_t launch_time_attention_tc(const AttnArgs& a, cudaStream_t s);
cudaError_t launch_variate_attention(const AttnArgs& a, cudaStream_t s);

}  // namespace jc

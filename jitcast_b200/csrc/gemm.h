// The tcgen05 GEMM engine's host-visible types: operand kinds, the fused-epilogue
// parameters and the launch entry. C[m, n] (+)= act(A[m, :]·W[n, :] + b[n]) with A [M, K]
// and W [N, K] both K-major (PyTorch [out, in] weights), the accumulator in TMEM.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace jc {

// How GEMM operands are stored in HBM.
enum OperandKind : int {
  kOpBF16 = 0,   // bfloat16; tcgen05 kind::f16
  kOpTF32 = 1,   // fp32 container rounded to TF32; kind::tf32
  kOpSplit = 2,  // fp32 as a TF32 hi/lo pair; four kind::tf32 MMAs (lo·lo + lo·hi + hi·lo + hi·hi)
  kOpF16 = 3,    // IEEE half; tcgen05 kind::f16
};

// How an epilogue writes its operand-typed copy of the result.
enum OutKind : int {
  kOutNone = 0,
  kOutBF16 = 1,
  kOutTF32 = 2,   // fp32, rounded to TF32
  kOutSplit = 3,  // fp32 hi (TF32) and lo (residual) buffers
  kOutF32 = 4,    // fp32, unrounded
  kOutF16 = 5,    // IEEE half, saturated to ±65504
};

// kActSiluRelu is the reference's SILU|RELU flag pair: ReLU(SiLU(v)).
enum Activation : int { kActNone = 0, kActSilu = 1, kActRelu = 2, kActGelu = 3, kActSigmoid = 4, kActSiluRelu = 5 };

enum EpiMode : int {
  kEpiPlain = 0,
  // Output columns come in 32-column pairs (silu half, linear half); writes N/2 columns of
  // SiLU(first)·second to the operand output.
  kEpiSwiGLU = 1,
  // Fused q|k|v|gate projection: RoPE on columns < rope_cols (per head of head_dim, pairs
  // e and e + head_dim/2), columns >= n_split go through a sigmoid to the gate output.
  kEpiQKV = 2,
};

// Flags, as the reference's Kernels.gemm (BIAS=1, ACCUMULATE=2, SILU=4, RELU=16) plus GELU=32.
constexpr int kFlagBias = 1;
constexpr int kFlagAccumulate = 2;
constexpr int kFlagSilu = 4;
constexpr int kFlagTwinOnly = 8;
constexpr int kFlagRelu = 16;
constexpr int kFlagGelu = 32;

struct EpiParams {
  int mode;        // EpiMode
  int act;         // Activation, applied after the bias
  int bias_on;
  int accumulate;  // C = C_in + act(...)
  const float* bias;
  float* c;        // fp32 output, row-remapped; may be null
  long long ldc;
  const float* cin;  // residual input for accumulate (usually == c)
  long long ldcin;
  void* o_hi;      // operand-typed output (OutKind); o_lo only for kOutSplit
  void* o_lo;
  long long ldo;
  int o_kind;
  // Row remap of the outputs: out_row = (r / rg) * rg_stride + r % rg + rg_off, plus rg_shift when
  // r % rg >= rg_split (places embedded tokens around inserted ones, e.g. a [REG] token).
  int rg, rg_stride, rg_off, rg_split, rg_shift;
  // kEpiQKV
  int rope_cols, head_dim;
  // pairs (e, e + head_dim/2) with a nonzero frequency, e < rope_pairs; 0 = all. A partial rotary factor
  // leaves the other pairs at cos 1, sin 0 — the identity — so the epilogue neither loads nor applies them.
  int rope_pairs;
  const int* pos;           // [M] index into rope_table rows
  const float* rope_table;  // [positions, head_dim]: cos at e, sin at head_dim/2 + e
  // Optional, with rope_pairs ≤ 16: the same values packed [positions, 32]: cos of pairs 0..15, then their sin
  // (zeros past rope_pairs). The staged epilogue reads a warp's 32 consecutive positions as one 4 KB block.
  const float* rope_pack;
  int n_split;
  void* g_out;  // gate output (sigmoid) in OutKind g_kind: kOutF32, kOutBF16 or kOutF16
  long long ldg;
  int g_kind;
  // A folded RMSNorm. Its producer (the GEMM that writes the residual stream x) stores, besides x, the Σ of the
  // squares of the FP32 output over each 64-column unit u: rowsq[out_row · rowsq_units + u] (optional). Its
  // consumer (the next GEMM, whose A is x's 16-bit copy and whose W holds the norm's weights) scales each output
  // row by 1 / sqrt(Σ_u norm_sq[row · norm_units + u] · norm_inv_d + norm_eps) before the bias (optional).
  float* rowsq;
  int rowsq_units;
  const float* norm_sq;
  int norm_units;
  float norm_inv_d, norm_eps;
  int vec_ok;  // all output pointers / leading dims allow 16-byte vector access
};

struct GemmArgs {
  int op;  // OperandKind
  const void* a_hi;
  const void* a_lo;
  long long lda;  // elements
  const void* w_hi;
  const void* w_lo;
  long long ldw;
  int M, N, K;
  int bn;  // 0 = choose
  EpiParams ep;
};

// Returns a zero-initialised EpiParams with the identity row remap.
EpiParams epi_default();

// Launches one GEMM on `stream`. `err` is a device word the kernel ORs error bits into.
// Returns cudaSuccess or the launch error; shape errors are reported as cudaErrorInvalidValue.
cudaError_t launch_gemm(const GemmArgs& g, cudaStream_t stream, uint32_t* err);

// Checks the alignment and shape rules of launch_gemm; returns nullptr or a message.
const char* check_gemm(const GemmArgs& g);

// Up to kMaxGemmGroup independent GEMMs of one operand kind as ONE persistent launch: the tiles of every
// problem in one walk over the SMs, each tile with its own problem's operands, shape and epilogue. For GEMMs
// that could run in any order (a headwise projection's heads; two projections of one input), it saves the
// launches, the grid tails and the prologues of all but one. Results equal separate launch_gemm calls.
constexpr int kMaxGemmGroup = 4;
cudaError_t launch_gemm_group(const GemmArgs* g, int count, cudaStream_t stream, uint32_t* err);
const char* check_gemm_group(const GemmArgs* g, int count);

// A 2-D TMA tensor map over a row-major [rows, k] matrix of operand kind `op` (row pitch `ld`
// elements): 128-byte swizzle, box = 128 bytes of a row × box_rows rows, zero fill past the edges.
// The layout the tcgen05 K-major (and, for 64 16-bit columns, MN-major) operand descriptors read.
bool make_operand_map(CUtensorMap* map, const void* base, int op, long long rows, long long k, long long ld,
                      int box_rows);

}  // namespace jc

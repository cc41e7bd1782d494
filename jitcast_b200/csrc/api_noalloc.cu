// jc_linear_device_noalloc: the device-buffer GEMM of jc_linear_device for callers that must not
// allocate GPU memory after start-up — for example a host that hands the whole GPU to a
// pre-sized arena or a fixed memory budget, where a cudaMalloc can fail or stall mid-stream, or code
// that must stay away from cudaMalloc/cudaFree because they can synchronise the whole device.
//
// The operand conversions that jc_linear_device writes into grown-on-demand library scratch go
// instead into one fixed array in the library's own device image (kNoAllocScratchBytes per GPU,
// present on every GPU that loads the library, until the process exits). Nothing here calls
// cudaMalloc, cudaFree or a library routine that allocates. Under CUDA's lazy module loading (the
// default since CUDA 12.2) the array is reserved on a device when the library's module is first
// loaded there, which the first call on that device does (or any earlier call of the library on it).
#include <mutex>
#include <string>

#include "gemm.h"
#include "kernels.cuh"
#include "runtime.h"

namespace {

// The fixed scratch: A then W in the precision's operand format (hi, plus lo for JC_FP32),
// K padded to 64 elements, each part 256-byte aligned.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
// Bounded-wait failures of the kernels launched by this entry point.
static __device__ __align__(16) uint32_t g_noalloc_err[4];

// Device addresses of the two symbols, looked up once per device with that device current. In
// host code the symbols' names are host-side stand-ins, not device addresses.
// One lock per device: calls on one device share that device's copy of the array and are serialised;
// calls on different devices use different copies and run side by side.
struct Addresses {
  std::mutex mu;
  bool ready = false;
  unsigned char* scratch = nullptr;
  uint32_t* err = nullptr;
};
Addresses g_addr[64];

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace

using namespace jc;

extern "C" jc_status jc_linear_device_noalloc(int device, jc_precision precision, const float* a, long long lda,
                                              const float* w, long long ldw, const float* bias, float* c,
                                              long long ldc, int m, int n, int k, int flags, void* stream) {
  clear_error();
  if (precision != JC_FP32 && precision != JC_TF32 && precision != JC_BF16 && precision != JC_FP16)
    return fail(JC_ERR_INVALID_ARG, "unknown precision");
  if (m < 1 || n < 1 || k < 1) return fail(JC_ERR_INVALID_ARG, "m, n and k must be positive");
  if (!a || !w || !c) return fail(JC_ERR_INVALID_ARG, "null buffer");
  if ((flags & JC_BIAS) && !bias) return fail(JC_ERR_INVALID_ARG, "JC_BIAS without a bias");
  if (lda < k || ldw < k || ldc < n) return fail(JC_ERR_INVALID_ARG, "leading dimension smaller than the row");
  const int known = JC_BIAS | JC_ACCUMULATE | JC_SILU | JC_RELU | JC_GELU;
  if (flags & ~known) return fail(JC_ERR_INVALID_ARG, "unsupported flag bits " + std::to_string(flags & ~known));
  const bool silu = flags & JC_SILU, relu = flags & JC_RELU, gelu = flags & JC_GELU;
  if (gelu && (silu || relu)) return fail(JC_ERR_INVALID_ARG, "JC_GELU cannot be combined with JC_SILU or JC_RELU");
  const int act = silu && relu ? kActSiluRelu : silu ? kActSilu : relu ? kActRelu : gelu ? kActGelu : kActNone;

  const int op = precision == JC_BF16   ? kOpBF16
                 : precision == JC_FP16 ? kOpF16
                 : precision == JC_TF32 ? kOpTF32
                                        : kOpSplit;
  const long long kp = round_up(k, 64);
  const size_t esz = (op == kOpBF16 || op == kOpF16) ? 2 : 4;
  // refuse before multiplying: m · kp · esz could wrap size_t when m and k are both near INT_MAX
  if (static_cast<size_t>(kp) > kNoAllocScratchBytes / esz / static_cast<size_t>(m > n ? m : n))
    return fail(JC_ERR_UNSUPPORTED_SHAPE,
                "jc_linear_device_noalloc: the operands of a " + std::to_string(m) + " x " + std::to_string(n) +
                    " x " + std::to_string(k) + " GEMM do not fit the fixed scratch of " +
                    std::to_string(kNoAllocScratchBytes) + " bytes");
  const size_t a_part = align256(static_cast<size_t>(m) * kp * esz);
  const size_t w_part = align256(static_cast<size_t>(n) * kp * esz);
  const size_t parts = op == kOpSplit ? 2 : 1;
  const size_t need = parts * (a_part + w_part);
  if (need > kNoAllocScratchBytes)
    return fail(JC_ERR_UNSUPPORTED_SHAPE,
                "jc_linear_device_noalloc: (m + n) x round_up(k, 64) operands need " + std::to_string(need) +
                    " bytes of scratch; the fixed scratch holds " + std::to_string(kNoAllocScratchBytes));

  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return fail(JC_ERR_NO_DEVICE, "no CUDA device");
  }
  if (device < 0 || device >= count || device >= 64) return fail(JC_ERR_NO_DEVICE, "device out of range");

  Addresses& ad = g_addr[device];
  std::lock_guard<std::mutex> lk(ad.mu);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return fail_cuda(e, "cudaSetDevice");
  if (!ad.ready) {
    // first call on this device: resolve the symbols' device addresses (make this first call
    // before any stream capture that would include the entry point)
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(scratch)");
    ad.scratch = static_cast<unsigned char*>(p);
    e = cudaGetSymbolAddress(&p, g_noalloc_err);
    if (e != cudaSuccess) return fail_cuda(e, "cudaGetSymbolAddress(error word)");
    ad.err = static_cast<uint32_t*>(p);
    ad.ready = true;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* base = ad.scratch;
  void* a_hi = base;
  void* w_hi = base + a_part;
  void* a_lo = op == kOpSplit ? base + a_part + w_part : nullptr;
  void* w_lo = op == kOpSplit ? base + 2 * a_part + w_part : nullptr;

  GemmArgs g{};
  g.op = op;
  g.a_hi = a_hi;
  g.a_lo = a_lo;
  g.lda = kp;
  g.w_hi = w_hi;
  g.w_lo = w_lo;
  g.ldw = kp;
  g.M = m;
  g.N = n;
  g.K = k;
  g.ep = epi_default();
  g.ep.act = act;
  g.ep.bias_on = (flags & JC_BIAS) != 0;
  g.ep.bias = bias;
  g.ep.accumulate = (flags & JC_ACCUMULATE) != 0;
  g.ep.c = c;
  g.ep.ldc = ldc;
  g.ep.cin = c;
  g.ep.ldcin = ldc;
  // every check comes before the first launch, so a refused call leaves the stream untouched
  if (const char* msg = check_gemm(g)) return fail(JC_ERR_UNSUPPORTED_SHAPE, msg);

  // the conversions write every element of the padded operands (zeros past k), so nothing left in
  // the shared scratch by an earlier call is read
  launch_convert(op, a, lda, a_hi, a_lo, kp, m, k, s);
  launch_convert(op, w, ldw, w_hi, w_lo, kp, n, k, s);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail_cuda(e, "operand conversion launch");
  e = cudaMemsetAsync(ad.err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return fail_cuda(e, "clearing the error word");
  e = launch_gemm(g, s, ad.err);
  if (e != cudaSuccess) return fail_cuda(e, "GEMM launch");
  // the scratch is reused by the next call, so the call completes before returning; the word
  // then tells whether a bounded wait inside the kernel gave up
  uint32_t word = 0;
  e = cudaMemcpyAsync(&word, ad.err, sizeof(uint32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail_cuda(e, "jc_linear_device_noalloc");
  if (word) return fail(JC_ERR_TIMEOUT, "a device wait gave up (error bits " + std::to_string(word) + ")");
  return JC_OK;
}

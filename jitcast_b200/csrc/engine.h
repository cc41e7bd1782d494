// Engine infrastructure shared by the model families: device allocations, operand-format
// matrices, strict name/shape binding of host weights, weight packing onto a device, and the
// per-device slot (stream, error word, plan cache) a forward runs on.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <functional>
#include <list>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <string>
#include <vector>

#include "../../include/jitcast_b200.h"
#include "gemm.h"

namespace jc {

// cudaMalloc'd blocks owned together and freed on destruction.
class DeviceMem {
 public:
  DeviceMem() = default;
  DeviceMem(const DeviceMem&) = delete;
  DeviceMem& operator=(const DeviceMem&) = delete;
  ~DeviceMem() { release(); }
  void* alloc(size_t bytes);  // 256-byte aligned; nullptr on failure (the error is left set)
  void release();
  size_t bytes() const { return total_; }

 private:
  std::vector<void*> ptrs_;
  size_t total_ = 0;
};

// A row-major matrix in a GEMM operand format (hi, plus lo for the split FP32 mode).
struct OpBuf {
  void* hi = nullptr;
  void* lo = nullptr;
  long long ld = 0;
  long long rows = 0;
};

// A packed linear layer on one device: W [out, in] in the operand format, bias fp32 or null.
struct DevLinear {
  OpBuf w;
  float* bias = nullptr;
  int in = 0, out = 0;
};

inline int op_of_precision(jc_precision p) {
  return p == JC_BF16 ? kOpBF16 : p == JC_FP16 ? kOpF16 : p == JC_TF32 ? kOpTF32 : kOpSplit;
}
inline int out_of_op(int op) {
  return op == kOpBF16 ? kOutBF16 : op == kOpF16 ? kOutF16 : op == kOpTF32 ? kOutTF32 : kOutSplit;
}
inline size_t op_esize(int op) { return (op == kOpBF16 || op == kOpF16) ? 2 : 4; }
inline bool op_is_16bit(int op) { return op == kOpBF16 || op == kOpF16; }
inline bool valid_precision_code(int p) { return p == JC_FP32 || p == JC_TF32 || p == JC_BF16 || p == JC_FP16; }

// Allocates an operand buffer of rows × round_up(cols, 64) elements.
// Rows a plan is built for: `x` itself up to 8, then the next multiple of a quarter of its power of two, so
// padding adds at most 25 % and the number of shapes grows with the logarithm of the size (the reference's
// bucket, TimestralForward.java:88-99).
int bucket_rows(int x);

bool alloc_op(DeviceMem& mem, int op, long long rows, long long cols, OpBuf* out);

// Host weights by name with strict binding: every tensor must be taken exactly once, with the
// expected shape (the reference's TimestralWeights.Binder, TimestralWeights.java:184-224).
class Binder {
 public:
  Binder(const jc_tensor_view* views, int n);
  // Returns the data of `name` with exactly `shape`; records an error and returns nullptr otherwise.
  const float* take(const std::string& name, std::initializer_list<long long> shape);
  const float* take_optional(const std::string& name, std::initializer_list<long long> shape);
  bool has(const std::string& name) const { return by_name_.count(name) != 0; }
  // Fails if some tensor was never bound.
  bool require_all_bound();
  const std::string& error() const { return error_; }
  bool ok() const { return error_.empty(); }

 private:
  std::map<std::string, const jc_tensor_view*> by_name_;
  std::set<std::string> bound_;
  std::string error_;
  bool duplicate_ = false;
};

// Uploads a host fp32 matrix [rows, cols] (row pitch cols) to an operand buffer on the current
// device (via a temporary fp32 copy and the conversion kernel). Synchronous.
bool upload_op(DeviceMem& mem, int op, const float* host, long long rows, long long cols, OpBuf* out,
               std::string* err);
float* upload_f32(DeviceMem& mem, const float* host, size_t count, std::string* err);
int* upload_i32(DeviceMem& mem, const int* host, size_t count, std::string* err);

// A linear layer from host W [out, in] (already rearranged) and optional bias.
bool upload_linear(DeviceMem& mem, int op, const float* w, const float* b, int in, int out, DevLinear* lin,
                   std::string* err);

// GEMM arguments for C = epilogue(A · Wᵀ) with A in `a` (rows m) and W from `lin`.
GemmArgs gemm_args(int op, const OpBuf& a, long long m, const DevLinear& lin);

// CUDA-event timing of kernel classes, for the "profile" engine option. Launches are bracketed by
// begin/end on the launching stream; collect() (after a synchronise) sums them per class.
class Profiler {
 public:
  bool on = false;
  ~Profiler();
  void begin(cudaStream_t s, const char* name, double flops);
  void end(cudaStream_t s);
  void collect();
  struct Acc {
    double ms = 0, flops = 0;
    long long launches = 0;
  };
  std::map<std::string, Acc> totals;

 private:
  struct Rec {
    const char* name;
    cudaEvent_t a, b;
    double flops;
  };
  std::vector<Rec> pending_;
  std::vector<cudaEvent_t> pool_;
  cudaEvent_t take();
};

// The device slot an engine owns on one GPU.
struct DeviceSlot {
  int device = 0;
  int slot = 0;  // its index among the engine's slots (two slots may share a GPU)
  cudaStream_t stream = nullptr;
  uint32_t* err = nullptr;
  DeviceMem weights;
  ~DeviceSlot();
};

// Splits `rows` into `parts` contiguous ranges that never cut a series (group_end[] gives each
// row's series end), as even as the series allow. Returns the range starts plus `rows`.
std::vector<int> shard_rows(int rows, const int* group_start, const int* group_end, int parts);

// A CUDA graph of one enqueue function, captured on first replay after an eager warm-up run.
struct GraphRunner {
  cudaGraphExec_t exec = nullptr;
  bool warmed = false;
  ~GraphRunner();
  // Runs `enqueue` on `s`: eagerly the first time, as a captured graph afterwards.
  cudaError_t run(cudaStream_t s, const std::function<cudaError_t(cudaStream_t)>& enqueue, bool use_graph);
};

}  // namespace jc

// The opaque engine handle of the C ABI: one model family's weights on its GPUs.
struct jc_engine {
  virtual ~jc_engine() = default;
  int family = 0;  // 1 Timestral, 2 Chronos-2, 3 TiRex-2
  std::mutex mu;   // serialises calls, as PlanCache.run holds its lock for the whole call
  bool use_graph = true;
  int max_plans = 8;
  bool profile = false;
  bool buckets = true;  // plans (and graphs) for bucketed row counts
  // Host-side failure injection (engine options "fail_plan_allocs" and "fail_slot"): the next N plan allocations
  // report out of memory, and the next forward's shard on slot fail_slot fails before it enqueues anything.
  // Shards of one call run on parallel host threads, hence the atomics.
  std::atomic<int> fail_plan_allocs{0};
  std::atomic<int> fail_slot{-1};
  bool take_plan_failure() {
    int n = fail_plan_allocs.load();
    while (n > 0)
      if (fail_plan_allocs.compare_exchange_weak(n, n - 1)) return true;
    return false;
  }
  bool take_slot_failure(int slot) {
    int s = slot;
    return fail_slot.compare_exchange_strong(s, -1);
  }
  virtual int slots() const = 0;
  virtual jc::DeviceSlot* slot(int i) = 0;
  virtual jc::Profiler* profiler(int i) = 0;
  virtual void drop_plans() = 0;
};

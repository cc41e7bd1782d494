// Engine infrastructure: device allocations, strict weight binding, weight packing, row
// sharding and CUDA-graph replay.
#include "engine.h"

#include <algorithm>
#include <cstring>

#include "kernels.cuh"
#include "runtime.h"

namespace jc {

void* DeviceMem::alloc(size_t bytes) {
  void* p = nullptr;
  const size_t b = static_cast<size_t>(round_up(static_cast<long long>(bytes ? bytes : 1), 256));
  if (cudaMalloc(&p, b) != cudaSuccess) return nullptr;
  ptrs_.push_back(p);
  total_ += b;
  return p;
}

void DeviceMem::release() {
  for (void* p : ptrs_) cudaFree(p);
  ptrs_.clear();
  total_ = 0;
}

int bucket_rows(int x) {
  if (x <= 8) return x;
  int hb = 1;
  while (hb <= (x - 1) / 2) hb *= 2;  // the highest power of two ≤ x − 1
  const int step = hb / 4;
  return (x + step - 1) / step * step;
}

bool alloc_op(DeviceMem& mem, int op, long long rows, long long cols, OpBuf* out) {
  out->ld = round_up(cols, 64);
  out->rows = rows;
  const size_t bytes = static_cast<size_t>(rows * out->ld) * op_esize(op);
  out->hi = mem.alloc(bytes);
  out->lo = op == kOpSplit ? mem.alloc(bytes) : nullptr;
  return out->hi && (op != kOpSplit || out->lo);
}

Binder::Binder(const jc_tensor_view* views, int n) {
  for (int i = 0; i < n; ++i) {
    const std::string name = views[i].name ? views[i].name : "";
    if (by_name_.count(name)) {
      error_ = "tensor " + name + " given twice";
      duplicate_ = true;
    }
    by_name_[name] = &views[i];
  }
}

static std::string shape_str(const long long* s, int n) {
  std::string r = "[";
  for (int i = 0; i < n; ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

const float* Binder::take(const std::string& name, std::initializer_list<long long> shape) {
  if (!error_.empty()) return nullptr;
  auto it = by_name_.find(name);
  if (it == by_name_.end()) {
    error_ = "checkpoint has no tensor " + name;
    return nullptr;
  }
  if (!bound_.insert(name).second) {
    error_ = name + " bound twice";
    return nullptr;
  }
  const jc_tensor_view* v = it->second;
  std::vector<long long> want(shape);
  bool same = v->ndim == static_cast<int>(want.size());
  for (size_t i = 0; same && i < want.size(); ++i) same = v->shape[i] == want[i];
  if (!same) {
    long long got[4] = {0, 0, 0, 0};
    for (int i = 0; i < v->ndim && i < 4; ++i) got[i] = v->shape[i];
    error_ = name + " has shape " + shape_str(got, v->ndim) + ", expected " +
             shape_str(want.data(), static_cast<int>(want.size()));
    return nullptr;
  }
  if (!v->data) {
    error_ = name + " has no data";
    return nullptr;
  }
  return v->data;
}

const float* Binder::take_optional(const std::string& name, std::initializer_list<long long> shape) {
  return has(name) ? take(name, shape) : nullptr;
}

bool Binder::require_all_bound() {
  if (!error_.empty()) return false;
  std::string extra;
  for (auto& kv : by_name_)
    if (!bound_.count(kv.first)) extra += (extra.empty() ? "" : ", ") + kv.first;
  if (!extra.empty()) {
    error_ = "unexpected tensors in checkpoint: [" + extra + "]";
    return false;
  }
  return true;
}

bool upload_op(DeviceMem& mem, int op, const float* host, long long rows, long long cols, OpBuf* out,
               std::string* err) {
  if (!alloc_op(mem, op, rows, cols, out)) {
    *err = "out of device memory for weights";
    return false;
  }
  float* tmp = nullptr;
  cudaError_t e = cudaMalloc(&tmp, sizeof(float) * rows * cols);
  if (e == cudaSuccess) e = cudaMemcpy(tmp, host, sizeof(float) * rows * cols, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    launch_convert(op, tmp, cols, out->hi, out->lo, out->ld, rows, static_cast<int>(cols), nullptr);
    e = cudaDeviceSynchronize();
  }
  if (tmp) cudaFree(tmp);
  if (e != cudaSuccess) {
    *err = std::string("weight upload: ") + cudaGetErrorString(e);
    return false;
  }
  return true;
}

float* upload_f32(DeviceMem& mem, const float* host, size_t count, std::string* err) {
  float* p = static_cast<float*>(mem.alloc(sizeof(float) * count));
  if (!p) {
    *err = "out of device memory";
    return nullptr;
  }
  if (cudaMemcpy(p, host, sizeof(float) * count, cudaMemcpyHostToDevice) != cudaSuccess) {
    *err = "upload failed";
    return nullptr;
  }
  return p;
}

int* upload_i32(DeviceMem& mem, const int* host, size_t count, std::string* err) {
  int* p = static_cast<int*>(mem.alloc(sizeof(int) * count));
  if (!p) {
    *err = "out of device memory";
    return nullptr;
  }
  if (cudaMemcpy(p, host, sizeof(int) * count, cudaMemcpyHostToDevice) != cudaSuccess) {
    *err = "upload failed";
    return nullptr;
  }
  return p;
}

bool upload_linear(DeviceMem& mem, int op, const float* w, const float* b, int in, int out, DevLinear* lin,
                   std::string* err) {
  lin->in = in;
  lin->out = out;
  if (!upload_op(mem, op, w, out, in, &lin->w, err)) return false;
  lin->bias = nullptr;
  if (b && !(lin->bias = upload_f32(mem, b, out, err))) return false;
  return true;
}

GemmArgs gemm_args(int op, const OpBuf& a, long long m, const DevLinear& lin) {
  GemmArgs g{};
  g.op = op;
  g.a_hi = a.hi;
  g.a_lo = a.lo;
  g.lda = a.ld;
  g.w_hi = lin.w.hi;
  g.w_lo = lin.w.lo;
  g.ldw = lin.w.ld;
  g.M = static_cast<int>(m);
  g.N = lin.out;
  g.K = lin.in;
  g.ep = epi_default();
  if (lin.bias) {
    g.ep.bias_on = 1;
    g.ep.bias = lin.bias;
  }
  return g;
}

DeviceSlot::~DeviceSlot() {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  if (stream) cudaStreamDestroy(stream);
  if (err) cudaFree(err);
  weights.release();
  cudaSetDevice(prev);
}

std::vector<int> shard_rows(int rows, const int* group_start, const int* group_end, int parts) {
  std::vector<int> cuts{0};
  for (int p = 1; p < parts; ++p) {
    int target = static_cast<int>((static_cast<long long>(rows) * p) / parts);
    if (target <= cuts.back()) target = cuts.back();
    // move the cut to the nearest series boundary at or after the target
    int c = target;
    if (c > 0 && c < rows && group_start[c] != c) c = group_end[c];
    if (c > rows) c = rows;
    cuts.push_back(std::max(c, cuts.back()));
  }
  cuts.push_back(rows);
  return cuts;
}

Profiler::~Profiler() {
  for (auto& r : pending_) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (cudaEvent_t e : pool_) cudaEventDestroy(e);
}

cudaEvent_t Profiler::take() {
  if (!pool_.empty()) {
    cudaEvent_t e = pool_.back();
    pool_.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

void Profiler::begin(cudaStream_t s, const char* name, double flops) {
  if (!on) return;
  Rec r{name, take(), take(), flops};
  cudaEventRecord(r.a, s);
  pending_.push_back(r);
}

void Profiler::end(cudaStream_t s) {
  if (!on || pending_.empty()) return;
  cudaEventRecord(pending_.back().b, s);
}

void Profiler::collect() {
  for (auto& r : pending_) {
    float ms = 0;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      Acc& a = totals[r.name];
      a.ms += ms;
      a.flops += r.flops;
      a.launches += 1;
    }
    pool_.push_back(r.a);
    pool_.push_back(r.b);
  }
  pending_.clear();
}

GraphRunner::~GraphRunner() {
  if (exec) cudaGraphExecDestroy(exec);
}

cudaError_t GraphRunner::run(cudaStream_t s, const std::function<cudaError_t(cudaStream_t)>& enqueue,
                             bool use_graph) {
  if (!use_graph || !warmed) {
    cudaError_t e = enqueue(s);
    if (e == cudaSuccess) warmed = true;
    return e;
  }
  if (!exec) {
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return e;
    cudaError_t ee = enqueue(s);
    e = cudaStreamEndCapture(s, &g);
    if (ee != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return ee;
    }
    if (e != cudaSuccess) return e;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
      exec = nullptr;
      return e;
    }
  }
  return cudaGraphLaunch(exec, s);
}

}  // namespace jc

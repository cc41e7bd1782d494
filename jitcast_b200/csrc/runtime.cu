// Device runtimes, scratch slots and error reporting for the C ABI.
#include "runtime.h"

#include <memory>

#include "ptx.cuh"

namespace jc {

namespace {
thread_local std::string t_error;
std::mutex g_rt_mu;
std::vector<std::unique_ptr<DeviceRt>> g_rts;
}  // namespace

void set_error(const std::string& msg) { t_error = msg; }
void clear_error() { t_error.clear(); }
const char* last_error() { return t_error.c_str(); }

jc_status fail(jc_status st, const std::string& msg) {
  set_error(msg);
  return st;
}

jc_status fail_cuda(cudaError_t e, const char* what) {
  std::string m = std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
  set_error(m);
  return e == cudaErrorMemoryAllocation ? JC_ERR_OOM : JC_ERR_CUDA;
}

DeviceRt* device_rt(int device, std::string* why) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    if (why) *why = "no CUDA device";
    return nullptr;
  }
  if (device < 0 || device >= count) {
    if (why) *why = "device " + std::to_string(device) + " out of range (" + std::to_string(count) + " devices)";
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_rt_mu);
  if (g_rts.size() < static_cast<size_t>(count)) g_rts.resize(count);
  if (!g_rts[device]) {
    auto rt = std::make_unique<DeviceRt>();
    rt->device = device;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&rt->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&rt->err, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMemset(rt->err, 0, sizeof(uint32_t));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
      if (why) *why = std::string("device init: ") + cudaGetErrorString(e);
      return nullptr;
    }
    g_rts[device] = std::move(rt);
  }
  return g_rts[device].get();
}

void* scratch(DeviceRt* rt, int slot, size_t bytes) {
  if (rt->slot_ptr.size() <= static_cast<size_t>(slot)) {
    rt->slot_ptr.resize(slot + 1, nullptr);
    rt->slot_bytes.resize(slot + 1, 0);
  }
  if (rt->slot_bytes[slot] >= bytes) return rt->slot_ptr[slot];
  if (rt->slot_ptr[slot]) {
    cudaDeviceSynchronize();
    cudaFree(rt->slot_ptr[slot]);
    rt->slot_ptr[slot] = nullptr;
    rt->slot_bytes[slot] = 0;
  }
  const size_t want = static_cast<size_t>(round_up(static_cast<long long>(bytes), 1 << 20));
  void* p = nullptr;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  rt->slot_ptr[slot] = p;
  rt->slot_bytes[slot] = want;
  return p;
}

jc_status take_device_error(DeviceRt* rt) {
  uint32_t host = 0;
  cudaError_t e = cudaMemcpyAsync(&host, rt->err, sizeof(uint32_t), cudaMemcpyDeviceToHost, rt->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(rt->stream);
  if (e != cudaSuccess) return fail_cuda(e, "reading the device error word");
  if (host) {
    cudaMemsetAsync(rt->err, 0, sizeof(uint32_t), rt->stream);
    cudaStreamSynchronize(rt->stream);
    return fail(JC_ERR_TIMEOUT, "a device wait gave up (error bits 0x" + [&] {
      char b[16];
      snprintf(b, sizeof b, "%x", host);
      return std::string(b);
    }() + ")");
  }
  return JC_OK;
}

}  // namespace jc

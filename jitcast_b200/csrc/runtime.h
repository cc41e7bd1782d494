// Per-device runtime state shared by the C-ABI entry points: a library stream, the device
// error word kernels report bounded-wait failures into, grow-only scratch slots, a mutex
// that serialises calls on the device, and the thread-local last-error message.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/jitcast_b200.h"

namespace jc {

struct DeviceRt {
  int device = 0;
  std::mutex mu;
  cudaStream_t stream = nullptr;
  uint32_t* err = nullptr;  // device word; kernels atomicOr DeviceError bits into it
  std::vector<void*> slot_ptr;
  std::vector<size_t> slot_bytes;
};

// The runtime of `device`, created on first use (nullptr and an error message if the device
// does not exist or cannot be initialised).
DeviceRt* device_rt(int device, std::string* why);

// A device buffer of at least `bytes` for slot `slot` of `rt`, grown on demand. Growing
// synchronises the device first, so buffers still in use by queued kernels are not freed.
void* scratch(DeviceRt* rt, int slot, size_t bytes);

// Thread-local last error.
void set_error(const std::string& msg);
void clear_error();
const char* last_error();

// Records `msg` (plus the CUDA error string) and returns the status.
jc_status fail(jc_status st, const std::string& msg);
jc_status fail_cuda(cudaError_t e, const char* what);

// Reads and clears the device error word (synchronises rt->stream first).
jc_status take_device_error(DeviceRt* rt);

inline long long round_up(long long x, long long m) { return (x + m - 1) / m * m; }

}  // namespace jc

// Family-independent engine entry points of the C ABI: sync, options, profiling, destroy.
#include <cstring>
#include <string>

#include "engine.h"
#include "runtime.h"

using namespace jc;

extern "C" {

jc_status jc_shard_rows(int rows, const int32_t* group_start, const int32_t* group_end, int parts, int32_t* cuts_out) {
  clear_error();
  if (rows < 0 || parts < 1) return fail(JC_ERR_INVALID_ARG, "rows must be >= 0 and parts >= 1");
  if (!cuts_out || (rows > 0 && (!group_start || !group_end))) return fail(JC_ERR_INVALID_ARG, "null array");
  for (int i = 0; i < rows; ++i) {
    const int s = group_start[i], t = group_end[i];
    if (s < 0 || s > i || t <= i || t > rows || group_start[s] != s || group_end[s] != t)
      return fail(JC_ERR_INVALID_ARG, "rows of a series are not contiguous (row " + std::to_string(i) + ")");
  }
  const std::vector<int> cuts = jc::shard_rows(rows, group_start, group_end, parts);
  for (int p = 0; p <= parts; ++p) cuts_out[p] = cuts[p];
  return JC_OK;
}

jc_status jc_engine_sync(jc_engine* engine) {
  clear_error();
  if (!engine) return fail(JC_ERR_INVALID_ARG, "null engine");
  std::lock_guard<std::mutex> lk(engine->mu);
  for (int i = 0; i < engine->slots(); ++i) {
    DeviceSlot* s = engine->slot(i);
    cudaSetDevice(s->device);
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_cuda(e, "engine sync");
    if (engine->profile) engine->profiler(i)->collect();
    uint32_t word = 0;
    cudaMemcpy(&word, s->err, sizeof word, cudaMemcpyDeviceToHost);
    if (word) {
      cudaMemset(s->err, 0, sizeof word);
      return fail(JC_ERR_TIMEOUT, "a device wait gave up on GPU " + std::to_string(s->device) + " (error bits " +
                                      std::to_string(word) + ")");
    }
  }
  return JC_OK;
}

jc_status jc_engine_set_option(jc_engine* engine, const char* key, long long value) {
  clear_error();
  if (!engine || !key) return fail(JC_ERR_INVALID_ARG, "null engine or key");
  std::lock_guard<std::mutex> lk(engine->mu);
  const std::string k = key;
  if (k == "cuda_graph") {
    engine->use_graph = value != 0;
  } else if (k == "max_plans") {
    if (value < 1) return fail(JC_ERR_INVALID_ARG, "max_plans must be >= 1");
    engine->max_plans = static_cast<int>(value);
    engine->drop_plans();
  } else if (k == "buckets") {
    engine->buckets = value != 0;
  } else if (k == "fail_plan_allocs") {
    if (value < 0 || value > 1000000) return fail(JC_ERR_INVALID_ARG, "fail_plan_allocs must be in [0, 1e6]");
    engine->fail_plan_allocs = static_cast<int>(value);
  } else if (k == "fail_slot") {
    if (value < -1 || value >= engine->slots()) return fail(JC_ERR_INVALID_ARG, "fail_slot must be -1 or a slot");
    engine->fail_slot = static_cast<int>(value);
  } else if (k == "profile") {
    engine->profile = value != 0;
    for (int i = 0; i < engine->slots(); ++i) engine->profiler(i)->on = engine->profile;
  } else {
    return fail(JC_ERR_INVALID_ARG, "unknown engine option " + k);
  }
  return JC_OK;
}

jc_status jc_engine_profile(jc_engine* engine, int slot, const char** names, double* ms, long long* launches,
                            double* flops, int cap, int* count) {
  clear_error();
  if (!engine || !count) return fail(JC_ERR_INVALID_ARG, "null engine or count");
  std::lock_guard<std::mutex> lk(engine->mu);
  if (slot < 0 || slot >= engine->slots()) return fail(JC_ERR_INVALID_ARG, "slot out of range");
  Profiler* p = engine->profiler(slot);
  cudaSetDevice(engine->slot(slot)->device);
  cudaDeviceSynchronize();
  p->collect();
  // names stay valid until the next call: they point into a per-engine-slot table
  static thread_local std::vector<std::string> keep;
  keep.clear();
  int n = 0;
  for (auto& kv : p->totals) keep.push_back(kv.first);
  for (auto& kv : p->totals) {
    if (n >= cap) break;
    if (names) names[n] = keep[n].c_str();
    if (ms) ms[n] = kv.second.ms;
    if (launches) launches[n] = kv.second.launches;
    if (flops) flops[n] = kv.second.flops;
    ++n;
  }
  *count = n;
  p->totals.clear();
  return JC_OK;
}

jc_status jc_engine_destroy(jc_engine* engine) {
  clear_error();
  if (!engine) return JC_OK;
  {
    std::lock_guard<std::mutex> lk(engine->mu);
    for (int i = 0; i < engine->slots(); ++i) {
      cudaSetDevice(engine->slot(i)->device);
      cudaDeviceSynchronize();
    }
  }
  delete engine;
  return JC_OK;
}

}  // extern "C"

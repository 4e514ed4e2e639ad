// launch_util.h -- raise a kernel's dynamic shared-memory limit only when a
// launch needs more than what was already granted on the current device, so
// steady-state launches make no extra driver call.
#pragma once
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

namespace mxmoe {

inline cudaError_t ensure_dynamic_smem(const void* func, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> granted;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t& g = granted[{func, dev}];
  if (bytes <= g) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e == cudaSuccess) g = bytes;
  return e;
}

}  // namespace mxmoe

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

// Programmatic dependent launch for the kernels of one forward chain: with
// it enabled (PdlScope on the launching thread), a kernel may start while
// the previous one in the stream finishes, so its prologue overlaps that
// tail.  Every kernel launched this way calls griddep_wait() before it reads
// anything an earlier kernel of the chain wrote.
inline bool& pdl_enabled() {
  static thread_local bool on = false;
  return on;
}
struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(pdl_enabled()) { pdl_enabled() = on; }
  ~PdlScope() { pdl_enabled() = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};

template <typename... KArgs, typename... Args>
inline cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                 Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl_enabled() ? &attr : nullptr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

#ifdef __CUDACC__
// Waits until the kernels this one depends on have completed and their
// writes are visible (returns at once for a plain launch).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the chain launch before this one completes.
// Invariant of every chain here: a kernel calls this only after its own
// griddep_wait().  So when a dependent starts, every kernel two or more
// launches back has completed and its writes are visible, and the dependent
// may read those before its own wait (the tensor-core GEMM reads the tile
// prefix sums of the permutation there, the W2 dequant-GEMV the pair counts).
// Only what the immediately preceding kernel writes needs the wait.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

}  // namespace mxmoe

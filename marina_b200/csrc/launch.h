// Kernel launches of the evaluator, with programmatic dependent launch where the caller asks
// for it.
//
// A forward pass is ~90 kernels in a row, each of which depends on the one before. Launched
// plainly, a kernel's blocks start only after the previous grid has drained, and each then
// spends its first microseconds on set-up (barrier initialisation, TMEM allocation, descriptor
// prefetch). With the programmatic-serialisation attribute, the next kernel launches while the
// current one finishes, runs that set-up on the SMs as they free up, and waits in
// grid_dep_wait() (ptx.cuh) for the previous grid's completion before it touches memory. Every
// kernel of this library makes that wait, so the attribute never changes a result.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace mrn {

// Per thread: do launches carry the programmatic-serialisation attribute? Off unless a PdlScope
// on the launching thread turns it on (the forward pass does, for the kernels after its first,
// where pdl_enabled() in runtime.cu says so).
inline bool& pdl_flag() {
  static thread_local bool on = false;
  return on;
}

struct PdlScope {
  bool saved;
  explicit PdlScope(bool on) : saved(pdl_flag()) { pdl_flag() = on; }
  ~PdlScope() { pdl_flag() = saved; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};

// The attribute to append to a launch configuration; returns the number of attributes added.
inline int pdl_attribute(cudaLaunchAttribute* attr) {
  if (!pdl_flag()) return 0;
  attr->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr->val.programmaticStreamSerializationAllowed = 1;
  return 1;
}

// kernel<<<grid, block, smem, stream>>>(args...), with the attribute when the flag is on.
// Kernels declared with __cluster_dims__ keep their compile-time cluster shape.
template <typename... Params, typename... Args>
cudaError_t launch_kernel(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = static_cast<unsigned int>(pdl_attribute(attr));
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace mrn

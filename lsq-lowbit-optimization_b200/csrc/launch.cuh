// Kernel launch with programmatic dependent launch (PDL): every kernel of
// the library is launched with programmatic stream serialization, so it may
// start while the kernel ahead of it in the stream is still running. Each
// kernel lets its successor launch early (pdl_trigger) and blocks in
// pdl_wait, before its first global-memory access, until its predecessor
// has completed and that kernel's memory operations are visible. What
// overlaps is the launch itself and each kernel's prologue (barrier setup,
// TMEM allocation, tensor-map prefetch, shared-memory zeroing) with the tail
// of the kernel before it. Setting W4A8_PDL=0 in the environment launches
// in plain stream order.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <utility>

namespace w4a8 {

// ------------------------- dependent launch --------------------------------
// griddepcontrol (sm_90+). pdl_wait blocks until the grids this one depends
// on programmatically (the kernel ahead of it in the stream, when launched
// with programmatic stream serialization) have completed and their memory
// operations are visible; it returns at once otherwise. pdl_trigger lets the
// dependent grid launch once every CTA of this grid has triggered or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("W4A8_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Launches kern<<<grid, block, smem, st>>>(args...) with the PDL attribute
// (plus the given extra attributes, e.g. a cluster shape).
template <typename... Exp, typename... Act>
cudaError_t launch_kernel_attrs(void (*kern)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                const cudaLaunchAttribute* extra, int n_extra, Act&&... args) {
  cudaLaunchConfig_t cfg;
  std::memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[4];
  if (n_extra < 0 || n_extra > 3) return cudaErrorInvalidValue;
  int n = 0;
  for (int i = 0; i < n_extra; ++i) attr[n++] = extra[i];
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = unsigned(n);
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Act>(args)...);
}

template <typename... Exp, typename... Act>
cudaError_t launch_kernel(void (*kern)(Exp...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Act&&... args) {
  return launch_kernel_attrs(kern, grid, block, smem, st, nullptr, 0, std::forward<Act>(args)...);
}

}  // namespace w4a8

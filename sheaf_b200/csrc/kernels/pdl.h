// Programmatic dependent launch for the hand-written kernels: a kernel
// launched with launch_pdl may be scheduled while the previous kernel in the
// stream drains; it must call pdl_prologue() before touching global memory
// (griddepcontrol.wait returns once the previous grids have completed and
// their writes are visible), which also lets the next kernel start launching.
#pragma once
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>

namespace sb {

// Kernel launches issued by this library in this process (every launch path
// counts itself here; read by sb_kernel_launch_count).
inline std::atomic<uint64_t>& launch_counter() {
  static std::atomic<uint64_t> n{0};
  return n;
}

__device__ __forceinline__ void pdl_prologue() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
}

inline void pdl_attribute(cudaLaunchAttribute* at) {
  at->id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at->val.programmaticStreamSerializationAllowed = 1;
}

template <typename... K, typename... A>
cudaError_t launch_pdl(void (*kern)(K...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute at[1];
  pdl_attribute(&at[0]);
  cfg.attrs = at;
  cfg.numAttrs = 1;
  launch_counter().fetch_add(1, std::memory_order_relaxed);
  return cudaLaunchKernelEx(&cfg, kern, std::forward<A>(args)...);
}

}  // namespace sb

// Programmatic dependent launch (PDL): a kernel launched with it may start while its predecessor in
// the stream is still running.  Each such kernel calls pdl_wait() before it reads anything a
// predecessor writes, or writes anything a predecessor may still read; work that depends only on
// weights (streaming them into shared memory) may run before that.  pdl_trigger() lets the next
// kernel launch early; it is issued at the start of every kernel here.  Both instructions are no-ops
// for kernels launched without the attribute.  BARQ_PDL=0 in the environment disables it.
#pragma once
#include <cuda_runtime.h>

#include <utility>

namespace barq {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();
// Per-call override (kept while set): 0 = launch without the attribute, 1 = with (BARQ_PDL=0 wins).
void set_pdl_mode(int mode);

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace barq

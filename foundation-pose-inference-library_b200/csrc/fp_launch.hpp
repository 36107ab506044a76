// Kernel launches with programmatic dependent launch (PDL).
//
// A kernel launched through launchPdl may begin while the previous kernel in
// the stream is still finishing: every such kernel calls tc::pdlTrigger() on
// entry (its dependents may be scheduled once all of its CTAs have started)
// and tc::pdlWait() before its first access to memory an earlier kernel
// writes or reads (griddepcontrol.wait returns once the previous grid has
// completed and its writes are visible). The prologue before the wait
// (barrier init, TMEM allocation, shared-memory tables) then overlaps the
// previous kernel's tail, and the launch latency between dependent kernels
// is hidden. Kernels launched without the attribute are unaffected by both
// calls.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace fpb {

template <typename... KArgs, typename... Args>
cudaError_t launchPdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace fpb

// launch.h -- programmatic dependent launch for the plan's kernels.
//
// Every kernel of a plan is launched with programmatic stream serialization:
// the next kernel may be scheduled (and run its prologue) while this one
// drains.  Each such kernel begins with pdl_entry(): griddepcontrol.wait
// blocks until every prerequisite grid has completed and its memory is
// visible, so no kernel touches global memory before its predecessors are
// done.  A kernel launched without the attribute passes griddepcontrol.wait
// at once.
#pragma once
#include <cuda_runtime.h>

namespace tb {

__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Whether launches carry the programmatic-serialization attribute (TB_PDL=0
// turns it off).
bool pdl_enabled();

template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace tb

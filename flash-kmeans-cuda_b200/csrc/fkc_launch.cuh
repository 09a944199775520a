// Kernel launches with programmatic dependent launch (PDL): a kernel launched
// this way may start while the previous kernel on the stream drains; it runs
// its independent prologue (barrier init, TMEM allocation, descriptor
// prefetch) and then waits in griddepcontrol.wait until the previous grid has
// completed and its memory is visible. On a stream whose previous operation is
// not a kernel the attribute has no effect and the wait returns at once.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "fkc_internal.h"

namespace fkc {

// Blocks until every prerequisite grid has completed (no-op without PDL).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
  count_launches(1);
  return FKC_OK;
}

// Zero-fills `bytes` (a multiple of 4) at `ptr` with a PDL kernel, so that a
// fill between two kernels keeps the launch chain programmatic.
int launch_zero_fill(void* ptr, size_t bytes, cudaStream_t stream);

}  // namespace fkc

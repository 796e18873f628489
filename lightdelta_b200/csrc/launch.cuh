// Kernel launch helper shared by the CUDA translation units of liblightdelta_b200.so.
//
// Every kernel of the library starts with grid_dependency_wait(): with programmatic dependent
// launch (PDL) enabled, the launch is marked programmatic-stream-serialised, so the kernel's
// CTAs may be scheduled while the preceding kernel on the stream is finishing, and they block
// there until that kernel has completed and its memory writes are visible.  The kernel then
// calls allow_dependent_launch() so the next PDL launch can be scheduled in turn.  Without the
// attribute (PDL disabled, or a preceding operation that is not a kernel) both instructions
// return at once and ordinary stream order applies.
#pragma once

#include <cuda_runtime.h>

#include <utility>

#include "internal.h"

namespace ldb {

__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// cudaLaunchKernelEx with the library's launch attributes: PDL when enabled, and a runtime
// cluster size when `cluster` > 1 (kernels with compile-time cluster dimensions pass 1).
template <typename... KernelArgs, typename... Args>
cudaError_t launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   unsigned int cluster, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attributes[2];
  unsigned int count = 0;
  if (programmatic_launch_enabled()) {
    attributes[count].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attributes[count].val.programmaticStreamSerializationAllowed = 1;
    ++count;
  }
  if (cluster > 1) {
    attributes[count].id = cudaLaunchAttributeClusterDimension;
    attributes[count].val.clusterDim.x = cluster;
    attributes[count].val.clusterDim.y = 1;
    attributes[count].val.clusterDim.z = 1;
    ++count;
  }
  config.attrs = attributes;
  config.numAttrs = count;
  return cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
}

}  // namespace ldb

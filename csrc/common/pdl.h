// Programmatic dependent launch (PDL) for the kernels of a decode step.
//
// A kernel launched with launch_pdl() may start while the previous kernel on
// its stream is still running, as soon as every CTA of that kernel has
// executed pdl_trigger() (or exited). Before it reads anything the previous
// kernel wrote, or writes anything the previous kernel may still read, it
// executes pdl_wait(), which returns once the previous kernel has completed
// and its memory operations are visible. Work that depends on neither
// (barrier and TMEM set-up, tensor-map prefetch, loads of weights that no
// kernel writes) runs before the wait and so overlaps the previous kernel's
// tail. Without a PDL predecessor both instructions are no-ops. CUDA graphs
// capture the programmatic edges.
#pragma once

#include <cuda_runtime.h>

#include "check.h"

namespace b200ar {

#if defined(__CUDACC__)
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Launches `kernel` with programmatic stream serialization enabled (and an
// optional cluster shape when cluster_x > 1).
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster_x,
                Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = 1;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  B200AR_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}
#endif

}  // namespace b200ar

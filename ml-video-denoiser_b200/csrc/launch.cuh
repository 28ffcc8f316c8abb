// Kernel launches with programmatic dependent launch (PDL).
//
// Every kernel of the forward is launched with programmatic stream
// serialisation: the next kernel in the stream may start as soon as every
// CTA of the current one has executed pdl_trigger(), so its launch and its
// prologue (weight loads, shared-memory set-up, TMEM allocation, barrier
// init) overlap the tail of the current kernel. Each kernel calls
// pdl_wait() before it reads anything an earlier kernel wrote and before
// its first global write; pdl_wait() returns once the preceding kernel has
// completed and its writes are visible (so ordering stays transitive along
// the stream).
//
// Order rule for kernels that allocate TMEM: tcgen05.alloc, the permit
// relinquish and the barrier that publishes the TMEM address all come
// BEFORE pdl_trigger(). A dependent grid can then only be scheduled once
// every CTA of this grid already holds its columns. Were the trigger first,
// a dependent CTA could take an SM's free columns while this grid's CTA on
// that SM still waits in tcgen05.alloc (which has no timeout); the dependent
// would then wait in griddepcontrol.wait for a grid that cannot finish.
#pragma once

#include <cuda_runtime.h>

#include <utility>

namespace dnb {

__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The same with clusters of two CTAs along x (CTA pairs for cta_group::2 MMAs).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_pair(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                            Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace dnb

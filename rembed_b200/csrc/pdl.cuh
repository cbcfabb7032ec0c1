// Programmatic dependent launch (PDL) for the forward's chain of kernels.
//
// Every kernel of this library is launched with programmatic stream
// serialisation (launch_pdl): it may be scheduled while the previous kernel
// on the stream is still running, so its launch and its prologue (barrier
// set-up, TMEM allocation, descriptor prefetch) overlap that kernel's tail.
// Before its first access to global memory every kernel calls pdl_wait(),
// which returns once the previous grid has completed and its writes are
// visible (immediately when there is no such grid); pdl_trigger() allows
// the next kernel to be scheduled.  Inside a captured CUDA graph the same
// launches become programmatic edges.
#pragma once

#include <cuda_runtime.h>

namespace rg {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace rg

// Programmatic dependent launch for chains of small dependent kernels (the
// recursive factorisation issues ~1300 of them per OBS pass).  A kernel
// launched by launch_pdl() may be scheduled while its predecessor in the
// stream is still running: it does its setup that touches no global memory
// (barrier init, TMEM allocation, tensor-map prefetch), then pdl_wait() blocks
// until the predecessor grid has completed and its writes are visible, and
// only then reads or writes global memory.  pdl_trigger() lets the kernel's
// own successor be scheduled; it is issued right after pdl_wait(), so at most
// one launch ahead is resident early.  A kernel launched without the attribute
// returns from pdl_wait() at once.
#pragma once

#include <cuda_runtime.h>

namespace tb {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
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
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace tb

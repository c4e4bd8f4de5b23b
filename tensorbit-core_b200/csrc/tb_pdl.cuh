// Programmatic dependent launch for chains of small dependent kernels (the
// recursive factorisation issues ~1300 of them per OBS pass).  A kernel
// launched by launch_pdl() is handed to the GPU before its predecessor in the
// stream has finished, so that it starts the moment the predecessor exits
// instead of a launch latency later.  It does its setup that touches no global
// memory (barrier init, TMEM allocation, tensor-map prefetch), then pdl_wait()
// blocks until the predecessor grid has completed and its writes are visible,
// and only then reads or writes global memory.  A kernel launched without the
// attribute returns from pdl_wait() at once.
//
// No kernel issues griddepcontrol.launch_dependents: its successor is released
// only when it exits.  With the trigger issued right after pdl_wait() in every
// kernel (successors resident early), the exact-OBS chain of a 14336-wide
// layer gave results that differed from run to run on B200, some with a failed
// Cholesky pivot, although every event and stream ordering of the schedule
// checks out.  The edge the trigger breaks is a cache contract, not an
// ordering: base_chol_inv_kernel reads the Schur-updated block A, and
// inblock_kernel the error-updated columns Wr and the factor V, through
// const __restrict__ pointers, which lets the compiler serve those loads from
// the non-coherent read-only path, whose contract is that the data does not
// change during the reading kernel's lifetime.  Each of those buffers is
// written by the launch just before the reader in its stream (a GEMM epilogue
// or the previous base kernel).  With an early trigger the reader's lifetime
// begins while those writes are still being made, so the contract no longer
// holds; without it a kernel starts only after its predecessor has exited and
// every read-only load sees the finished data.  The schedule is therefore
// race-free exactly as launched here: stream order for a kernel's own
// predecessor, events for the other streams, and no kernel resident before
// the kernel whose output it reads has ended.  (The early trigger was also
// not faster: 26.3 against 25.7 ms per pass.)
#pragma once

#include <cuda_runtime.h>

#include <vector>

namespace tb {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Streams whose next launch must be an ordinary one: the first launch behind a
// cudaStreamWaitEvent takes no attribute, so that nothing rests on how a
// programmatic launch combines the predecessor kernel with the awaited event.
// Every cross-stream wait marks its stream with pdl_fence(); pdl_allowed()
// reads and clears the mark.  The marks are per host thread; a stream is
// driven from one thread at a time.
inline thread_local std::vector<cudaStream_t> g_pdl_fences;

inline void pdl_fence(cudaStream_t st) {
    for (cudaStream_t x : g_pdl_fences)
        if (x == st) return;
    g_pdl_fences.push_back(st);
}

// True if the next launch on st may be programmatic; clears st's mark.
inline bool pdl_allowed(cudaStream_t st) {
    auto& f = g_pdl_fences;
    for (size_t i = 0; i < f.size(); ++i)
        if (f[i] == st) {
            f[i] = f.back();
            f.pop_back();
            return false;
        }
    return true;
}

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
    attr[0].val.programmaticStreamSerializationAllowed = pdl_allowed(st) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

}  // namespace tb

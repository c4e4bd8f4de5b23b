// Internal runtime helpers shared by the kernel translation units.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "tb_kernels.h"

namespace tb {

// Records printf-style text for tb_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// TB_ERR_CUDA with the runtime's error string.
int cuda_fail(cudaError_t e, const char* what);
// Converts a pending launch error into a status.
int check_launch(const char* what);
// TB_ERR_NO_DEVICE unless a device is current; returns its ordinal.
int require_device(int* dev_out);
// Device copy of the top-n-of-m tie table for the current device, built on
// first use (a cudaMalloc + copy, so first use must precede stream capture).
int topn_table(int n, int m, const uint8_t** out);
// True when the current device already holds the top-n-of-m tie table
// (no build, no allocation).
bool topn_table_ready(int n, int m);
// Stream-ordered scratch for a call's small working buffers, from a memory
// pool the library keeps per device with its memory retained between calls
// (release threshold: never), so that after the first calls no allocation
// reaches the driver's memory manager - where it could wait behind other
// clients of the driver, such as a clock sampler - and calls on different
// streams still get separate buffers.
int scratch_alloc(void** ptr, size_t bytes, cudaStream_t stream);
void scratch_free(void* ptr, cudaStream_t stream);

}  // namespace tb

// Internal interface of the radix threshold select (tb_threshold.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace tb {

// Device scratch of one selection: digit histogram and the running state.
struct SelectState {
    unsigned long long hist[2048];
    unsigned long long target;   // rank still to find inside the current prefix
    unsigned long long pruned;   // elements below the threshold
    uint32_t prefix;             // key digits fixed so far
    float threshold;
    unsigned int done;           // histogram blocks finished in the current pass (the last one scans)
};

// keep = (size_t)(sparsity * (float)N), at least 1 (ehap.hpp:301-307);
// TB_ERR_ZERO_SIZE / TB_ERR_CONFIG as the reference's enum would report.
int threshold_args(size_t N, float sparsity, size_t* keep_out);
// Enqueues the three digit passes and the mask pass on `stream`.
int threshold_launch(const float* scores, size_t N, size_t keep, uint8_t* mask_out, SelectState* st,
                     cudaStream_t stream);
// Enqueues only the three digit passes (keep < N): st->threshold holds the
// threshold afterwards and st->pruned is zero, for a later pass that applies
// the threshold itself and counts what it drops into st->pruned.
int threshold_digits(const float* scores, size_t N, size_t keep, SelectState* st, cudaStream_t stream);
// Reads threshold and pruned count back (synchronises `stream`); with both
// outputs null it does nothing.
int threshold_finish(size_t N, size_t keep, const SelectState* st, float* thr_out, uint64_t* pruned_out,
                     cudaStream_t stream);
// Enqueues zeroing of a state whose threshold and count are to be read
// without a selection (keep >= N: nothing is pruned).
int threshold_clear(SelectState* st, cudaStream_t stream);

}  // namespace tb

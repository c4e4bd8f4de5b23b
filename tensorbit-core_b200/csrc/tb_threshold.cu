// EHAP global-threshold selection (EHAPPruner::select_pruning_mask,
// include/tensorbit/core/ehap.hpp:290-329) as a device radix select.
//
// The reference copies the N scores, runs std::nth_element for the (N-keep)-th
// smallest and keeps every score >= that value.  The threshold is an order
// statistic, so any exact selection returns the same value; ties at it are all
// kept by the >= comparison.  Here the FP32 scores are mapped to order-
// preserving 32-bit keys and the key of rank t = N - keep is found digit by
// digit (11 + 11 + 10 bits): three histogram passes over the scores; the last
// block of each pass to finish (a ticket counter, no waiting) scans the
// histogram, picks the digit and narrows the rank.  A final pass writes the
// 1-byte-per-element mask (ehap.hpp:320-327) and counts the pruned elements.
//
// Scratch (device memory beyond the inputs and outputs): one 2048-bin u64
// histogram plus a small state block (struct SelectState, about 16.4 KB).
#include <algorithm>

#include "tb_device.cuh"
#include "tb_runtime.h"
#include "tb_threshold.h"

namespace tb {
namespace {

constexpr int kThreads = 512;
constexpr int kBins = 2048;

__device__ __forceinline__ uint32_t order_key(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_float(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Run by one whole block of kThreads once a pass's histogram is complete: find
// the digit whose cumulative count covers the target rank, extend the prefix,
// narrow the rank, and clear the histogram and the ticket for the next pass
// (the last pass also sets the threshold).  The histogram is read from L2
// (it was built by atomics).
__device__ void scan_digit(SelectState* __restrict__ st, int pass) {
    __shared__ unsigned long long part[kThreads];
    const int t = threadIdx.x;
    const int bins = pass == 2 ? 1024 : 2048;
    const int per = bins / kThreads;
    unsigned long long local = 0;
    for (int j = 0; j < per; ++j) local += __ldcg(&st->hist[t * per + j]);
    part[t] = local;
    __syncthreads();
    // inclusive scan over the kThreads partial sums (Hillis-Steele)
    for (int off = 1; off < kThreads; off <<= 1) {
        const unsigned long long v = t >= off ? part[t - off] : 0ull;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    const unsigned long long target = st->target;
    const unsigned long long before = t ? part[t - 1] : 0ull;
    if (target >= before && target < part[t]) {
        unsigned long long c = before;
        for (int j = 0; j < per; ++j) {
            const unsigned long long h = __ldcg(&st->hist[t * per + j]);
            if (target < c + h) {
                const int digit = t * per + j;
                const int width = pass == 2 ? 10 : 11;
                const uint32_t prefix = (st->prefix << width) | static_cast<uint32_t>(digit);
                st->prefix = prefix;
                st->target = target - c;
                if (pass == 2) st->threshold = key_float(prefix);
                break;
            }
            c += h;
        }
    }
    __syncthreads();
    for (int i = t; i < kBins; i += kThreads) st->hist[i] = 0;
    if (t == 0) st->done = 0;
}

// Histogram of digit `(key >> shift) & (bins-1)` over keys whose bits above
// `shift + width` equal `prefix` (all keys when width == 32 - shift).
__global__ void __launch_bounds__(kThreads) radix_hist_kernel(const float* __restrict__ s, size_t N,
                                                               SelectState* __restrict__ st, int pass) {
    __shared__ unsigned int sh[kBins];
    for (int i = threadIdx.x; i < kBins; i += kThreads) sh[i] = 0;
    __syncthreads();
    const int shift = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
    const uint32_t dmask = pass == 2 ? 1023u : 2047u;
    const uint32_t prefix = st->prefix;
    const int hi = shift + (pass == 2 ? 10 : 11);  // bits at and above `hi` must match prefix
    const size_t n4 = N / 4;
    const float4* s4 = reinterpret_cast<const float4*>(s);
    const size_t stride = (size_t)gridDim.x * kThreads;
    // One shared-memory atomic per element.  (Aggregating the lanes of a warp
    // that share a bin with __match_any_sync measured slower on B200: 3.67
    // against 2.63 ms for tb-prune's sequence over a 7B-class layer.)
    auto add = [&](float f) {
        const uint32_t k = order_key(f);
        if (hi >= 32 || (k >> hi) == prefix) atomicAdd(&sh[(k >> shift) & dmask], 1u);
    };
    if ((reinterpret_cast<uintptr_t>(s) & 15u) == 0) {
        for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < n4; i += stride) {
            const float4 v = __ldcs(s4 + i);
            add(v.x); add(v.y); add(v.z); add(v.w);
        }
        for (size_t i = n4 * 4 + blockIdx.x * (size_t)kThreads + threadIdx.x; i < N; i += stride) add(s[i]);
    } else {
        for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < N; i += stride) add(s[i]);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kBins; i += kThreads)
        if (sh[i]) atomicAdd(&st->hist[i], static_cast<unsigned long long>(sh[i]));
    // The last block to finish scans the histogram: every block's additions
    // are made visible (fence) before it takes its ticket.
    __threadfence();
    __syncthreads();
    __shared__ unsigned int ticket;
    if (threadIdx.x == 0) ticket = atomicAdd(&st->done, 1u);
    __syncthreads();
    if (ticket != gridDim.x - 1) return;
    __threadfence();
    scan_digit(st, pass);
}

// mask[i] = s[i] >= thr (1 byte per element); counts elements not kept.
__global__ void __launch_bounds__(kThreads) threshold_mask_kernel(const float* __restrict__ s, size_t N,
                                                                   uint8_t* __restrict__ mask,
                                                                   SelectState* __restrict__ st) {
    const float thr = st->threshold;
    unsigned long long pruned = 0;
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < N; i += (size_t)gridDim.x * kThreads) {
        const bool keep = s[i] >= thr;
        if (mask) mask[i] = keep ? 1 : 0;
        pruned += keep ? 0 : 1;
    }
    const unsigned long long tot = __reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(pruned));
    if ((threadIdx.x & 31) == 0 && tot) atomicAdd(&st->pruned, tot);
}

__global__ void init_state_kernel(SelectState* st, unsigned long long target) {
    for (int i = threadIdx.x; i < kBins; i += blockDim.x) st->hist[i] = 0;
    if (threadIdx.x == 0) {
        st->prefix = 0;
        st->target = target;
        st->pruned = 0;
        st->threshold = 0.0f;
        st->done = 0;
    }
}

unsigned grid_for(size_t n) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t want = (n / 4 + kThreads - 1) / kThreads;
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(want, static_cast<size_t>(sms) * 4)));
}

}  // namespace

int threshold_args(size_t N, float sparsity, size_t* keep_out) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty importance tensor");
    if (sparsity <= 0.0f || sparsity >= 1.0f) return fail(TB_ERR_CONFIG, "sparsity_ratio %g outside (0, 1)", sparsity);
    size_t keep = static_cast<size_t>(sparsity * static_cast<float>(N));  // ehap.hpp:306
    if (keep == 0) keep = 1;
    *keep_out = keep;
    return TB_OK;
}

int threshold_launch(const float* scores, size_t N, size_t keep, uint8_t* mask_out, SelectState* st,
                     cudaStream_t stream) {
    if (keep >= N) {
        // ehap.hpp:308-311: everything kept, nothing pruned; no threshold exists.
        if (mask_out) {
            cudaError_t e = cudaMemsetAsync(mask_out, 1, N, stream);
            if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(mask)");
        }
        return TB_OK;
    }
    init_state_kernel<<<1, 1024, 0, stream>>>(st, static_cast<unsigned long long>(N - keep));
    const unsigned grid = grid_for(N);
    for (int pass = 0; pass < 3; ++pass) radix_hist_kernel<<<grid, kThreads, 0, stream>>>(scores, N, st, pass);
    threshold_mask_kernel<<<grid, kThreads, 0, stream>>>(scores, N, mask_out, st);
    return check_launch("threshold select");
}

int threshold_digits(const float* scores, size_t N, size_t keep, SelectState* st, cudaStream_t stream) {
    init_state_kernel<<<1, 1024, 0, stream>>>(st, static_cast<unsigned long long>(N - keep));
    const unsigned grid = grid_for(N);
    for (int pass = 0; pass < 3; ++pass) radix_hist_kernel<<<grid, kThreads, 0, stream>>>(scores, N, st, pass);
    return check_launch("threshold digits");
}

int threshold_clear(SelectState* st, cudaStream_t stream) {
    init_state_kernel<<<1, 1024, 0, stream>>>(st, 0ull);
    return check_launch("threshold clear");
}

int threshold_finish(size_t N, size_t keep, const SelectState* st, float* thr_out, uint64_t* pruned_out,
                     cudaStream_t stream) {
    if (!thr_out && !pruned_out) return TB_OK;  // nothing to read back: no host wait
    float thr = 0.0f;
    unsigned long long pruned = 0;
    if (keep < N) {
        cudaError_t e = cudaMemcpyAsync(&thr, &st->threshold, sizeof(float), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&pruned, &st->pruned, sizeof(pruned), cudaMemcpyDeviceToHost, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "threshold result D2H");
    } else {
        cudaError_t e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    }
    if (thr_out) *thr_out = thr;
    if (pruned_out) *pruned_out = pruned;
    return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_threshold_select(const float* scores, size_t N, float sparsity, uint8_t* mask_out, float* threshold_out,
                        uint64_t* pruned_out, void* stream) {
    size_t keep = 0;
    int rc = threshold_args(N, sparsity, &keep);
    if (rc) return rc;
    if (!scores) return fail(TB_ERR_ARG, "tb_threshold_select: null scores");
    if ((rc = require_device(nullptr))) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    SelectState* scratch = nullptr;
    if (keep < N) {
        if ((rc = scratch_alloc(reinterpret_cast<void**>(&scratch), sizeof(SelectState), st))) return rc;
    }
    rc = threshold_launch(scores, N, keep, mask_out, scratch, st);
    if (rc == TB_OK) rc = threshold_finish(N, keep, scratch, threshold_out, pruned_out, st);
    scratch_free(scratch, st);
    return rc;
}

}  // extern "C"

// EHAPPruner loops that the reference runs on the host only
// (include/tensorbit/core/ehap.hpp): the 1-byte-per-element mask apply, the
// Fisher L2 normalisation and the two weight-compensation modes.
//
// Two of them are defined by the reference as one serial float sum over the
// whole tensor (apply_fisher_normalization, ehap.hpp:720-731, and kBias
// compensation, ehap.hpp:382-386).  Float addition is not associative, so the
// only way to return the same bits is the same serial order: those sums run
// on one thread, reading ahead in 16-byte vectors.  Both are off by default in
// the reference and in tb-prune.
#include <algorithm>

#include "tb_device.cuh"
#include "tb_runtime.h"

namespace tb {
namespace {

constexpr int kThreads = 256;

unsigned grid_for(size_t work) {
    size_t b = (work + kThreads - 1) / kThreads;
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(b, 148u * 32u)));
}

// EHAPPruner::apply_mask (ehap.hpp:342-348): w[i] = 0 where mask[i] == 0.
__global__ void ehap_apply_kernel(float* __restrict__ w, const uint8_t* __restrict__ mask, size_t N,
                                  unsigned long long* __restrict__ pruned) {
    unsigned long long cnt = 0;
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < N; i += (size_t)gridDim.x * kThreads)
        if (!mask[i]) { w[i] = 0.0f; ++cnt; }
    const unsigned tot = __reduce_add_sync(0xFFFFFFFFu, static_cast<unsigned>(cnt));
    if ((threadIdx.x & 31) == 0 && tot && pruned) atomicAdd(pruned, static_cast<unsigned long long>(tot));
}

// apply_fisher_normalization (ehap.hpp:720-731): serial sum of squares, sqrt,
// then every element scaled by the reciprocal.  Thread 0 of block 0 sums; the
// scale is applied by the grid-wide kernel below.
__global__ void fisher_norm_sum_kernel(const float* __restrict__ F, size_t N, float* __restrict__ norm_out) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    float norm = 0.0f;
    for (size_t i = 0; i < N; ++i) norm = __fadd_rn(norm, __fmul_rn(F[i], F[i]));
    *norm_out = __fsqrt_rn(norm);
}

__global__ void fisher_scale_kernel(float* __restrict__ F, size_t N, const float* __restrict__ norm_in) {
    const float norm = *norm_in;
    if (!(norm > 0.0f)) return;  // the reference leaves F unchanged unless norm > 0
    const float inv = __fdiv_rn(1.0f, norm);
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < N; i += (size_t)gridDim.x * kThreads)
        F[i] = __fmul_rn(F[i], inv);
}

// kBias (ehap.hpp:382-386): delta = serial sum of the pruned weights, added to
// the last weight.
__global__ void compensate_bias_kernel(float* __restrict__ w, const uint8_t* __restrict__ mask, size_t N) {
    if (blockIdx.x != 0 || threadIdx.x != 0) return;
    float delta = 0.0f;
    for (size_t i = 0; i < N; ++i)
        if (!mask[i]) delta = __fadd_rn(delta, w[i]);
    w[N - 1] = __fadd_rn(w[N - 1], delta);
}

// kRedist (ehap.hpp:387-401): per group of 8 (the last one may be short),
// pruned weights summed and spread over the kept ones in proportion to their
// scores.
__global__ void compensate_redist_kernel(float* __restrict__ w, const uint8_t* __restrict__ mask,
                                         const float* __restrict__ s, size_t N) {
    const size_t G = (N + 7) / 8;
    for (size_t g = blockIdx.x * (size_t)kThreads + threadIdx.x; g < G; g += (size_t)gridDim.x * kThreads) {
        const size_t b = g * 8, e = b + 8 < N ? b + 8 : N;
        float t_pruned = 0.0f, t_weight = 0.0f;
        for (size_t i = b; i < e; ++i) {
            if (!mask[i]) t_pruned = __fadd_rn(t_pruned, w[i]);
            else t_weight = __fadd_rn(t_weight, s[i]);
        }
        if (t_weight <= 0.0f) continue;
        for (size_t i = b; i < e; ++i)
            if (mask[i]) w[i] = __fadd_rn(w[i], __fdiv_rn(__fmul_rn(t_pruned, s[i]), t_weight));
    }
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

int tb_ehap_apply_mask(float* weights, const uint8_t* mask, size_t N, uint64_t* pruned_out, void* stream) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty tensor");
    if (!weights || !mask) return fail(TB_ERR_ARG, "tb_ehap_apply_mask: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    unsigned long long* cnt = nullptr;
    if (pruned_out) {
        if ((rc = scratch_alloc(reinterpret_cast<void**>(&cnt), sizeof(*cnt), st))) return rc;
        cudaError_t e = cudaMemsetAsync(cnt, 0, sizeof(*cnt), st);
        if (e != cudaSuccess) {
            scratch_free(cnt, st);
            return cuda_fail(e, "tb_ehap_apply_mask counter");
        }
    }
    ehap_apply_kernel<<<grid_for(N), kThreads, 0, st>>>(weights, mask, N, cnt);
    rc = check_launch("ehap_apply_kernel");
    if (cnt) {
        unsigned long long h = 0;
        cudaError_t e = cudaMemcpyAsync(&h, cnt, sizeof(h), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        scratch_free(cnt, st);
        if (!rc && e != cudaSuccess) rc = cuda_fail(e, "tb_ehap_apply_mask readback");
        *pruned_out = h;
    }
    return rc;
}

int tb_fisher_normalize(float* fisher, size_t N, void* stream) {
    if (N == 0) return TB_OK;
    if (!fisher) return fail(TB_ERR_ARG, "tb_fisher_normalize: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    float* norm = nullptr;
    if ((rc = scratch_alloc(reinterpret_cast<void**>(&norm), sizeof(float), st))) return rc;
    fisher_norm_sum_kernel<<<1, 32, 0, st>>>(fisher, N, norm);
    fisher_scale_kernel<<<grid_for(N), kThreads, 0, st>>>(fisher, N, norm);
    rc = check_launch("fisher normalisation");
    scratch_free(norm, st);
    return rc;
}

int tb_compensate(float* weights, const uint8_t* mask, const float* importance, size_t N, int mode, void* stream) {
    if (mode == 0) return TB_OK;  // CompensationMode::kNone
    if (mode < 0 || mode > 2) return fail(TB_ERR_ARG, "bad compensation mode %d", mode);
    if (N == 0) return TB_OK;
    if (!weights || !mask || (mode == 2 && !importance)) return fail(TB_ERR_ARG, "tb_compensate: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    if (mode == 1) compensate_bias_kernel<<<1, 32, 0, st>>>(weights, mask, N);
    else compensate_redist_kernel<<<grid_for((N + 7) / 8), kThreads, 0, st>>>(weights, mask, importance, N);
    return check_launch("compensation");
}

}  // extern "C"

// Per-stage kernels: the reference's seven launchers (kernels.hpp:24-124) and
// the device versions of the pruners' host loops (ehap.hpp / coring.hpp).
//
// These are bandwidth-trivial element-wise passes; each uses a grid-stride
// loop sized to a few waves of the 148 SMs.  The fused single-pass kernel in
// tb_fused.cu is the throughput path.
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

#define TB_GRID_STRIDE(i, n) \
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (n); i += (size_t)gridDim.x * blockDim.x)

__global__ void fisher_diagonal_kernel(const float* __restrict__ g, float* __restrict__ F, size_t B, size_t N) {
    TB_GRID_STRIDE(i, N) {
        float acc = 0.0f;
        for (size_t b = 0; b < B; ++b) {
            const float x = g[b * N + i];
            acc = __fadd_rn(acc, __fmul_rn(x, x));
        }
        F[i] = acc;
    }
}

__global__ void fisher_accumulate_kernel(float* __restrict__ F, const float* __restrict__ g, size_t N, float alpha) {
    TB_GRID_STRIDE(i, N) F[i] = __fadd_rn(F[i], __fmul_rn(__fmul_rn(alpha, g[i]), g[i]));
}

__global__ void beta_decay_kernel(float* __restrict__ F, float beta, size_t N) {
    TB_GRID_STRIDE(i, N) F[i] = __fmul_rn(beta, F[i]);
}

template <int GDT>
__global__ void ema_step_kernel(float* __restrict__ F, const void* __restrict__ g, size_t N, float alpha,
                                float beta, float contrib, int first) {
    TB_GRID_STRIDE(i, N) {
        const float x = Dtype<GDT>::load(g, i);
        F[i] = first ? ema_first(alpha, x) : ema_next(F[i], beta, contrib, x);
    }
}

template <int WDT>
__global__ void importance_kernel(const void* __restrict__ w, const float* __restrict__ F, float* __restrict__ s,
                                  size_t N, float damp, int mode) {
    const bool have_f = F != nullptr;
    TB_GRID_STRIDE(i, N) s[i] = importance(Dtype<WDT>::load(w, i), have_f ? F[i] : 0.0f, damp, mode, have_f);
}

template <int M>
__global__ void nm_mask_kernel(const float* __restrict__ s, uint8_t* __restrict__ mask, size_t G, int n,
                               int strategy, int rounds, int permute, const uint8_t* __restrict__ lut) {
    TB_GRID_STRIDE(g, G) {
        float v[M];
#pragma unroll
        for (int k = 0; k < M; ++k) v[k] = s[g * M + k];
        mask[g] = static_cast<uint8_t>(select_group<M>(v, n, strategy, rounds, permute != 0, lut));
    }
}

__global__ void apply_mask_kernel(float* __restrict__ w, const uint8_t* __restrict__ mask, size_t an, int m) {
    TB_GRID_STRIDE(i, an) {
        if (!((mask[i / m] >> (i % m)) & 1u)) w[i] = 0.0f;
    }
}

template <int M>
__global__ void redistribute_kernel(float* __restrict__ w, const uint8_t* __restrict__ mask,
                                    const float* __restrict__ s, size_t G, int mode) {
    TB_GRID_STRIDE(g, G) {
        float wg[M], sg[M];
#pragma unroll
        for (int k = 0; k < M; ++k) { wg[k] = w[g * M + k]; sg[k] = s[g * M + k]; }
        redistribute_group<M>(wg, sg, mask[g], mode);
#pragma unroll
        for (int k = 0; k < M; ++k) w[g * M + k] = wg[k];
    }
}

int check_nm(size_t N, int n, int m) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty tensor");
    if (n <= 0 || m <= 0 || n >= m) return fail(TB_ERR_CONFIG, "invalid N:M %d:%d", n, m);
    if (N % static_cast<size_t>(m) != 0) return fail(TB_ERR_SHAPE, "numel %zu not divisible by M=%d", N, m);
    if (m > 8) return fail(TB_ERR_UNSUPPORTED, "M=%d > 8: masks hold one byte per group", m);
    return TB_OK;
}

template <template <int> class K, typename... Args>
int launch_by_m(int m, size_t work, cudaStream_t st, Args... args) {
    const unsigned grid = grid_for(work);
    switch (m) {
    case 2: K<2>::launch(grid, st, args...); break;
    case 3: K<3>::launch(grid, st, args...); break;
    case 4: K<4>::launch(grid, st, args...); break;
    case 5: K<5>::launch(grid, st, args...); break;
    case 6: K<6>::launch(grid, st, args...); break;
    case 7: K<7>::launch(grid, st, args...); break;
    case 8: K<8>::launch(grid, st, args...); break;
    default: return fail(TB_ERR_UNSUPPORTED, "M=%d", m);
    }
    return TB_OK;
}

template <int M> struct NmMaskLaunch {
    template <typename... A>
    static void launch(unsigned grid, cudaStream_t st, A... a) { nm_mask_kernel<M><<<grid, kThreads, 0, st>>>(a...); }
};
template <int M> struct RedistLaunch {
    template <typename... A>
    static void launch(unsigned grid, cudaStream_t st, A... a) { redistribute_kernel<M><<<grid, kThreads, 0, st>>>(a...); }
};

int nm_mask_impl(const float* s, uint8_t* mask, size_t N, int n, int m, int strategy, int rounds, int permute,
                 cudaStream_t st) {
    int rc = check_nm(N, n, m);
    if (rc) return rc;
    if (!s || !mask) return fail(TB_ERR_ARG, "tb_nm_mask: null pointer");
    if (strategy < TB_MASK_TOPN || strategy > TB_MASK_ITERATIVE) return fail(TB_ERR_ARG, "bad strategy %d", strategy);
    if ((rc = require_device(nullptr))) return rc;
    const uint8_t* lut = nullptr;
    if (strategy != TB_MASK_OPTIMAL && (rc = topn_table(n, m, &lut))) return rc;
    const size_t G = N / static_cast<size_t>(m);
    rc = launch_by_m<NmMaskLaunch>(m, G, st, s, mask, G, n, strategy, rounds, permute, lut);
    return rc ? rc : check_launch("nm_mask_kernel");
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

int tb_fisher_diagonal(const float* gradients, float* fisher_diag, size_t B, size_t N, void* stream) {
    if (N == 0) return TB_OK;  // reference launcher returns early on empty input (src/kernels.cu:347)
    if (!gradients || !fisher_diag) return fail(TB_ERR_ARG, "tb_fisher_diagonal: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    fisher_diagonal_kernel<<<grid_for(N), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(gradients, fisher_diag, B, N);
    return check_launch("fisher_diagonal_kernel");
}

int tb_fisher_accumulate(float* fisher_diag, const float* gradients, size_t N, float alpha, void* stream) {
    if (N == 0) return TB_OK;
    if (!gradients || !fisher_diag) return fail(TB_ERR_ARG, "tb_fisher_accumulate: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    fisher_accumulate_kernel<<<grid_for(N), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(fisher_diag, gradients, N, alpha);
    return check_launch("fisher_accumulate_kernel");
}

int tb_fisher_beta_decay(float* fisher_diag, float beta, size_t N, void* stream) {
    if (N == 0) return TB_OK;
    if (!fisher_diag) return fail(TB_ERR_ARG, "tb_fisher_beta_decay: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    beta_decay_kernel<<<grid_for(N), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(fisher_diag, beta, N);
    return check_launch("beta_decay_kernel");
}

int tb_fisher_ema_step(float* fisher, const void* gradients, int g_dtype, size_t N, float alpha, float beta,
                       int first_step, void* stream) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty gradient tensor");
    if (!fisher || !gradients) return fail(TB_ERR_ARG, "tb_fisher_ema_step: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    const float one_m_beta = 1.0f - beta;
    const float contrib = alpha * one_m_beta;
    auto st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_for(N);
    switch (g_dtype) {
    case TB_F32: ema_step_kernel<TB_F32><<<grid, kThreads, 0, st>>>(fisher, gradients, N, alpha, beta, contrib, first_step); break;
    case TB_BF16: ema_step_kernel<TB_BF16><<<grid, kThreads, 0, st>>>(fisher, gradients, N, alpha, beta, contrib, first_step); break;
    case TB_F16: ema_step_kernel<TB_F16><<<grid, kThreads, 0, st>>>(fisher, gradients, N, alpha, beta, contrib, first_step); break;
    default: return fail(TB_ERR_ARG, "bad gradient dtype %d", g_dtype);
    }
    return check_launch("ema_step_kernel");
}

int tb_importance(const void* weights, int w_dtype, const float* fisher, float* importance_out, size_t N,
                  float damping, int mode, void* stream) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty tensor");
    if (!weights || !importance_out) return fail(TB_ERR_ARG, "tb_importance: null pointer");
    if (mode < TB_IMP_OBD || mode > TB_IMP_NORMALIZED) return fail(TB_ERR_ARG, "bad importance mode %d", mode);
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_for(N);
    switch (w_dtype) {
    case TB_F32: importance_kernel<TB_F32><<<grid, kThreads, 0, st>>>(weights, fisher, importance_out, N, damping, mode); break;
    case TB_BF16: importance_kernel<TB_BF16><<<grid, kThreads, 0, st>>>(weights, fisher, importance_out, N, damping, mode); break;
    case TB_F16: importance_kernel<TB_F16><<<grid, kThreads, 0, st>>>(weights, fisher, importance_out, N, damping, mode); break;
    default: return fail(TB_ERR_ARG, "bad weight dtype %d", w_dtype);
    }
    return check_launch("importance_kernel");
}

int tb_ehap_importance(const float* weights, const float* fisher_diag, float* importance_out, size_t N,
                       float damping, void* stream) {
    if (N == 0) return TB_OK;
    return tb_importance(weights, TB_F32, fisher_diag, importance_out, N, damping, TB_IMP_OBD, stream);
}

int tb_nm_mask(const float* importance_in, uint8_t* mask_out, size_t N, int n, int m, int strategy, int rounds,
               int permute, void* stream) {
    return nm_mask_impl(importance_in, mask_out, N, n, m, strategy, rounds, permute, static_cast<cudaStream_t>(stream));
}

int tb_nm_mask_2_4(const float* importance_in, uint8_t* mask_out, size_t N, void* stream) {
    if (N < 4) return TB_OK;  // src/kernels.cu:399
    return nm_mask_impl(importance_in, mask_out, N - N % 4, 2, 4, TB_MASK_TOPN, 0, 0, static_cast<cudaStream_t>(stream));
}

int tb_nm_mask_generic(const float* importance_in, uint8_t* mask_out, size_t N_elements, int group_n, int group_m,
                       void* stream) {
    if (group_m <= 0 || N_elements < static_cast<size_t>(group_m)) return TB_OK;  // src/kernels.cu:414
    const size_t an = N_elements - N_elements % static_cast<size_t>(group_m);
    return nm_mask_impl(importance_in, mask_out, an, group_n, group_m, TB_MASK_TOPN, 0, 0,
                        static_cast<cudaStream_t>(stream));
}

int tb_apply_mask(float* weights, const uint8_t* mask, size_t N, int group_m, void* stream) {
    if (N == 0 || group_m <= 0) return TB_OK;  // src/kernels.cu:429
    if (!weights || !mask) return fail(TB_ERR_ARG, "tb_apply_mask: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    const size_t an = N - N % static_cast<size_t>(group_m);
    apply_mask_kernel<<<grid_for(an), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(weights, mask, an, group_m);
    return check_launch("apply_mask_kernel");
}

int tb_redistribute(float* weights, const uint8_t* mask, const float* importance_in, size_t N, int m, int mode,
                    void* stream) {
    if (mode == TB_REDIST_NONE) return TB_OK;
    if (mode < TB_REDIST_NONE || mode > TB_REDIST_UNIFORM) return fail(TB_ERR_ARG, "bad redistribution mode %d", mode);
    if (m <= 0) return fail(TB_ERR_CONFIG, "M=%d", m);
    if (m > 8) return fail(TB_ERR_UNSUPPORTED, "M=%d > 8", m);
    if (!weights || !mask || !importance_in) return fail(TB_ERR_ARG, "tb_redistribute: null pointer");
    const size_t G = N / static_cast<size_t>(m);
    if (G == 0) return TB_OK;
    int rc = require_device(nullptr);
    if (rc) return rc;
    if (m == 1) return fail(TB_ERR_UNSUPPORTED, "M=1");
    rc = launch_by_m<RedistLaunch>(m, G, static_cast<cudaStream_t>(stream), weights, mask, importance_in, G, mode);
    return rc ? rc : check_launch("redistribute_kernel");
}

}  // extern "C"

namespace tb {
namespace {
template <int DT>
__global__ void decode_kernel(const void* __restrict__ in, float* __restrict__ out, size_t N) {
    TB_GRID_STRIDE(i, N) out[i] = Dtype<DT>::load(in, i);
}
}  // namespace
}  // namespace tb

// Safetensors element widening of load_safetensor (src/main.cpp:204-250) on the
// device: BF16 exactly, F16 with the reference's handling of exponent 0, F32 copied.
extern "C" int tb_decode_to_f32(const void* in, int dtype, float* out, size_t N, void* stream) {
    if (N == 0) return TB_OK;
    if (!in || !out) return fail(TB_ERR_ARG, "tb_decode_to_f32: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_for(N);
    switch (dtype) {
    case TB_F32: decode_kernel<TB_F32><<<grid, kThreads, 0, st>>>(in, out, N); break;
    case TB_BF16: decode_kernel<TB_BF16><<<grid, kThreads, 0, st>>>(in, out, N); break;
    case TB_F16: decode_kernel<TB_F16><<<grid, kThreads, 0, st>>>(in, out, N); break;
    default: return fail(TB_ERR_ARG, "bad dtype %d", dtype);
    }
    return check_launch("decode_kernel");
}

// ---- sample-split Fisher partial sums ----------------------------------------
// When calibration samples are split across ranks, the EMA
//   F_S = beta F_{S-1} + (alpha (1-beta)) g_{S-1}^2,  F_1 = alpha g_0^2
// is rewritten as the weighted sum F = sum_t c_t g_t^2 with
//   c_0 = alpha beta^(S-1),  c_t = alpha (1-beta) beta^(S-1-t)  (t >= 1),
// which each rank evaluates over its own samples before one all-reduce.  The
// association differs from the serial recurrence, so F agrees with it to
// FP32 rounding, not bit for bit.
namespace tb {
namespace {
constexpr int kMaxWeights = 64;
struct SampleWeights {
    float c[kMaxWeights];
};

template <int GDT>
__global__ void weighted_sq_sum_kernel(float* __restrict__ F, const void* __restrict__ g, size_t S, size_t gstride,
                                       size_t N, SampleWeights cw, int accumulate) {
    TB_GRID_STRIDE(i, N) {
        float acc = accumulate ? F[i] : 0.0f;
        for (size_t s = 0; s < S; ++s) {
            const float x = Dtype<GDT>::load(g, s * gstride + i);
            acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(cw.c[s], x), x));
        }
        F[i] = acc;
    }
}
}  // namespace
}  // namespace tb

extern "C" int tb_fisher_weighted_sum(float* fisher, const void* gradients, int g_dtype, size_t S, size_t g_stride,
                                      size_t N, const float* weights_host, int accumulate, void* stream) {
    if (N == 0) return TB_OK;
    if (!fisher || (S && (!gradients || !weights_host))) return fail(TB_ERR_ARG, "tb_fisher_weighted_sum: null pointer");
    if (g_dtype < TB_F32 || g_dtype > TB_BF16) return fail(TB_ERR_ARG, "bad gradient dtype %d", g_dtype);
    const size_t stride = g_stride ? g_stride : N;
    if (stride < N) return fail(TB_ERR_ARG, "g_stride < N");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const unsigned grid = grid_for(N);
    const int esize = g_dtype == TB_F32 ? 4 : 2;
    size_t done = 0;
    do {  // batches of up to 64 samples, the first overwriting unless accumulating
        const size_t n = std::min<size_t>(S - done, kMaxWeights);
        SampleWeights cw{};
        for (size_t k = 0; k < n; ++k) cw.c[k] = weights_host[done + k];
        const void* gp = S ? static_cast<const char*>(gradients) + done * stride * esize : gradients;
        const int acc = (done > 0 || accumulate) ? 1 : 0;
        switch (g_dtype) {
        case TB_F32: weighted_sq_sum_kernel<TB_F32><<<grid, kThreads, 0, st>>>(fisher, gp, n, stride, N, cw, acc); break;
        case TB_BF16: weighted_sq_sum_kernel<TB_BF16><<<grid, kThreads, 0, st>>>(fisher, gp, n, stride, N, cw, acc); break;
        default: weighted_sq_sum_kernel<TB_F16><<<grid, kThreads, 0, st>>>(fisher, gp, n, stride, N, cw, acc); break;
        }
        if ((rc = check_launch("weighted_sq_sum_kernel"))) return rc;
        done += n;
    } while (done < S);
    return TB_OK;
}

#pragma once

/// @file kernels.hpp
/// @brief The reference's seven kernel launchers, as thin C++ wrappers over the C ABI.
///
/// Same names and arguments as include/tensorbit/core/kernels.hpp:24-124 of the
/// reference, so existing callers still compile and link.  Like the reference
/// launchers (which abort through CUDA_CHECK, common.hpp:38-49), a failing call
/// prints the library's error text and aborts; callers that want a status code
/// use the tb_* functions of tb_kernels.h directly.

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "tb_kernels.h"

namespace tensorbit::core::kernels {

namespace detail {
inline void check(int rc, const char* what) {
    if (rc != TB_OK) {
        std::fprintf(stderr, "[CUDA ERROR] %s: %s (status %d)\n", what, tb_last_error(), rc);
        std::abort();
    }
}
}  // namespace detail

inline void launch_fisher_diagonal(const float* gradients, float* fisher_diag, std::size_t B, std::size_t N,
                                   void* stream) {
    detail::check(tb_fisher_diagonal(gradients, fisher_diag, B, N, stream), "launch_fisher_diagonal");
}

inline void launch_fisher_accumulate(float* fisher_diag, const float* gradients, std::size_t N, float alpha,
                                     void* stream) {
    detail::check(tb_fisher_accumulate(fisher_diag, gradients, N, alpha, stream), "launch_fisher_accumulate");
}

inline void launch_fisher_beta_decay(float* fisher_diag, float beta, std::size_t N, void* stream) {
    detail::check(tb_fisher_beta_decay(fisher_diag, beta, N, stream), "launch_fisher_beta_decay");
}

inline void launch_ehap_importance(const float* weights, const float* fisher_diag, float* importance,
                                   std::size_t N, float damping, void* stream) {
    detail::check(tb_ehap_importance(weights, fisher_diag, importance, N, damping, stream), "launch_ehap_importance");
}

inline void launch_nm_mask_2_4(const float* importance, uint8_t* mask_out, std::size_t N, void* stream) {
    detail::check(tb_nm_mask_2_4(importance, mask_out, N, stream), "launch_nm_mask_2_4");
}

inline void launch_nm_mask_generic(const float* importance, uint8_t* mask_out, std::size_t N_elements,
                                   int group_n, int group_m, void* stream) {
    detail::check(tb_nm_mask_generic(importance, mask_out, N_elements, group_n, group_m, stream),
                  "launch_nm_mask_generic");
}

inline void launch_apply_mask(float* weights, const uint8_t* mask, std::size_t N, int group_m, void* stream) {
    detail::check(tb_apply_mask(weights, mask, N, group_m, stream), "launch_apply_mask");
}

}  // namespace tensorbit::core::kernels

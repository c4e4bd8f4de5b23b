#pragma once

/// @file coring.hpp
/// @brief CORING N:M structured sparsity on the GPU, with the reference's API.
///
/// Same types, configuration and member functions as the reference's
/// CORINGPruner (include/tensorbit/core/coring.hpp:29-460).  Every loop runs as
/// a device kernel through the C ABI; host tensors are staged through device
/// buffers and copied back, so results are the same whichever side the
/// tensors live on.  Results are bit-identical to the reference's CPU path,
/// including top-N tie order.
///
/// Differences from the reference, all where its device branches were
/// unreachable or could not run:
///   * masks of every strategy are produced on the device (the reference's GPU
///     branch covered float top-N only, coring.hpp:111-123);
///   * redistribute() accepts device tensors (reference: kCudaNotAvailable,
///     coring.hpp:234-235);
///   * M > 8 returns kInvalidNMConfig: the mask stores one byte per group
///     (coring.hpp:388-390), so the reference silently drops bits above 7;
///   * double tensors return kCudaNotAvailable: the device path is FP32.

#include <cstddef>
#include <cstdint>
#include <span>
#include <type_traits>

#include "tb_kernels.h"
#include "tensorbit/core/staging.hpp"
#include "tensorbit/core/tensor.hpp"

namespace tensorbit::core {

enum class CORINGError : uint8_t {
    kOk = 0,
    kShapeMismatch = 1,
    kZeroSizeTensor = 2,
    kInvalidNMConfig = 3,
    kCudaNotAvailable = 4,
};

enum class MaskStrategy : uint8_t { kTopN = 0, kOptimal = 1, kIterative = 2 };
enum class RedistMode : uint8_t { kNone = 0, kProportional = 1, kUniform = 2 };

struct CORINGConfig {
    int N = 2;
    int M = 4;
    bool use_cuda = true;
    MaskStrategy mask_strategy = MaskStrategy::kTopN;
    RedistMode redist_mode = RedistMode::kNone;
    int iterative_rounds = 3;
    bool permute_weights = false;
    bool hardware_aware_layout = false;  // a no-op for row-major layouts, as in the reference
};

template <FloatingPoint F>
class CORINGPruner {
public:
    explicit CORINGPruner(CORINGConfig config) : config_(config) {}
    CORINGPruner(const CORINGPruner&) = delete;
    CORINGPruner& operator=(const CORINGPruner&) = delete;
    CORINGPruner(CORINGPruner&&) noexcept = default;
    CORINGPruner& operator=(CORINGPruner&&) noexcept = default;

    /// One byte per group of M written to the first N/M bytes of out_mask
    /// (coring.hpp:90-165).
    auto generate_nm_mask(const TensorDense<F>& importance, TensorDense<uint8_t>& out_mask)
        -> Result<void, CORINGError> {
        if (importance.empty() || out_mask.empty()) return unexpected(CORINGError::kZeroSizeTensor);
        if (importance.size() != out_mask.size()) return unexpected(CORINGError::kShapeMismatch);
        if (auto v = validate_config(importance.size()); !v) return unexpected(v.error());
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(CORINGError::kCudaNotAvailable);
        } else {
            detail::Staged<float> s(importance);
            detail::Staged<uint8_t> mk(out_mask, false);
            int rc = s.status() ? s.status() : mk.status();
            if (!rc)
                rc = tb_nm_mask(s.get(), mk.get(), importance.size(), config_.N, config_.M,
                                static_cast<int>(config_.mask_strategy), config_.iterative_rounds,
                                config_.permute_weights ? 1 : 0, nullptr);
            if (!rc) rc = detail::sync();
            if (!rc && out_mask.device() == DeviceLocation::kHost) rc = commit_prefix(mk, out_mask, importance.size() / config_.M);
            return map(rc);
        }
    }

    /// Zeroes pruned weights; returns the analytic count G*(M-N) (coring.hpp:170-223).
    auto apply_mask(TensorDense<F>& weights, const TensorDense<uint8_t>& mask) -> Result<std::size_t, CORINGError> {
        if (weights.empty() || mask.empty()) return unexpected(CORINGError::kZeroSizeTensor);
        if (weights.size() != mask.size()) return unexpected(CORINGError::kShapeMismatch);
        const std::size_t M = static_cast<std::size_t>(config_.M);
        const std::size_t an = weights.size() / M * M;
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(CORINGError::kCudaNotAvailable);
        } else {
            detail::Staged<float> w(weights, true);
            detail::Staged<uint8_t> mk(mask);
            int rc = w.status() ? w.status() : mk.status();
            if (!rc) rc = tb_apply_mask(w.get(), mk.get(), an, config_.M, nullptr);
            if (!rc) rc = detail::sync();
            if (!rc) rc = w.commit();
            if (rc) return unexpected(to_error(rc));
            return (an / M) * static_cast<std::size_t>(config_.M - config_.N);
        }
    }

    /// Magnitude redistribution of the weights as they are (coring.hpp:228-294).
    auto redistribute(TensorDense<F>& weights, const TensorDense<uint8_t>& mask, const TensorDense<F>& importance)
        -> Result<void, CORINGError> {
        if (config_.redist_mode == RedistMode::kNone) return {};
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(CORINGError::kCudaNotAvailable);
        } else {
            detail::Staged<float> w(weights, true);
            detail::Staged<uint8_t> mk(mask);
            detail::Staged<float> s(importance);
            int rc = w.status() ? w.status() : (mk.status() ? mk.status() : s.status());
            if (!rc)
                rc = tb_redistribute(w.get(), mk.get(), s.get(), weights.size(), config_.M,
                                     static_cast<int>(config_.redist_mode), nullptr);
            if (!rc) rc = detail::sync();
            if (!rc) rc = w.commit();
            return map(rc);
        }
    }

    /// generate_nm_mask -> apply_mask -> redistribute (coring.hpp:299-313).
    auto prune(const TensorDense<F>& importance, TensorDense<F>& weights) -> Result<std::size_t, CORINGError> {
        if (importance.size() != weights.size()) return unexpected(CORINGError::kShapeMismatch);
        TensorDense<uint8_t> mask(importance.shape(), weights.device());
        auto mr = generate_nm_mask(importance, mask);
        if (!mr) return unexpected(mr.error());
        auto ar = apply_mask(weights, mask);
        if (!ar) return unexpected(ar.error());
        redistribute(weights, mask, importance);
        return ar.value();
    }

    [[nodiscard]] const CORINGConfig& config() const noexcept { return config_; }

private:
    auto validate_config(std::size_t n) const -> Result<void, CORINGError> {
        if (config_.N <= 0 || config_.M <= 0) return unexpected(CORINGError::kInvalidNMConfig);
        if (config_.N >= config_.M) return unexpected(CORINGError::kInvalidNMConfig);
        if (n > 0 && n % static_cast<std::size_t>(config_.M) != 0) return unexpected(CORINGError::kShapeMismatch);
        if (config_.M > 8) return unexpected(CORINGError::kInvalidNMConfig);
        return {};
    }

    static CORINGError to_error(int rc) {
        switch (detail::classify(rc)) {
        case detail::DevStatus::kShape: return CORINGError::kShapeMismatch;
        case detail::DevStatus::kZero: return CORINGError::kZeroSizeTensor;
        case detail::DevStatus::kConfig: return CORINGError::kInvalidNMConfig;
        default: return CORINGError::kCudaNotAvailable;
        }
    }
    static Result<void, CORINGError> map(int rc) {
        if (rc == TB_OK) return {};
        return unexpected(to_error(rc));
    }
    // Only the group bytes are written; the rest of the caller's buffer keeps
    // its contents, as with the reference's host loop.
    static int commit_prefix(detail::Staged<uint8_t>& mk, TensorDense<uint8_t>& out, std::size_t groups) {
        int rc = tb_memcpy_d2h(out.data(), mk.get(), groups, nullptr);
        return rc ? rc : tb_stream_sync(nullptr);
    }

    CORINGConfig config_;
};

}  // namespace tensorbit::core

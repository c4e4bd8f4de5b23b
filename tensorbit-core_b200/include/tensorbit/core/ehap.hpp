#pragma once

/// @file ehap.hpp
/// @brief Efficient Hessian-Aware Pruning on the GPU, with the reference's API.
///
/// Same types, configuration and members as the reference's EHAPPruner
/// (include/tensorbit/core/ehap.hpp:41-737): EMA Fisher diagonal, OBD / OBS /
/// Normalized importance, global-threshold masks, one-shot / iterative /
/// blockwise-OBS pruning and weight compensation.  Every loop runs on the
/// device through the C ABI; host tensors are staged through device buffers.
/// FP32 results are bit-identical to the reference's CPU path (block OBS
/// follows the same operation order; see tb_block_obs).
///
/// Differences, where the reference's device branches could not run:
///   * select_pruning_mask, compensate_weights, prune and store_gradient accept
///     device tensors (reference: kCudaNotAvailable, ehap.hpp:125-126,298-299,
///     374-375,412-413);
///   * the Fisher state lives on the side of the first gradient tensor, as in
///     the reference, and is updated in place on the device;
///   * double tensors return kCudaNotAvailable: the device path is FP32.

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <span>
#include <type_traits>
#include <vector>

#include "tb_kernels.h"
#include "tensorbit/core/staging.hpp"
#include "tensorbit/core/tensor.hpp"

namespace tensorbit::core {

enum class EHAPError : uint8_t {
    kOk = 0,
    kShapeMismatch = 1,
    kZeroSizeTensor = 2,
    kInvalidConfig = 3,
    kCudaNotAvailable = 4,
};

enum class ImportanceMode : uint8_t { kOBD = 0, kOBS = 1, kNormalized = 2 };
enum class PruneStrategy : uint8_t { kOneShot = 0, kIterative = 1, kBlockOBS = 2 };
enum class CompensationMode : uint8_t { kNone = 0, kBias = 1, kRedist = 2 };

struct EHAPConfig {
    float damping = 0.01f;
    bool use_diagonal_fisher = true;
    float sparsity_ratio = 0.5f;  // fraction KEPT by select_pruning_mask
    float ema_decay = 0.99f;
    std::size_t accumulation_steps = 100;
    ImportanceMode importance_mode = ImportanceMode::kOBD;
    PruneStrategy prune_strategy = PruneStrategy::kOneShot;
    std::size_t prune_rounds = 5;
    float prune_fraction_per_round = 0.2f;
    CompensationMode compensation_mode = CompensationMode::kNone;
    bool normalize_fisher = false;
    std::size_t obs_block_size = 128;
    float obs_off_diag_alpha = 0.01f;
    std::size_t gradient_history_size = 4;
};

template <FloatingPoint F>
class EHAPPruner {
public:
    explicit EHAPPruner(EHAPConfig config) : config_(config), step_count_(0) {}
    EHAPPruner(const EHAPPruner&) = delete;
    EHAPPruner& operator=(const EHAPPruner&) = delete;
    EHAPPruner(EHAPPruner&&) noexcept = default;
    EHAPPruner& operator=(EHAPPruner&&) noexcept = default;

    /// Keeps a copy of the gradient in a ring of the last K snapshots
    /// (ehap.hpp:121-143).  Snapshots live on the device.
    auto store_gradient(const TensorDense<F>& g) -> Result<void, EHAPError> {
        if (g.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        const std::size_t K = config_.gradient_history_size;
        if (K == 0) return {};
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            if (g_hist_.size() >= K) g_hist_.erase(g_hist_.begin());
            TensorDense<F> snap(g.shape(), DeviceLocation::kDevice);
            const int rc = g.device() == DeviceLocation::kDevice
                               ? tb_memcpy_d2d(snap.data(), g.data(), g.bytes(), nullptr)
                               : tb_memcpy_h2d(snap.data(), g.data(), g.bytes(), nullptr);
            if (rc || detail::sync()) return unexpected(EHAPError::kCudaNotAvailable);
            g_hist_.push_back(std::move(snap));
            return {};
        }
    }

    /// One EMA step of the Fisher diagonal (ehap.hpp:148-201).
    auto accumulate_fisher(const TensorDense<F>& g, F alpha) -> Result<void, EHAPError> {
        if (g.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        if (!config_.use_diagonal_fisher) return {};
        if (fisher_diag_.empty()) {
            fisher_diag_ = TensorDense<F>(g.shape(), g.device());
            step_count_ = 0;
        }
        if (fisher_diag_.size() != g.size()) return unexpected(EHAPError::kShapeMismatch);
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            detail::Staged<float> f(fisher_diag_, step_count_ > 0);
            detail::Staged<float> gd(g);
            int rc = f.status() ? f.status() : gd.status();
            if (!rc)
                rc = tb_fisher_ema_step(f.get(), gd.get(), TB_F32, g.size(), alpha, config_.ema_decay,
                                        step_count_ == 0 ? 1 : 0, nullptr);
            if (!rc) rc = detail::sync();
            if (!rc) rc = f.commit();
            if (rc) return unexpected(to_error(rc));
            ++step_count_;
            return {};
        }
    }

    /// OBD / OBS / Normalized scores (ehap.hpp:206-285).
    auto compute_importance(const TensorDense<F>& weights, TensorDense<F>& out) -> Result<void, EHAPError> {
        if (weights.empty() || out.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        if (weights.size() != out.size()) return unexpected(EHAPError::kShapeMismatch);
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            const bool have_f = !fisher_diag_.empty();
            detail::Staged<float> f(fisher_diag_, true);
            detail::Staged<float> w(weights);
            detail::Staged<float> s(out, false);
            int rc = f.status() ? f.status() : (w.status() ? w.status() : s.status());
            if (!rc && have_f && config_.normalize_fisher) {
                rc = tb_fisher_normalize(f.get(), fisher_diag_.size(), nullptr);
                if (!rc) rc = detail::sync();
                if (!rc) rc = f.commit();
            }
            if (!rc)
                rc = tb_importance(w.get(), TB_F32, have_f ? f.get() : nullptr, s.get(), weights.size(),
                                   config_.damping, static_cast<int>(config_.importance_mode), nullptr);
            if (!rc) rc = detail::sync();
            if (!rc) rc = s.commit();
            return map(rc);
        }
    }

    /// Global threshold: keep the sparsity_ratio fraction with the largest
    /// scores; returns the number pruned (ehap.hpp:290-329).
    auto select_pruning_mask(const TensorDense<F>& importance, TensorDense<uint8_t>& out_mask)
        -> Result<std::size_t, EHAPError> {
        if (importance.empty() || out_mask.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        if (importance.size() != out_mask.size()) return unexpected(EHAPError::kShapeMismatch);
        const float sp = config_.sparsity_ratio;
        if (sp <= 0.0f || sp >= 1.0f) return unexpected(EHAPError::kInvalidConfig);
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            detail::Staged<float> s(importance);
            detail::Staged<uint8_t> mk(out_mask, false);
            int rc = s.status() ? s.status() : mk.status();
            float thr = 0.0f;
            uint64_t pruned = 0;
            if (!rc) rc = tb_threshold_select(s.get(), importance.size(), sp, mk.get(), &thr, &pruned, nullptr);
            if (!rc) rc = mk.commit();
            if (rc) return unexpected(to_error(rc));
            return static_cast<std::size_t>(pruned);
        }
    }

    /// Zeroes weights whose mask byte is 0; returns how many (ehap.hpp:334-362).
    auto apply_mask(TensorDense<F>& weights, const TensorDense<uint8_t>& mask) -> Result<std::size_t, EHAPError> {
        if (weights.empty() || mask.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        if (weights.size() != mask.size()) return unexpected(EHAPError::kShapeMismatch);
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            detail::Staged<float> w(weights, true);
            detail::Staged<uint8_t> mk(mask);
            int rc = w.status() ? w.status() : mk.status();
            uint64_t pruned = 0;
            if (!rc) rc = tb_ehap_apply_mask(w.get(), mk.get(), weights.size(), &pruned, nullptr);
            if (!rc) rc = w.commit();
            if (rc) return unexpected(to_error(rc));
            return static_cast<std::size_t>(pruned);
        }
    }

    /// kBias / kRedist compensation (ehap.hpp:367-403).
    auto compensate_weights(TensorDense<F>& weights, const TensorDense<uint8_t>& mask, const TensorDense<F>& importance)
        -> Result<void, EHAPError> {
        if (config_.compensation_mode == CompensationMode::kNone) return {};
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            detail::Staged<float> w(weights, true);
            detail::Staged<uint8_t> mk(mask);
            detail::Staged<float> s(importance);
            int rc = w.status() ? w.status() : (mk.status() ? mk.status() : s.status());
            if (!rc)
                rc = tb_compensate(w.get(), mk.get(), s.get(), weights.size(),
                                   static_cast<int>(config_.compensation_mode), nullptr);
            if (!rc) rc = detail::sync();
            if (!rc) rc = w.commit();
            return map(rc);
        }
    }

    /// Strategy dispatch (ehap.hpp:408-420).
    auto prune(TensorDense<F>& weights) -> Result<std::size_t, EHAPError> {
        if (weights.empty()) return unexpected(EHAPError::kZeroSizeTensor);
        if (config_.prune_strategy == PruneStrategy::kIterative) return prune_iterative(weights);
        if (config_.prune_strategy == PruneStrategy::kBlockOBS) return prune_block_obs(weights);
        return prune_one_shot(weights);
    }

    /// importance -> global mask -> apply -> compensate (ehap.hpp:425-439).
    auto prune_one_shot(TensorDense<F>& weights) -> Result<std::size_t, EHAPError> {
        TensorDense<F> imp(weights.shape(), DeviceLocation::kDevice);
        TensorDense<uint8_t> msk(weights.shape(), DeviceLocation::kDevice);
        auto r1 = compute_importance(weights, imp);
        if (!r1) return unexpected(r1.error());
        auto r2 = select_pruning_mask(imp, msk);
        if (!r2) return unexpected(r2.error());
        auto r3 = apply_mask(weights, msk);
        if (!r3) return unexpected(r3.error());
        compensate_weights(weights, msk, imp);
        return r3.value();
    }

    /// Cubic keep schedule over prune_rounds one-shot rounds (ehap.hpp:444-478).
    auto prune_iterative(TensorDense<F>& weights) -> Result<std::size_t, EHAPError> {
        const std::size_t rounds = config_.prune_rounds;
        const float target_sp = config_.sparsity_ratio;
        std::size_t total = 0;
        float cur_keep = 1.0f;
        for (std::size_t r = 0; r < rounds; ++r) {
            const float t = static_cast<float>(r + 1) / static_cast<float>(rounds);
            const float target_keep = target_sp + (1.0f - target_sp) * static_cast<float>(std::pow(1.0 - t, 3));
            float round_keep = target_keep / cur_keep;
            if (round_keep < 0.0f) round_keep = 0.0f;
            if (round_keep > 1.0f) round_keep = 1.0f;
            const float saved = config_.sparsity_ratio;
            config_.sparsity_ratio = round_keep;
            auto res = prune_one_shot(weights);
            config_.sparsity_ratio = saved;
            if (!res) return unexpected(res.error());
            total += res.value();
            cur_keep = round_keep;
        }
        return total;
    }

    /// Blockwise OBS with a diagonal + low-rank Hessian (ehap.hpp:502-704).
    auto prune_block_obs(TensorDense<F>& weights) -> Result<std::size_t, EHAPError> {
        if constexpr (!std::is_same_v<F, float>) {
            return unexpected(EHAPError::kCudaNotAvailable);
        } else {
            detail::Staged<float> w(weights, true);
            detail::Staged<float> f(fisher_diag_, true);
            int rc = w.status() ? w.status() : f.status();
            std::vector<const float*> hist;
            for (auto& h : g_hist_) hist.push_back(h.data());
            uint64_t pruned = 0;
            if (!rc)
                rc = tb_block_obs(w.get(), fisher_diag_.empty() ? nullptr : f.get(),
                                  hist.empty() ? nullptr : hist.data(), static_cast<int>(hist.size()),
                                  weights.size(), config_.obs_block_size, config_.sparsity_ratio,
                                  config_.damping, config_.obs_off_diag_alpha, &pruned, nullptr);
            if (!rc) rc = w.commit();
            if (rc) return unexpected(to_error(rc));
            return static_cast<std::size_t>(pruned);
        }
    }

    [[nodiscard]] const EHAPConfig& config() const noexcept { return config_; }
    [[nodiscard]] const TensorDense<F>& fisher_diagonal() const noexcept { return fisher_diag_; }
    [[nodiscard]] std::size_t step_count() const noexcept { return step_count_; }
    [[nodiscard]] const std::vector<TensorDense<F>>& gradient_history() const noexcept { return g_hist_; }
    void reset() {
        fisher_diag_ = TensorDense<F>{};
        g_hist_.clear();
        step_count_ = 0;
    }

private:
    static EHAPError to_error(int rc) {
        switch (detail::classify(rc)) {
        case detail::DevStatus::kShape: return EHAPError::kShapeMismatch;
        case detail::DevStatus::kZero: return EHAPError::kZeroSizeTensor;
        case detail::DevStatus::kConfig: return EHAPError::kInvalidConfig;
        default: return EHAPError::kCudaNotAvailable;
        }
    }
    static Result<void, EHAPError> map(int rc) {
        if (rc == TB_OK) return {};
        return unexpected(to_error(rc));
    }

    EHAPConfig config_;
    TensorDense<F> fisher_diag_;
    std::vector<TensorDense<F>> g_hist_;
    std::size_t step_count_;
};

}  // namespace tensorbit::core

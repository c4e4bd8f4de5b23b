#pragma once

/// @file staging.hpp
/// @brief Device views of host or device tensors for the pruners.
///
/// The pruners run every loop on the GPU.  A tensor that already lives on the
/// device is used in place; a host tensor is copied to a device buffer for the
/// call (and copied back if the call writes it).  All work goes on the legacy
/// default stream and each pruner call synchronises before returning, as the
/// reference's device branches do (CUDA_SYNC_CHECK after every launch).

#include <cstddef>

#include "tb_kernels.h"
#include "tensorbit/core/tensor.hpp"

namespace tensorbit::core::detail {

/// Status of the last C-ABI call chain, folded into the pruners' error enums.
enum class DevStatus { kOk, kShape, kZero, kConfig, kDevice };

inline DevStatus classify(int rc) {
    switch (rc) {
    case TB_OK: return DevStatus::kOk;
    case TB_ERR_SHAPE: return DevStatus::kShape;
    case TB_ERR_ZERO_SIZE: return DevStatus::kZero;
    case TB_ERR_CONFIG: return DevStatus::kConfig;
    default: return DevStatus::kDevice;
    }
}

template <typename T>
class Staged {
public:
    /// Read-only view.
    explicit Staged(const TensorDense<T>& t) : host_(nullptr), src_(&t) { init(true); }
    /// Writable view; `upload` copies current contents in, commit() copies back.
    Staged(TensorDense<T>& t, bool upload) : host_(&t), src_(&t) { init(upload); }

    Staged(const Staged&) = delete;
    Staged& operator=(const Staged&) = delete;
    ~Staged() { if (owned_) tb_free(dev_); }

    [[nodiscard]] T* get() const noexcept { return dev_; }
    [[nodiscard]] int status() const noexcept { return rc_; }

    /// Copies a staged host tensor back (no-op for device tensors).
    int commit() {
        if (rc_ != TB_OK || !owned_ || !host_) return rc_;
        int rc = tb_memcpy_d2h(host_->data(), dev_, host_->bytes(), nullptr);
        if (rc == TB_OK) rc = tb_stream_sync(nullptr);
        return rc;
    }

private:
    void init(bool upload) {
        if (src_->device() == DeviceLocation::kDevice || src_->empty()) {
            dev_ = const_cast<T*>(src_->data());
            return;
        }
        void* p = nullptr;
        rc_ = tb_malloc(&p, src_->bytes());
        if (rc_ != TB_OK) return;
        dev_ = static_cast<T*>(p);
        owned_ = true;
        if (upload) rc_ = tb_memcpy_h2d(dev_, src_->data(), src_->bytes(), nullptr);
    }

    TensorDense<T>* host_;
    const TensorDense<T>* src_;
    T* dev_ = nullptr;
    bool owned_ = false;
    int rc_ = TB_OK;
};

/// Scratch device buffer freed on scope exit.
template <typename T>
class DeviceBuffer {
public:
    explicit DeviceBuffer(std::size_t n) {
        void* p = nullptr;
        rc_ = n ? tb_malloc(&p, n * sizeof(T)) : TB_OK;
        ptr_ = static_cast<T*>(p);
    }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { tb_free(ptr_); }
    [[nodiscard]] T* get() const noexcept { return ptr_; }
    [[nodiscard]] int status() const noexcept { return rc_; }

private:
    T* ptr_ = nullptr;
    int rc_ = TB_OK;
};

inline int sync() { return tb_stream_sync(nullptr); }

}  // namespace tensorbit::core::detail

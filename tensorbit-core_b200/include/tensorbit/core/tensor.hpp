#pragma once

/// @file tensor.hpp
/// @brief Owning dense tensor on the host or on the current CUDA device.
///
/// Same interface as the reference TensorDense (include/tensorbit/core/tensor.hpp:74-261).
/// The difference is where device memory comes from: the reference allocates
/// with cudaMalloc only when the including file is compiled by nvcc
/// (tensor.hpp:97-104), so the host-compiled pruners could never create a
/// device tensor.  Here device memory is obtained through the C ABI
/// (tb_malloc / tb_free / tb_memcpy_*), so plain C++ translation units create,
/// fill and read device tensors.  Device buffers are zero-initialised, like
/// the host ones (`new T[n]()`).

#include <array>
#include <concepts>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <type_traits>
#include <utility>

#include "tb_kernels.h"
#include "tensorbit/core/common.hpp"

namespace tensorbit::core {

template <typename T>
concept FloatingPoint = std::is_floating_point_v<T>;

template <typename T>
concept TensorType = requires(T t) {
    typename T::value_type;
    { t.data() } -> std::same_as<typename T::value_type*>;
    { t.size() } -> std::convertible_to<std::size_t>;
    { t.shape() } -> std::convertible_to<std::span<const std::size_t>>;
    { t.rank() } -> std::convertible_to<std::size_t>;
};

enum class DeviceLocation : uint8_t { kHost = 0, kDevice = 1 };

template <typename T>
class TensorDense {
public:
    using value_type = T;
    static constexpr std::size_t kMaxRank = 8;

    TensorDense() = default;

    explicit TensorDense(std::span<const std::size_t> dims, DeviceLocation dev = DeviceLocation::kHost)
        : device_(dev) {
        TENSORBIT_CHECK(dims.size() <= kMaxRank, "Tensor rank exceeds maximum supported dimensions");
        rank_ = dims.size();
        size_ = rank_ ? 1 : 0;
        for (std::size_t d = 0; d < rank_; ++d) {
            shape_[d] = dims[d];
            size_ *= dims[d];
        }
        if (size_ == 0) return;
        if (dev == DeviceLocation::kDevice) {
            void* p = nullptr;
            const int rc = tb_malloc(&p, size_ * sizeof(T));
            if (rc != TB_OK) {
                std::fprintf(stderr, "[TENSORBIT ERROR] device allocation of %zu bytes failed: %s\n",
                             size_ * sizeof(T), tb_last_error());
                std::abort();
            }
            TENSORBIT_CHECK(tb_memset(p, 0, size_ * sizeof(T), nullptr) == TB_OK &&
                                tb_stream_sync(nullptr) == TB_OK,
                            "device tensor initialisation failed");
            data_ = Owner(static_cast<T*>(p), &device_delete);
        } else {
            data_ = Owner(new T[size_](), &host_delete);
        }
    }

    /// Takes ownership of a host buffer allocated with new T[].
    TensorDense(T* data, std::span<const std::size_t> dims) : device_(DeviceLocation::kHost) {
        TENSORBIT_CHECK(dims.size() <= kMaxRank, "Tensor rank exceeds maximum supported dimensions");
        rank_ = dims.size();
        size_ = rank_ ? 1 : 0;
        for (std::size_t d = 0; d < rank_; ++d) {
            shape_[d] = dims[d];
            size_ *= dims[d];
        }
        data_ = Owner(data, &host_delete);
    }

    TensorDense(const TensorDense&) = delete;
    TensorDense& operator=(const TensorDense&) = delete;
    TensorDense(TensorDense&& o) noexcept
        : data_(std::move(o.data_)), shape_(o.shape_), size_(o.size_), rank_(o.rank_), device_(o.device_) {
        o.size_ = 0;
        o.rank_ = 0;
        o.device_ = DeviceLocation::kHost;
    }
    TensorDense& operator=(TensorDense&& o) noexcept {
        if (this != &o) {
            data_ = std::move(o.data_);
            shape_ = o.shape_;
            size_ = o.size_;
            rank_ = o.rank_;
            device_ = o.device_;
            o.size_ = 0;
            o.rank_ = 0;
            o.device_ = DeviceLocation::kHost;
        }
        return *this;
    }

    [[nodiscard]] T* data() noexcept { return data_.get(); }
    [[nodiscard]] const T* data() const noexcept { return data_.get(); }
    [[nodiscard]] std::size_t size() const noexcept { return size_; }
    [[nodiscard]] std::span<const std::size_t> shape() const noexcept { return {shape_.data(), rank_}; }
    [[nodiscard]] std::size_t rank() const noexcept { return rank_; }
    [[nodiscard]] DeviceLocation device() const noexcept { return device_; }
    [[nodiscard]] std::size_t bytes() const noexcept { return size_ * sizeof(T); }
    [[nodiscard]] bool empty() const noexcept { return size_ == 0; }

    /// Host-only element access (no bounds check).
    [[nodiscard]] T& operator[](std::size_t i) { return data_.get()[i]; }
    [[nodiscard]] const T& operator[](std::size_t i) const { return data_.get()[i]; }

    /// Copy of a host tensor on the current device (tensor.hpp:202-216).
    [[nodiscard]] TensorDense to_device() const {
        TENSORBIT_CHECK(device_ == DeviceLocation::kHost, "to_device() requires a host-resident source tensor");
        TensorDense r(shape(), DeviceLocation::kDevice);
        if (size_) {
            TENSORBIT_CHECK(tb_memcpy_h2d(r.data(), data(), bytes(), nullptr) == TB_OK &&
                                tb_stream_sync(nullptr) == TB_OK,
                            "host to device copy failed");
        }
        return r;
    }

    /// Copy of a device tensor in host memory (tensor.hpp:221-235).
    [[nodiscard]] TensorDense to_host() const {
        TENSORBIT_CHECK(device_ == DeviceLocation::kDevice, "to_host() requires a device-resident source tensor");
        TensorDense r(shape(), DeviceLocation::kHost);
        if (size_) {
            TENSORBIT_CHECK(tb_memcpy_d2h(r.data(), data(), bytes(), nullptr) == TB_OK &&
                                tb_stream_sync(nullptr) == TB_OK,
                            "device to host copy failed");
        }
        return r;
    }

private:
    using Owner = std::unique_ptr<T[], void (*)(T*)>;
    static void host_delete(T* p) { delete[] p; }
    static void device_delete(T* p) { tb_free(p); }

    Owner data_{nullptr, &host_delete};
    std::array<std::size_t, kMaxRank> shape_{};
    std::size_t size_ = 0;
    std::size_t rank_ = 0;
    DeviceLocation device_ = DeviceLocation::kHost;
};

template <typename T>
TensorDense(T*, std::span<const std::size_t>) -> TensorDense<T>;

}  // namespace tensorbit::core

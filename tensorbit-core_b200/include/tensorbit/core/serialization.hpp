#pragma once

/// @file serialization.hpp
/// @brief The unchanged .tb file format: writer and reader.
///
/// Layout (the reference's include/tensorbit/core/serialization.hpp:7-54, kept
/// byte for byte so files stay interchangeable):
///   [0, 4096)              packed little-endian TBHeader, unused bytes zero
///   [4096, 4096 + N*sz)    weights (FP32; FP64 for double tensors)
///   [masks_offset, ...)    one mask byte per group of M, bit i = keep element i
/// The kernels write the weight and mask sections directly, so a .tb image is
/// this header followed by two device buffers.

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <span>
#include <string>
#include <string_view>
#include <type_traits>

#include "tensorbit/core/common.hpp"
#include "tensorbit/core/tensor.hpp"

namespace tensorbit::core {

inline constexpr uint32_t kTBMagic = 0x31304254;  // "TB01"
inline constexpr uint32_t kTBVersion = 1;
inline constexpr std::size_t kTBHeaderSize = 4096;

#pragma pack(push, 1)
struct TBHeader {
    uint32_t magic = kTBMagic;
    uint32_t version = kTBVersion;
    uint32_t nm_n = 0;
    uint32_t nm_m = 0;
    uint64_t num_weights = 0;
    uint64_t num_mask_bytes = 0;
    uint64_t weights_offset = kTBHeaderSize;
    uint64_t masks_offset = kTBHeaderSize;
    uint8_t precision = 0;  // 0 = FP32, 1 = FP16, 2 = BF16, 3 = FP64
    uint8_t reserved[4047];
};
#pragma pack(pop)
static_assert(sizeof(TBHeader) == kTBHeaderSize, "TBHeader must be exactly 4096 bytes");

enum class TBError : uint8_t {
    kOk = 0,
    kFileOpen = 1,
    kFileWrite = 2,
    kFileRead = 3,
    kBadMagic = 4,
    kVersionMismatch = 5,
    kTruncated = 6,
    kSeekFailed = 7,
};

/// Header for `num_weights` weights of `elem_size` bytes and `num_mask_bytes`
/// mask bytes, as TBWriter::write fills it (serialization.hpp:115-134).
inline TBHeader make_tb_header(uint32_t nm_n, uint32_t nm_m, uint64_t num_weights, uint64_t num_mask_bytes,
                               std::size_t elem_size) {
    TBHeader h{};
    std::memset(&h, 0, sizeof(h));
    h.magic = kTBMagic;
    h.version = kTBVersion;
    h.nm_n = nm_n;
    h.nm_m = nm_m;
    h.num_weights = num_weights;
    h.num_mask_bytes = num_mask_bytes;
    h.weights_offset = kTBHeaderSize;
    h.masks_offset = kTBHeaderSize + num_weights * elem_size;
    h.precision = elem_size == 8 ? 3 : 0;
    return h;
}

class TBWriter {
public:
    TBWriter() = default;
    TBWriter(const TBWriter&) = delete;
    TBWriter& operator=(const TBWriter&) = delete;
    TBWriter(TBWriter&&) noexcept = default;
    TBWriter& operator=(TBWriter&&) noexcept = default;

    /// Writes header, weights and masks (host spans) to `path`.
    template <FloatingPoint F>
    auto write(std::string_view path, std::span<const F> weights, std::span<const uint8_t> masks, uint32_t nm_n,
               uint32_t nm_m) -> Result<void, TBError> {
        std::ofstream file(std::string(path), std::ios::binary | std::ios::trunc);
        if (!file.is_open()) return unexpected(TBError::kFileOpen);
        const TBHeader hdr = make_tb_header(nm_n, nm_m, weights.size(), masks.size(), sizeof(F));
        file.write(reinterpret_cast<const char*>(&hdr), sizeof(hdr));
        if (!file.good()) return unexpected(TBError::kFileWrite);
        file.write(reinterpret_cast<const char*>(weights.data()), static_cast<std::streamsize>(weights.size_bytes()));
        if (!file.good()) return unexpected(TBError::kFileWrite);
        file.write(reinterpret_cast<const char*>(masks.data()), static_cast<std::streamsize>(masks.size()));
        if (!file.good()) return unexpected(TBError::kFileWrite);
        return {};
    }
};

class TBReader {
public:
    TBReader() = default;
    TBReader(const TBReader&) = delete;
    TBReader& operator=(const TBReader&) = delete;
    TBReader(TBReader&&) noexcept = default;
    TBReader& operator=(TBReader&&) noexcept = default;

    /// Opens `path` and validates magic and version (serialization.hpp:178-196).
    auto open(std::string_view path) -> Result<TBHeader, TBError> {
        file_.open(std::string(path), std::ios::binary);
        if (!file_.is_open()) return unexpected(TBError::kFileOpen);
        TBHeader hdr{};
        if (auto r = read_section(0, sizeof(hdr), &hdr, TBError::kTruncated); !r) return unexpected(r.error());
        if (hdr.magic != kTBMagic) return unexpected(TBError::kBadMagic);
        if (hdr.version != kTBVersion) return unexpected(TBError::kVersionMismatch);
        header_ = hdr;
        return hdr;
    }

    /// The weight section (num_weights values at weights_offset).
    template <FloatingPoint F>
    auto read_weights(std::span<F> out) -> Result<void, TBError> {
        if (!file_.is_open()) return unexpected(TBError::kFileOpen);
        if (out.size() < header_.num_weights) return unexpected(TBError::kTruncated);
        return read_section(header_.weights_offset, header_.num_weights * sizeof(F), out.data(), TBError::kFileRead);
    }

    /// The mask section (num_mask_bytes at masks_offset).
    auto read_masks(std::span<uint8_t> out) -> Result<void, TBError> {
        if (!file_.is_open()) return unexpected(TBError::kFileOpen);
        if (out.size() < header_.num_mask_bytes) return unexpected(TBError::kTruncated);
        return read_section(header_.masks_offset, header_.num_mask_bytes, out.data(), TBError::kFileRead);
    }

    void close() { file_.close(); }
    [[nodiscard]] const TBHeader& header() const noexcept { return header_; }

private:
    /// `bytes` from file offset `offset` into dst.  The codes are the
    /// reader's interface: a seek that fails is kSeekFailed, a read that fails
    /// or comes up short is `on_short` (kTruncated for the header, kFileRead
    /// for a section).
    auto read_section(std::uint64_t offset, std::size_t bytes, void* dst, TBError on_short) -> Result<void, TBError> {
        file_.seekg(static_cast<std::streamoff>(offset));
        if (!file_.good()) return unexpected(TBError::kSeekFailed);
        file_.read(static_cast<char*>(dst), static_cast<std::streamsize>(bytes));
        if (!file_.good() || file_.gcount() != static_cast<std::streamsize>(bytes)) return unexpected(on_short);
        return {};
    }

    std::ifstream file_;
    TBHeader header_{};
};

}  // namespace tensorbit::core

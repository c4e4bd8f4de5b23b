#pragma once

/// @file loader.hpp
/// @brief .safetensors reader: header parsing and raw tensor reads.
///
/// Same interface as the reference's SafeTensorsFile
/// (include/tensorbit/core/loader.hpp:41-306): tensor metadata in file order,
/// lookup by name, raw byte reads.  The header is parsed by a small
/// recursive-descent JSON reader written for this library (objects, arrays,
/// strings with escapes, numbers, literals).  As in the reference every
/// top-level key becomes an entry (so "__metadata__" appears with an unknown
/// dtype), a shape of [] gives numel 0, and a missing data_offsets gives the
/// length numel * element size.
///
/// File format: [0, 8) little-endian u64 header length H; [8, 8+H) JSON
/// header; then the data section, which data_offsets index.

#include <cstddef>
#include <cstdint>
#include <fstream>
#include <span>
#include <string>
#include <string_view>
#include <vector>

#include "tensorbit/core/common.hpp"

namespace tensorbit::core::loader {

enum class LoaderError : uint8_t {
    kOk = 0,
    kFileOpen = 1,
    kBadHeader = 2,
    kBadJSON = 3,
    kUnsupportedDtype = 4,
    kNotFound = 5,
};

enum class STDtype : uint8_t { kF32 = 0, kF16 = 1, kBF16 = 2, kI64 = 3, kUnknown = 255 };

inline std::size_t dtype_size(STDtype dt) {
    switch (dt) {
    case STDtype::kF32: return 4;
    case STDtype::kF16: return 2;
    case STDtype::kBF16: return 2;
    case STDtype::kI64: return 8;
    default: return 0;
    }
}

/// Accepted spellings are those of loader.hpp:72-78.
inline STDtype parse_dtype(std::string_view s) {
    if (s == "F32" || s == "float32") return STDtype::kF32;
    if (s == "F16" || s == "float16") return STDtype::kF16;
    if (s == "BF16" || s == "bfloat16") return STDtype::kBF16;
    if (s == "I64" || s == "int64") return STDtype::kI64;
    return STDtype::kUnknown;
}

struct TensorMeta {
    std::string name;
    STDtype dtype = STDtype::kUnknown;
    std::vector<std::size_t> shape;
    std::size_t offset = 0;  // from the start of the data section
    std::size_t length = 0;  // bytes
    std::size_t numel = 0;
};

namespace detail {

/// Minimal JSON reader over a string; `ok` turns false on the first error.
class Json {
public:
    explicit Json(std::string_view s) : s_(s) {}
    bool ok = true;

    void ws() {
        while (p_ < s_.size() && (s_[p_] == ' ' || s_[p_] == '\n' || s_[p_] == '\r' || s_[p_] == '\t')) ++p_;
    }
    bool peek(char c) {
        ws();
        return p_ < s_.size() && s_[p_] == c;
    }
    bool eat(char c) {
        if (!peek(c)) return false;
        ++p_;
        return true;
    }
    void expect(char c) {
        if (!eat(c)) ok = false;
    }
    std::string str() {
        std::string out;
        if (!eat('"')) { ok = false; return out; }
        while (p_ < s_.size() && s_[p_] != '"') {
            char c = s_[p_++];
            if (c == '\\' && p_ < s_.size()) {
                const char e = s_[p_++];
                switch (e) {
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u': {
                    unsigned v = 0;
                    for (int k = 0; k < 4 && p_ < s_.size(); ++k) {
                        const char h = s_[p_++];
                        v = v * 16 + static_cast<unsigned>(h >= 'a' ? h - 'a' + 10 : h >= 'A' ? h - 'A' + 10 : h - '0');
                    }
                    if (v < 0x80) out += static_cast<char>(v);
                    else if (v < 0x800) { out += static_cast<char>(0xC0 | (v >> 6)); out += static_cast<char>(0x80 | (v & 0x3F)); }
                    else { out += static_cast<char>(0xE0 | (v >> 12)); out += static_cast<char>(0x80 | ((v >> 6) & 0x3F)); out += static_cast<char>(0x80 | (v & 0x3F)); }
                    break;
                }
                default: out += e; break;
                }
            } else {
                out += c;
            }
        }
        if (p_ >= s_.size()) ok = false;
        else ++p_;
        return out;
    }
    uint64_t uint() {
        ws();
        uint64_t v = 0;
        const std::size_t start = p_;
        while (p_ < s_.size() && s_[p_] >= '0' && s_[p_] <= '9') v = v * 10 + static_cast<uint64_t>(s_[p_++] - '0');
        if (p_ == start) ok = false;
        return v;
    }
    /// Skips any JSON value.
    void skip() {
        ws();
        if (p_ >= s_.size()) { ok = false; return; }
        const char c = s_[p_];
        if (c == '"') { str(); return; }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++p_;
            if (eat(close)) return;
            do {
                if (c == '{') { str(); expect(':'); }
                skip();
            } while (ok && eat(','));
            expect(close);
            return;
        }
        while (p_ < s_.size() && s_[p_] != ',' && s_[p_] != '}' && s_[p_] != ']' && s_[p_] != ' ' && s_[p_] != '\n') ++p_;
    }

private:
    std::string_view s_;
    std::size_t p_ = 0;
};

}  // namespace detail

class SafeTensorsFile {
public:
    SafeTensorsFile() = default;
    ~SafeTensorsFile() { close(); }
    SafeTensorsFile(const SafeTensorsFile&) = delete;
    SafeTensorsFile& operator=(const SafeTensorsFile&) = delete;

    auto open(std::string_view path) -> Result<void, LoaderError> {
        file_.open(std::string(path), std::ios::binary);
        if (!file_.is_open()) return unexpected(LoaderError::kFileOpen);
        uint64_t header_len = 0;
        file_.read(reinterpret_cast<char*>(&header_len), 8);
        if (!file_.good() || header_len == 0 || header_len > 100'000'000ULL) return unexpected(LoaderError::kBadHeader);
        std::string json(header_len, '\0');
        file_.read(json.data(), static_cast<std::streamsize>(header_len));
        if (!file_.good()) return unexpected(LoaderError::kBadHeader);
        data_offset_ = 8 + header_len;
        return parse(json);
    }

    [[nodiscard]] const std::vector<TensorMeta>& tensors() const noexcept { return tensors_; }

    [[nodiscard]] const TensorMeta* find(std::string_view name) const noexcept {
        for (auto& t : tensors_)
            if (t.name == name) return &t;
        return nullptr;
    }

    /// Reads the raw bytes of one tensor into `buffer` (>= meta.length bytes).
    auto read_tensor_data(const TensorMeta& meta, std::span<std::byte> buffer) -> Result<void, LoaderError> {
        if (!file_.is_open()) return unexpected(LoaderError::kFileOpen);
        if (buffer.size() < meta.length) return unexpected(LoaderError::kBadHeader);
        file_.seekg(static_cast<std::streamoff>(data_offset_ + meta.offset));
        if (!file_.good()) return unexpected(LoaderError::kBadHeader);
        file_.read(reinterpret_cast<char*>(buffer.data()), static_cast<std::streamsize>(meta.length));
        if (!file_.good()) return unexpected(LoaderError::kBadHeader);
        return {};
    }

    void close() { file_.close(); }
    [[nodiscard]] std::size_t data_offset() const noexcept { return data_offset_; }

private:
    auto parse(const std::string& text) -> Result<void, LoaderError> {
        tensors_.clear();
        detail::Json j(text);
        j.expect('{');
        if (!j.ok) return unexpected(LoaderError::kBadJSON);
        if (j.eat('}')) return {};
        do {
            TensorMeta meta;
            meta.name = j.str();
            j.expect(':');
            if (!j.ok) return unexpected(LoaderError::kBadJSON);
            if (!j.peek('{')) {
                j.skip();
            } else {
                j.expect('{');
                bool have_len = false;
                if (!j.eat('}')) {
                    do {
                        const std::string key = j.str();
                        j.expect(':');
                        if (key == "dtype" && j.peek('"')) {
                            meta.dtype = parse_dtype(j.str());
                        } else if (key == "shape" && j.peek('[')) {
                            j.expect('[');
                            if (!j.eat(']')) {
                                do meta.shape.push_back(static_cast<std::size_t>(j.uint()));
                                while (j.ok && j.eat(','));
                                j.expect(']');
                            }
                        } else if (key == "data_offsets" && j.peek('[')) {
                            j.expect('[');
                            const uint64_t a = j.uint();
                            j.expect(',');
                            const uint64_t b = j.uint();
                            j.expect(']');
                            meta.offset = static_cast<std::size_t>(a);
                            meta.length = static_cast<std::size_t>(b - a);
                            have_len = true;
                        } else {
                            j.skip();
                        }
                    } while (j.ok && j.eat(','));
                    j.expect('}');
                }
                if (!have_len) meta.length = 0;
            }
            if (!j.ok) return unexpected(LoaderError::kBadJSON);
            meta.numel = 0;
            if (!meta.shape.empty()) {
                meta.numel = 1;
                for (auto d : meta.shape) meta.numel *= d;
            }
            if (meta.length == 0) meta.length = meta.numel * dtype_size(meta.dtype);
            tensors_.push_back(std::move(meta));
        } while (j.eat(','));
        j.expect('}');
        if (!j.ok) return unexpected(LoaderError::kBadJSON);
        return {};
    }

    std::ifstream file_;
    std::size_t data_offset_ = 0;
    std::vector<TensorMeta> tensors_;
};

}  // namespace tensorbit::core::loader

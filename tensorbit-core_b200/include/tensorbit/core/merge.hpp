#pragma once

/// @file merge.hpp
/// @brief Native .tbm merge: several directories of .tb files -> one container.
///
/// The reference does this step in Python (scripts/merge_tbm.py:30-213); this
/// is the same operation in C++ with the same output bytes and messages:
///
///   * inputs are visited in argument order; a path that is not a directory is
///     reported and skipped (merge_tbm.py:173-177);
///   * in each directory every entry matching `*.tb` (hidden names included),
///     ordered by name as byte strings, becomes a tensor named by its stem with
///     every ".tbm" and then every ".tb" removed (:179-184);
///   * a name already taken is reported and skipped; the name is taken before
///     the header is read, so a file whose header is bad still reserves it
///     (:186-191);
///   * a header shorter than 4096 bytes or with the wrong magic is reported and
///     the file skipped (:30-39,200-201);
///   * the container is the files' bytes back to back, then a compact JSON
///     index, then the index length as a little-endian u32 (:117-150).  Index
///     offsets advance by 4096 + 4 * num_weights + num_mask_bytes taken from
///     each header, whatever the file's real length (:87-112); shapes are
///     [num_weights, 1] (:62-75); dtype follows the header's precision byte
///     (:93-99).  The JSON text is what Python's json.dumps writes with
///     separators (",", ":"): ASCII only, lowercase \u escapes, surrogate
///     pairs above U+FFFF, invalid UTF-8 bytes as \udc80..\udcff.
///
/// One deliberate difference: a tensor name holding a control character
/// (below 0x20, or 0x7f) is rejected before anything is written, where the
/// script raises after writing the data section and leaves a container
/// without an index.

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <string>
#include <string_view>
#include <system_error>
#include <vector>

#include "tensorbit/core/common.hpp"

namespace tensorbit::core {

enum class MergeError : uint8_t {
    kOk = 0,
    kNoInputs = 1,   // no readable .tb file in any input
    kFileOpen = 2,   // an input could not be opened, or the output created
    kFileRead = 3,
    kFileWrite = 4,
    kBadName = 5,    // a tensor name with a control character
};

struct MergeReport {
    std::size_t files = 0;        // .tb files in the container
    std::uintmax_t bytes = 0;     // size of the container file
    std::vector<std::string> log; // the lines the script prints, in order
    std::string detail;           // what failed, for an error result
};

namespace merge_detail {

inline constexpr std::size_t kHeader = 4096;
inline constexpr uint32_t kMagic = 0x31304254;

/// str(pathlib.PurePosixPath(p)): empty and "." parts dropped, a leading "//"
/// kept as is, one or three or more leading slashes become "/", "" -> ".".
inline std::string py_path(std::string_view p) {
    std::string root;
    if (p.size() >= 2 && p[0] == '/' && p[1] == '/' && (p.size() == 2 || p[2] != '/'))
        root = "//";
    else if (!p.empty() && p[0] == '/')
        root = "/";
    std::string out = root;
    bool first = true;
    std::size_t i = 0;
    while (i <= p.size()) {
        std::size_t j = p.find('/', i);
        if (j == std::string_view::npos) j = p.size();
        std::string_view part = p.substr(i, j - i);
        if (!part.empty() && part != ".") {
            if (!first) out += '/';
            out += part;
            first = false;
        }
        i = j + 1;
    }
    return out.empty() ? std::string(".") : out;
}

/// str(Path(dir) / name) for a normalised `dir`.
inline std::string py_join(const std::string& dir, const std::string& name) {
    if (dir == ".") return name;
    if (!dir.empty() && dir.back() == '/') return dir + name;
    return dir + "/" + name;
}

/// Code points of `s` decoded as UTF-8 with Python's surrogateescape: every
/// byte that is not part of a well-formed sequence becomes U+DC00 + byte.
inline std::vector<uint32_t> decode_utf8(std::string_view s) {
    std::vector<uint32_t> cps;
    const auto* b = reinterpret_cast<const unsigned char*>(s.data());
    const std::size_t n = s.size();
    std::size_t i = 0;
    while (i < n) {
        const uint32_t c = b[i];
        int len = 0;
        uint32_t cp = 0, lo = 0;
        if (c < 0x80) { cps.push_back(c); ++i; continue; }
        if (c >= 0xC2 && c <= 0xDF) { len = 2; cp = c & 0x1F; lo = 0x80; }
        else if (c >= 0xE0 && c <= 0xEF) { len = 3; cp = c & 0x0F; lo = 0x800; }
        else if (c >= 0xF0 && c <= 0xF4) { len = 4; cp = c & 0x07; lo = 0x10000; }
        bool ok = len > 0 && i + len <= n;
        for (int k = 1; ok && k < len; ++k) {
            if ((b[i + k] & 0xC0) != 0x80) ok = false;
            else cp = (cp << 6) | (b[i + k] & 0x3F);
        }
        if (ok && (cp < lo || cp > 0x10FFFF || (cp >= 0xD800 && cp <= 0xDFFF))) ok = false;
        if (ok) { cps.push_back(cp); i += len; }
        else { cps.push_back(0xDC00 + c); ++i; }
    }
    return cps;
}

/// json.dumps(s) body (without the quotes) with ensure_ascii.
inline std::string json_ascii(std::string_view s) {
    std::string out;
    char buf[16];
    for (uint32_t c : decode_utf8(s)) {
        switch (c) {
        case '"': out += "\\\""; continue;
        case '\\': out += "\\\\"; continue;
        case '\n': out += "\\n"; continue;
        case '\r': out += "\\r"; continue;
        case '\t': out += "\\t"; continue;
        case '\b': out += "\\b"; continue;
        case '\f': out += "\\f"; continue;
        default: break;
        }
        if (c >= 0x20 && c < 0x7F) {
            out += static_cast<char>(c);
        } else if (c < 0x10000) {
            std::snprintf(buf, sizeof buf, "\\u%04x", c);
            out += buf;
        } else {
            const uint32_t v = c - 0x10000;
            std::snprintf(buf, sizeof buf, "\\u%04x\\u%04x", 0xD800 + (v >> 10), 0xDC00 + (v & 0x3FF));
            out += buf;
        }
    }
    return out;
}

inline std::string u128_str(unsigned __int128 v) {
    if (v == 0) return "0";
    std::string s;
    while (v) { s.insert(s.begin(), static_cast<char>('0' + static_cast<int>(v % 10))); v /= 10; }
    return s;
}

/// f"{n:,}"
inline std::string with_commas(std::uintmax_t n) {
    std::string d = std::to_string(n), out;
    for (std::size_t i = 0; i < d.size(); ++i) {
        if (i && (d.size() - i) % 3 == 0) out += ',';
        out += d[i];
    }
    return out;
}

/// The stem of `file` (name without its last suffix) with ".tbm" then ".tb"
/// removed everywhere, as str.replace does (left to right, non-overlapping).
inline std::string tensor_name(const std::string& file) {
    std::string stem = file;
    const auto dot = stem.rfind('.');
    if (dot != std::string::npos && dot != 0) stem.resize(dot);
    auto strip = [](std::string s, std::string_view pat) {
        std::string out;
        std::size_t i = 0;
        while (true) {
            const auto j = s.find(pat, i);
            if (j == std::string::npos) { out.append(s, i, std::string::npos); break; }
            out.append(s, i, j - i);
            i = j + pat.size();
        }
        return out;
    };
    return strip(strip(stem, ".tbm"), ".tb");
}

struct Entry {
    std::string path;  // as the script prints it
    std::filesystem::path fs;
    std::string name;
    uint32_t nm_n, nm_m;
    uint64_t num_weights, num_mask_bytes;
    uint8_t precision;
};

template <typename T>
T load_le(const unsigned char* p) {
    T v = 0;
    for (std::size_t k = 0; k < sizeof(T); ++k) v |= static_cast<T>(p[k]) << (8 * k);
    return v;
}

}  // namespace merge_detail

/// Merge the `*.tb` files of `inputs` into the container `output`
/// (merge_tbm.py:158-213).  On success the report's log holds the warning
/// lines and the closing summary line; on error it holds the lines printed
/// so far and `detail` says what failed.
inline auto merge_tb_directories(const std::vector<std::string>& inputs, const std::string& output,
                                 std::string_view architecture, MergeReport* report)
    -> Result<void, MergeError> {
    namespace fs = std::filesystem;
    using namespace merge_detail;
    MergeReport local;
    MergeReport& rep = report ? *report : local;
    rep = MergeReport{};
    auto fail = [&](MergeError e, std::string why) -> Result<void, MergeError> {
        rep.detail = std::move(why);
        return unexpected(e);
    };

    std::vector<Entry> entries;
    std::vector<std::string> seen;
    for (const auto& in : inputs) {
        std::error_code ec;
        const std::string dir = py_path(in);
        if (!fs::is_directory(fs::path(dir), ec)) {
            rep.log.push_back("[WARN] Not a directory, skipping: " + in);
            continue;
        }
        std::vector<std::string> names;
        for (fs::directory_iterator it(fs::path(dir), ec), end; !ec && it != end; it.increment(ec)) {
            const std::string f = it->path().filename().string();
            if (f.size() >= 3 && f.compare(f.size() - 3, 3, ".tb") == 0) names.push_back(f);
        }
        if (ec) return fail(MergeError::kFileRead, "cannot list " + in + ": " + ec.message());
        std::sort(names.begin(), names.end());
        for (const auto& f : names) {
            if (f == "model.tbm") continue;
            const std::string name = tensor_name(f);
            if (std::find(seen.begin(), seen.end(), name) != seen.end()) {
                rep.log.push_back("[WARN] Duplicate tensor name: " + name + " (skipping)");
                continue;
            }
            seen.push_back(name);
            Entry e{py_join(dir, f), fs::path(py_join(dir, f)), name, 0, 0, 0, 0, 0};
            std::ifstream file(e.fs, std::ios::binary);
            if (!file.is_open() || fs::is_directory(e.fs, ec))
                return fail(MergeError::kFileOpen, "cannot open " + e.path);
            unsigned char h[kHeader];
            file.read(reinterpret_cast<char*>(h), kHeader);
            if (static_cast<std::size_t>(file.gcount()) < kHeader) {
                rep.log.push_back("[WARN] Truncated .tb header in " + e.path);
                continue;
            }
            const auto magic = load_le<uint32_t>(h);
            if (magic != kMagic) {
                char buf[16];
                std::snprintf(buf, sizeof buf, "0x%08X", magic);
                rep.log.push_back(std::string("[WARN] Bad magic ") + buf + " in " + e.path);
                continue;
            }
            e.nm_n = load_le<uint32_t>(h + 8);
            e.nm_m = load_le<uint32_t>(h + 12);
            e.num_weights = load_le<uint64_t>(h + 16);
            e.num_mask_bytes = load_le<uint64_t>(h + 24);
            e.precision = h[48];
            entries.push_back(std::move(e));
        }
    }
    if (entries.empty()) {
        rep.log.push_back("[ERROR] No valid .tb files found");
        return fail(MergeError::kNoInputs, "no valid .tb files found");
    }
    for (const auto& e : entries)
        for (uint32_t c : decode_utf8(e.name))
            if (c < 32 || c == 127) {
                char buf[8];
                std::snprintf(buf, sizeof buf, "%02X", c);
                return fail(MergeError::kBadName,
                            std::string("Tensor name contains unprintable char 0x") + buf + ": " + e.name);
            }

    // The JSON index (merge_tbm.py:78-135).
    std::string json = "{\"architecture\":\"" + json_ascii(architecture) + "\",\"config\":{\"num_layers\":" +
                       std::to_string(entries.size()) + "},\"tensors\":[";
    unsigned __int128 offset = 0;
    for (std::size_t i = 0; i < entries.size(); ++i) {
        const auto& e = entries[i];
        const char* dtype = e.precision == 1 ? "fp16" : e.precision == 2 ? "bf16" : e.precision == 3 ? "fp64" : "fp32";
        if (i) json += ',';
        json += "{\"name\":\"" + json_ascii(e.name) + "\",\"offset\":" + u128_str(offset) + ",\"shape\":[" +
                std::to_string(e.num_weights) + ",1],\"nm_n\":" + std::to_string(e.nm_n) +
                ",\"nm_m\":" + std::to_string(e.nm_m) + ",\"dtype\":\"" + dtype +
                "\",\"num_weights\":" + std::to_string(e.num_weights) +
                ",\"num_mask_bytes\":" + std::to_string(e.num_mask_bytes) + "}";
        offset += static_cast<unsigned __int128>(kHeader) + static_cast<unsigned __int128>(e.num_weights) * 4 +
                  e.num_mask_bytes;
    }
    json += "]}";
    if (json.size() > 0xFFFFFFFFull) return fail(MergeError::kFileWrite, "JSON index longer than 4 GiB");

    const fs::path out(py_path(output));
    std::error_code ec;
    if (out.has_parent_path()) fs::create_directories(out.parent_path(), ec);
    std::ofstream dst(out, std::ios::binary | std::ios::trunc);
    if (!dst.is_open()) return fail(MergeError::kFileOpen, "cannot create " + output);
    std::vector<char> buf(std::size_t{16} << 20);
    for (const auto& e : entries) {
        std::ifstream src(e.fs, std::ios::binary);
        if (!src.is_open()) return fail(MergeError::kFileOpen, "cannot open " + e.path);
        while (src) {
            src.read(buf.data(), static_cast<std::streamsize>(buf.size()));
            const auto got = src.gcount();
            if (got > 0) dst.write(buf.data(), got);
            if (!dst.good()) return fail(MergeError::kFileWrite, "write failed: " + output);
        }
        if (src.bad()) return fail(MergeError::kFileRead, "read failed: " + e.path);
    }
    dst.write(json.data(), static_cast<std::streamsize>(json.size()));
    const uint32_t len = static_cast<uint32_t>(json.size());
    const unsigned char tail[4] = {static_cast<unsigned char>(len), static_cast<unsigned char>(len >> 8),
                                   static_cast<unsigned char>(len >> 16), static_cast<unsigned char>(len >> 24)};
    dst.write(reinterpret_cast<const char*>(tail), 4);
    dst.close();
    if (!dst.good()) return fail(MergeError::kFileWrite, "write failed: " + output);

    rep.files = entries.size();
    rep.bytes = fs::file_size(out, ec);
    rep.log.push_back("[merge_tbm] Merged " + std::to_string(entries.size()) + " .tb files into '" + py_path(output) +
                      "' (" + with_commas(rep.bytes) + " bytes, " + std::to_string(entries.size()) + " tensors)");
    return {};
}

}  // namespace tensorbit::core

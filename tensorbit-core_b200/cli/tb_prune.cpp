/// @file tb_prune.cpp
/// @brief `tb-prune`: the pruning CLI of tensorbit-core, with every stage on the GPU.
///
/// Same flags, defaults, log lines and outputs as the reference CLI
/// (src/main.cpp:11-22,284-644):
///   mock mode  - one mock tensor (mt19937(42), normal(0, 0.5), weights and
///                gradients drawn alternately), EHAP prune, CORING top-N 2:4 with
///                proportional redistribution, one .tb file;
///   real mode  - every F32/BF16/F16 tensor of a .safetensors file pruned the same
///                way with gradients 0.01*w, one .tb per tensor plus model.tbm
///                (the .tb files concatenated, a JSON index, its u32 length).
/// The tensors are moved to the device once per tensor and every pruner call
/// runs there; .tb files are byte-identical to the reference's.

#include <algorithm>
#include <charconv>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <random>
#include <span>
#include <string>
#include <string_view>
#include <vector>

#include "tb_kernels.h"
#include "tensorbit/core/common.hpp"
#include "tensorbit/core/coring.hpp"
#include "tensorbit/core/ehap.hpp"
#include "tensorbit/core/loader.hpp"
#include "tensorbit/core/serialization.hpp"
#include "tensorbit/core/tensor.hpp"

using namespace tensorbit::core;

namespace {

struct Options {
    std::string model_path;
    std::string output_path = "output.tb";
    std::string method = "EHAP";
    std::string strategy = "OneShot";
    std::string architecture = "llama";
    int nm_n = 2, nm_m = 4;
    float damping = 0.01f;
    float sparsity_ratio = 0.5f;
    std::size_t mock_size = 4096;
    int hidden_size = 4096, num_heads = 32, num_kv_heads = 8, intermediate_size = 14336;
    int vocab_size = 32000, max_seq_len = 2048;
    float norm_eps = 1e-5f, rope_theta = 10000.0f;
    bool use_mock = false, show_help = false, show_version = false;
};

void usage(const char* prog) {
    std::fprintf(stderr,
                 "tb-prune - Tensorbit Core pruner on B200 (sm_100a)\n\n"
                 "Usage: %s --model <PATH> [OPTIONS]\n\n"
                 "  --model PATH        .safetensors file                    [or omit for mock]\n"
                 "  --sparsity N:M      N:M pattern                          [default: 2:4]\n"
                 "  --output PATH       .tb path (mock) or directory (real)  [default: output.tb]\n"
                 "  --method NAME       EHAP | Magnitude                     [default: EHAP]\n"
                 "  --strategy NAME     OneShot | Iterative | BlockOBS       [default: OneShot]\n"
                 "  --architecture A    architecture name for model.tbm      [default: llama]\n"
                 "  --hidden-size N, --num-heads N, --num-kv-heads N, --intermediate-size N,\n"
                 "  --vocab-size N, --max-seq-len N   model.tbm config fields\n"
                 "  --damping VAL       EHAP Fisher damping                  [default: 0.01]\n"
                 "  --mock-size N       elements of the mock tensor          [default: 4096]\n"
                 "  --help, -h / --version\n",
                 prog);
}

bool parse_nm(std::string_view spec, int& n, int& m) {
    const auto pos = spec.find(':');
    if (pos == std::string_view::npos) return false;
    auto num = [](std::string_view s, int& v) {
        auto r = std::from_chars(s.data(), s.data() + s.size(), v);
        return r.ec == std::errc{} && v > 0;
    };
    return num(spec.substr(0, pos), n) && num(spec.substr(pos + 1), m) && n < m;
}

template <typename T>
void parse_number(std::string_view v, T& out) {
    if (!v.empty()) std::from_chars(v.data(), v.data() + v.size(), out);
}

std::string sanitise(std::string_view name) {
    std::string s(name);
    for (auto& c : s)
        if (c == '/' || c == '\\') c = '_';
    return s;
}

std::string json_escape(std::string_view s) {
    std::string out;
    for (char c : s) {
        const auto u = static_cast<unsigned char>(c);
        switch (u) {
        case '"': out += "\\\""; break;
        case '\\': out += "\\\\"; break;
        case '\n': out += "\\n"; break;
        case '\t': out += "\\t"; break;
        case '\r': out += "\\r"; break;
        case '\b': out += "\\b"; break;
        case '\f': out += "\\f"; break;
        default:
            if (u < 0x20) {
                char buf[8];
                std::snprintf(buf, sizeof(buf), "\\u%04X", u);
                out += buf;
            } else {
                out += c;
            }
        }
    }
    return out;
}

EHAPConfig ehap_config(const Options& o) {
    EHAPConfig c;
    c.damping = o.damping;
    c.sparsity_ratio = o.sparsity_ratio;
    c.use_diagonal_fisher = o.method != "Magnitude";
    c.ema_decay = 0.99f;
    c.importance_mode = ImportanceMode::kOBD;
    if (o.strategy == "BlockOBS") {
        c.prune_strategy = PruneStrategy::kBlockOBS;
        c.obs_block_size = 128;
        c.obs_off_diag_alpha = 0.01f;
    } else if (o.strategy == "Iterative") {
        c.prune_strategy = PruneStrategy::kIterative;
        c.prune_rounds = 5;
    } else {
        c.prune_strategy = PruneStrategy::kOneShot;
    }
    return c;
}

CORINGConfig coring_config(const Options& o) {
    CORINGConfig c;
    c.N = o.nm_n;
    c.M = o.nm_m;
    c.use_cuda = true;
    c.mask_strategy = MaskStrategy::kTopN;
    c.redist_mode = RedistMode::kProportional;
    c.hardware_aware_layout = true;
    return c;
}

TensorDense<float> device_copy(const float* host, std::size_t n) {
    TensorDense<float> d(std::span<const std::size_t>(&n, 1), DeviceLocation::kDevice);
    if (n && (tb_memcpy_h2d(d.data(), host, n * sizeof(float), nullptr) || tb_stream_sync(nullptr))) {
        TENSORBIT_LOG_ERROR("host to device copy failed: {}", tb_last_error());
        std::exit(1);
    }
    return d;
}

struct Pruned {
    std::vector<float> weights;
    std::vector<uint8_t> masks;
    std::size_t ehap_pruned = 0;
    std::size_t coring_pruned = 0;
};

enum class Stage { kOk, kEhap, kCoring };

/// The per-tensor sequence of src/main.cpp:372-409 on device tensors.
Stage prune_tensor(const Options& o, TensorDense<float>& w, const TensorDense<float>& g, Pruned& out) {
    const auto shape = w.shape();
    EHAPPruner<float> ehap(ehap_config(o));
    ehap.accumulate_fisher(g, 0.01f);
    if (o.strategy == "BlockOBS" && o.method != "Magnitude") {
        for (int k = 0; k < 4; ++k) {
            // Snapshot k = g * (0.9 + 0.02 k), scaled on the host as the reference does.
            auto hg = g.to_host();
            const float f = 0.9f + 0.02f * static_cast<float>(k);
            for (std::size_t i = 0; i < hg.size(); ++i) hg[i] *= f;
            ehap.store_gradient(hg);
        }
    }
    auto er = ehap.prune(w);
    if (!er) return Stage::kEhap;
    out.ehap_pruned = er.value();
    CORINGPruner<float> coring(coring_config(o));
    TensorDense<float> imp(shape, DeviceLocation::kDevice);
    TensorDense<uint8_t> msk(shape, DeviceLocation::kDevice);
    ehap.compute_importance(w, imp);
    auto cr = coring.prune(imp, w);
    if (!cr) return Stage::kCoring;
    out.coring_pruned = cr.value();
    coring.generate_nm_mask(imp, msk);
    const std::size_t groups = w.size() / static_cast<std::size_t>(o.nm_m);
    out.weights.resize(w.size());
    out.masks.resize(groups);
    if (tb_memcpy_d2h(out.weights.data(), w.data(), w.bytes(), nullptr) ||
        tb_memcpy_d2h(out.masks.data(), msk.data(), groups, nullptr) || tb_stream_sync(nullptr)) {
        TENSORBIT_LOG_ERROR("device to host copy failed: {}", tb_last_error());
        return Stage::kCoring;
    }
    return Stage::kOk;
}

int run_mock(const Options& o) {
    TENSORBIT_LOG_INFO("[Load] Generating mock weight tensor ({} elements)", o.mock_size);
    std::vector<float> hw(o.mock_size), hg(o.mock_size);
    std::mt19937 rng(42);
    std::normal_distribution<float> dist(0.0f, 0.5f);
    for (std::size_t i = 0; i < o.mock_size; ++i) {
        hw[i] = dist(rng);
        hg[i] = dist(rng) * 0.1f;
    }
    auto w = device_copy(hw.data(), hw.size());
    auto g = device_copy(hg.data(), hg.size());
    Pruned p;
    const Stage s = prune_tensor(o, w, g, p);
    if (s == Stage::kEhap) { TENSORBIT_LOG_ERROR("EHAP pruning failed"); return 1; }
    if (s == Stage::kCoring) { TENSORBIT_LOG_ERROR("CORING pruning failed"); return 1; }
    const double n = static_cast<double>(o.mock_size);
    TENSORBIT_LOG_INFO("  EHAP pruned: {} weights ({:.1f}%)", p.ehap_pruned, 100.0 * static_cast<double>(p.ehap_pruned) / n);
    TENSORBIT_LOG_INFO("  CORING ({}/{}): {} weights pruned ({:.1f}% sparsity)", o.nm_n, o.nm_m, p.coring_pruned,
                       100.0 * static_cast<double>(p.coring_pruned) / n);
    TENSORBIT_LOG_INFO("[Save] Writing .tb file...");
    TBWriter writer;
    auto wr = writer.write<float>(o.output_path, p.weights, p.masks, static_cast<uint32_t>(o.nm_n),
                                  static_cast<uint32_t>(o.nm_m));
    if (!wr) { TENSORBIT_LOG_ERROR("Failed to write .tb file"); return 1; }
    const double kb = static_cast<double>(4096 + p.weights.size() * 4 + p.masks.size()) / 1024.0;
    TENSORBIT_LOG_INFO("  Saved to '{}' ({:.2f} KB)", o.output_path, kb);
    TBReader reader;
    if (auto h = reader.open(o.output_path)) {
        TENSORBIT_LOG_INFO("[Verify] .tb valid: magic=0x{:08X} v{} {}/{} sparsity {} wts", h->magic, h->version, h->nm_n,
                           h->nm_m, h->num_weights);
        reader.close();
    }
    TENSORBIT_LOG_INFO("Done.");
    return 0;
}

struct TbmEntry {
    std::string name, path;
    std::size_t num_weights, num_mask_bytes, shape0, shape1;
    int nm_n, nm_m;
};

int run_model(const Options& o) {
    loader::SafeTensorsFile sf;
    if (auto r = sf.open(o.model_path); !r) {
        TENSORBIT_LOG_ERROR("Failed to open model: safetensors parse error (code={})", static_cast<int>(r.error()));
        return 1;
    }
    const auto& metas = sf.tensors();
    if (metas.empty()) { TENSORBIT_LOG_ERROR("No tensors found in safetensors file"); return 1; }
    std::filesystem::path out_dir(o.output_path);
    std::error_code ec;
    std::filesystem::create_directories(out_dir, ec);
    if (ec) { TENSORBIT_LOG_ERROR("Failed to create output directory: {}", o.output_path); return 1; }
    std::vector<TbmEntry> entries;
    std::size_t count = 0, total = 0, total_pruned = 0;
    TENSORBIT_LOG_INFO("[Load] Processing {} tensor(s) from '{}'", metas.size(), o.model_path);
    for (const auto& meta : metas) {
        if (meta.dtype != loader::STDtype::kF32 && meta.dtype != loader::STDtype::kBF16 &&
            meta.dtype != loader::STDtype::kF16)
            continue;
        std::vector<std::byte> raw(meta.length);
        if (!sf.read_tensor_data(meta, raw)) { TENSORBIT_LOG_WARN("  SKIP {}: read error", meta.name); continue; }
        // Widen on the device (src/main.cpp:213-245), then gradients = 0.01 * w (src/main.cpp:253-259).
        const std::size_t n = meta.numel;
        const int dt = meta.dtype == loader::STDtype::kF32 ? TB_F32 : meta.dtype == loader::STDtype::kBF16 ? TB_BF16 : TB_F16;
        TensorDense<uint8_t> draw(std::span<const std::size_t>(&meta.length, 1), DeviceLocation::kDevice);
        TensorDense<float> w(std::span<const std::size_t>(meta.shape.data(), meta.shape.size()), DeviceLocation::kDevice);
        if (w.size() != n || (n && (tb_memcpy_h2d(draw.data(), raw.data(), meta.length, nullptr) ||
                                    tb_decode_to_f32(draw.data(), dt, w.data(), n, nullptr) || tb_stream_sync(nullptr)))) {
            TENSORBIT_LOG_WARN("  SKIP {}: read error", meta.name);
            continue;
        }
        auto hw = w.to_host();
        std::vector<float> hg(n);
        for (std::size_t i = 0; i < n; ++i) hg[i] = hw[i] * 0.01f;
        TensorDense<float> g(w.shape(), DeviceLocation::kDevice);
        if (n && (tb_memcpy_h2d(g.data(), hg.data(), n * 4, nullptr) || tb_stream_sync(nullptr))) continue;
        TENSORBIT_LOG_INFO("  [{}] {} — {} elements", count, meta.name, meta.numel);
        Pruned p;
        const Stage s = w.empty() ? Stage::kEhap : prune_tensor(o, w, g, p);
        if (s == Stage::kEhap) { TENSORBIT_LOG_WARN("    SKIP (EHAP failed)"); continue; }
        if (s == Stage::kCoring) { TENSORBIT_LOG_WARN("    SKIP (CORING failed)"); continue; }
        const auto fname = sanitise(meta.name) + ".tb";
        const auto path = out_dir / fname;
        TBWriter writer;
        if (!writer.write<float>(path.string(), p.weights, p.masks, static_cast<uint32_t>(o.nm_n),
                                 static_cast<uint32_t>(o.nm_m))) {
            TENSORBIT_LOG_WARN("    SKIP (write error)");
            continue;
        }
        const double kb = static_cast<double>(4096 + p.weights.size() * 4 + p.masks.size()) / 1024.0;
        TENSORBIT_LOG_INFO("    -> '{}' ({:.1f} KB — {} wts, {} pruned by CORING)", fname, kb, meta.numel, p.coring_pruned);
        entries.push_back({meta.name, path.string(), meta.numel, p.masks.size(), meta.shape.empty() ? 0 : meta.shape[0],
                           meta.shape.size() > 1 ? meta.shape[1] : 1, o.nm_n, o.nm_m});
        ++count;
        total += meta.numel;
        total_pruned += p.coring_pruned;
    }
    sf.close();
    if (!entries.empty()) {
        const auto tbm_path = out_dir / "model.tbm";
        TENSORBIT_LOG_INFO("[TBM] Building container: {}", tbm_path.string());
        std::ofstream tbm(tbm_path, std::ios::binary | std::ios::trunc);
        if (!tbm.is_open()) {
            TENSORBIT_LOG_ERROR("Failed to create .tbm file");
        } else {
            std::string json = "{\"architecture\":\"" + json_escape(o.architecture) + "\",\"config\":{";
            json += "\"num_layers\":" + std::to_string(count);
            json += ",\"hidden_size\":" + std::to_string(o.hidden_size);
            json += ",\"num_heads\":" + std::to_string(o.num_heads);
            json += ",\"num_kv_heads\":" + std::to_string(o.num_kv_heads);
            json += ",\"intermediate_size\":" + std::to_string(o.intermediate_size);
            json += ",\"vocab_size\":" + std::to_string(o.vocab_size);
            json += ",\"max_seq_len\":" + std::to_string(o.max_seq_len);
            json += ",\"norm_eps\":" + std::to_string(o.norm_eps);
            json += ",\"rope_theta\":" + std::to_string(o.rope_theta);
            json += "},\"tensors\":[";
            const char* sep = "";
            for (const auto& e : entries) {
                const auto offset = static_cast<std::size_t>(tbm.tellp());
                std::ifstream tb(e.path, std::ios::binary);
                std::vector<char> buf((std::istreambuf_iterator<char>(tb)), std::istreambuf_iterator<char>());
                tbm.write(buf.data(), static_cast<std::streamsize>(buf.size()));
                json += sep;
                json += "{\"name\":\"" + json_escape(e.name) + "\",\"offset\":" + std::to_string(offset) +
                        ",\"shape\":[" + std::to_string(e.shape0) + "," + std::to_string(e.shape1) + "],\"nm_n\":" +
                        std::to_string(e.nm_n) + ",\"nm_m\":" + std::to_string(e.nm_m) +
                        ",\"dtype\":\"fp32\",\"num_weights\":" + std::to_string(e.num_weights) +
                        ",\"num_mask_bytes\":" + std::to_string(e.num_mask_bytes) + "}";
                sep = ",";
            }
            json += "]}";
            tbm.write(json.data(), static_cast<std::streamsize>(json.size()));
            const uint32_t len = static_cast<uint32_t>(json.size());
            tbm.write(reinterpret_cast<const char*>(&len), sizeof(len));
            tbm.close();
            TENSORBIT_LOG_INFO("[TBM] Container written: model.tbm ({} tensors)", entries.size());
        }
    }
    const double pct = 100.0 * static_cast<double>(total_pruned) / static_cast<double>(std::max<std::size_t>(total, 1));
    TENSORBIT_LOG_INFO("Done. {} tensors, {} total weights, {} pruned ({:.1f}%). Output: {}", count, total, total_pruned,
                       pct, o.output_path);
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    Options o;
    for (int i = 1; i < argc; ++i) {
        const std::string_view a(argv[i]);
        auto next = [&]() -> std::string_view { return i + 1 < argc ? std::string_view(argv[++i]) : std::string_view{}; };
        if (a == "--model") o.model_path = std::string(next());
        else if (a == "--sparsity") {
            const auto spec = next();
            if (spec.empty() || !parse_nm(spec, o.nm_n, o.nm_m)) {
                TENSORBIT_LOG_FATAL("--sparsity requires a valid N:M (e.g. 2:4)");
                return 1;
            }
        } else if (a == "--output") o.output_path = std::string(next());
        else if (a == "--method") o.method = std::string(next());
        else if (a == "--strategy") o.strategy = std::string(next());
        else if (a == "--architecture") o.architecture = std::string(next());
        else if (a == "--hidden-size") parse_number(next(), o.hidden_size);
        else if (a == "--num-heads") parse_number(next(), o.num_heads);
        else if (a == "--num-kv-heads") parse_number(next(), o.num_kv_heads);
        else if (a == "--intermediate-size") parse_number(next(), o.intermediate_size);
        else if (a == "--vocab-size") parse_number(next(), o.vocab_size);
        else if (a == "--max-seq-len") parse_number(next(), o.max_seq_len);
        else if (a == "--damping") parse_number(next(), o.damping);
        else if (a == "--mock-size") { parse_number(next(), o.mock_size); o.use_mock = true; }
        else if (a == "--help" || a == "-h") o.show_help = true;
        else if (a == "--version") o.show_version = true;
        else TENSORBIT_LOG_WARN("Unknown flag: '{}'", a);
    }
    if (o.show_help) { usage(argv[0]); return 0; }
    if (o.show_version) { std::fprintf(stdout, "tb-prune v0.2.0 — Tensorbit Core (B200 sm_100a)\n"); return 0; }
    if (o.model_path.empty()) o.use_mock = true;
    int ndev = 0;
    tb_device_count(&ndev);
    if (ndev == 0) {
        TENSORBIT_LOG_FATAL("no CUDA device: tb-prune runs every stage on the GPU");
        return 1;
    }
    TENSORBIT_LOG_INFO("Tensorbit Core v0.2.0 — Pruning Pipeline (B200)");
    return o.use_mock ? run_mock(o) : run_model(o);
}

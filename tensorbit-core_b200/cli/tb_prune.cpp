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
#include <condition_variable>
#include <deque>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <mutex>
#include <random>
#include <span>
#include <string>
#include <string_view>
#include <thread>
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
    int gpus = 1;  // devices pruning whole tensors side by side in real mode
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
                 "  --gpus N            GPUs pruning tensors side by side    [default: 1, real mode]\n"
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

/// dst = src * f element by element (FP32, round to nearest) on the device:
/// a device copy followed by the legacy launcher that multiplies in place
/// (launch_fisher_beta_decay, kernels.hpp:51-54); the product is the same
/// single multiplication as the reference's host loops.
bool scaled_copy(const TensorDense<float>& src, float f, TensorDense<float>& dst) {
    if (src.empty()) return true;
    if (tb_memcpy_d2d(dst.data(), src.data(), src.bytes(), nullptr) ||
        tb_fisher_beta_decay(dst.data(), f, src.size(), nullptr)) {
        TENSORBIT_LOG_ERROR("device scale failed: {}", tb_last_error());
        return false;
    }
    return true;
}

struct Pruned {
    std::vector<float> weights;
    std::vector<uint8_t> masks;
    std::size_t ehap_pruned = 0;
    std::size_t coring_pruned = 0;
};

enum class Stage { kOk, kEhap, kCoring };

/// The OneShot sequence of src/main.cpp:372-409 (accumulate_fisher with alpha
/// 0.01, EHAP one-shot prune, compute_importance, CORING top-N prune with
/// proportional redistribution, generate_nm_mask) as one library call: two
/// fused passes around the global radix select, bit-identical to the calls
/// made one by one.  EHAP's own failures (empty tensor, sparsity) are ruled
/// out before, so a failed call is CORING's (N:M, numel % M) or the device's.
Stage prune_one_shot_fused(const Options& o, const TensorDense<float>& w, const TensorDense<float>& g, Pruned& out) {
    const std::size_t n = w.size();
    const std::size_t groups = n / static_cast<std::size_t>(o.nm_m);
    const bool fisher = o.method != "Magnitude";
    if (n == 0 || !(o.sparsity_ratio > 0.0f && o.sparsity_ratio < 1.0f)) return Stage::kEhap;
    TensorDense<float> wo(w.shape(), DeviceLocation::kDevice), F(w.shape(), DeviceLocation::kDevice),
        s(w.shape(), DeviceLocation::kDevice);
    TensorDense<uint8_t> mk(std::span<const std::size_t>(&groups, 1), DeviceLocation::kDevice);
    tb_prune_args a{};
    a.struct_size = sizeof(a);
    a.weights = w.data();
    a.w_dtype = TB_F32;
    a.grads = fisher ? g.data() : nullptr;
    a.g_dtype = TB_F32;
    a.S = fisher ? 1 : 0;
    a.N = n;
    a.alpha = 0.01f;  // src/main.cpp:375
    a.beta = ehap_config(o).ema_decay;
    a.damping = o.damping;
    a.importance_mode = TB_IMP_OBD;
    a.use_fisher = fisher ? 1 : 0;
    a.nm_n = o.nm_n;
    a.nm_m = o.nm_m;
    a.mask_strategy = TB_MASK_TOPN;
    a.iterative_rounds = 3;
    a.redist_mode = TB_REDIST_PROPORTIONAL;
    a.w_out = wo.data();
    a.mask_out = mk.data();
    a.fisher_out = F.data();
    a.scores_out = s.data();
    uint64_t ehap_pruned = 0, coring_pruned = 0;
    if (tb_prune_one_shot_nm(&a, o.sparsity_ratio, nullptr, &ehap_pruned, &coring_pruned, nullptr)) {
        TENSORBIT_LOG_DEBUG("one-shot N:M pass: {}", tb_last_error());
        return Stage::kCoring;
    }
    out.ehap_pruned = ehap_pruned;
    out.coring_pruned = coring_pruned;
    out.weights.resize(n);
    out.masks.resize(groups);
    if (tb_memcpy_d2h(out.weights.data(), wo.data(), wo.bytes(), nullptr) ||
        tb_memcpy_d2h(out.masks.data(), mk.data(), groups, nullptr) || tb_stream_sync(nullptr)) {
        TENSORBIT_LOG_ERROR("device to host copy failed: {}", tb_last_error());
        return Stage::kCoring;
    }
    return Stage::kOk;
}

/// The per-tensor sequence of src/main.cpp:372-409 on device tensors.
Stage prune_tensor(const Options& o, TensorDense<float>& w, const TensorDense<float>& g, Pruned& out) {
    if (o.strategy != "Iterative" && o.strategy != "BlockOBS") return prune_one_shot_fused(o, w, g, out);
    const auto shape = w.shape();
    EHAPPruner<float> ehap(ehap_config(o));
    ehap.accumulate_fisher(g, 0.01f);
    if (o.strategy == "BlockOBS" && o.method != "Magnitude") {
        for (int k = 0; k < 4; ++k) {
            // Snapshot k = g * (0.9 + 0.02 k): the reference scales a host copy,
            // one float product per element; the same product on the device.
            const float f = 0.9f + 0.02f * static_cast<float>(k);
            TensorDense<float> snap(shape, DeviceLocation::kDevice);
            if (!scaled_copy(g, f, snap)) return Stage::kEhap;
            ehap.store_gradient(snap);
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

/// One eligible tensor of a real-mode run as it moves through the pipeline.
struct Job {
    const loader::TensorMeta* meta = nullptr;
    std::byte* raw = nullptr;  // pinned host copy of the tensor's bytes
    std::size_t cap = 0;
    bool read_ok = false;
    bool done = false;
    Stage stage = Stage::kOk;
    bool skip_silently = false;  // a device copy failed after decoding (the reference's silent `continue`)
    Pruned result;
};

/// Real mode as a pipeline over the tensors of one .safetensors file.  A reader
/// thread copies the next tensors' bytes into page-locked buffers (at most
/// `gpus + 1` ahead); one worker thread per GPU takes whole tensors, which are
/// independent, and runs decode -> gradients -> EHAP -> CORING -> mask on its
/// device; the calling thread logs and writes the .tb files in tensor order.
/// Files, the model.tbm container and messages are those of the serial
/// reference loop (src/main.cpp:437-636); only the overlap of disk, PCIe and
/// GPU work differs.
class Pipeline {
public:
    Pipeline(const Options& o, loader::SafeTensorsFile& sf, std::vector<Job>& jobs, int gpus)
        : o_(o), sf_(sf), jobs_(jobs), gpus_(gpus) {}

    void start() {
        reader_ = std::thread([this] { read_all(); });
        for (int d = 0; d < gpus_; ++d) workers_.emplace_back([this, d] { work(d); });
    }

    /// Blocks until job i is finished.  At most `gpus + 1` jobs are between
    /// being read and being released by the caller, which bounds the pinned
    /// buffers and the host copies of finished outputs.
    Job& wait(std::size_t i) {
        std::unique_lock<std::mutex> lk(mu_);
        cv_done_.wait(lk, [&] { return jobs_[i].done; });
        return jobs_[i];
    }

    void join() {
        if (reader_.joinable()) reader_.join();
        for (auto& t : workers_) t.join();
        for (auto& b : pool_) tb_host_free(b.first);
        pool_.clear();
    }

private:
    void read_all() {
        for (std::size_t i = 0; i < jobs_.size(); ++i) {
            Job& j = jobs_[i];
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_room_.wait(lk, [&] { return in_flight_ < static_cast<std::size_t>(gpus_ + 1); });
                ++in_flight_;
                take_buffer(j);  // under the lock: the pool is shared with the workers
            }
            if (j.raw) j.read_ok = static_cast<bool>(sf_.read_tensor_data(*j.meta, std::span<std::byte>(j.raw, j.meta->length)));
            else j.read_ok = j.meta->length == 0;
            {
                std::lock_guard<std::mutex> lk(mu_);
                ready_.push_back(i);
            }
            cv_ready_.notify_one();
        }
        {
            std::lock_guard<std::mutex> lk(mu_);
            reader_done_ = true;
        }
        cv_ready_.notify_all();
    }

    // A pooled pinned buffer of at least the tensor's size, or a new one.
    void take_buffer(Job& j) {
        const std::size_t need = j.meta->length;
        if (need == 0) return;
        std::size_t best = pool_.size();
        for (std::size_t k = 0; k < pool_.size(); ++k)
            if (pool_[k].second >= need && (best == pool_.size() || pool_[k].second < pool_[best].second)) best = k;
        if (best < pool_.size()) {
            j.raw = pool_[best].first;
            j.cap = pool_[best].second;
            pool_.erase(pool_.begin() + static_cast<std::ptrdiff_t>(best));
            return;
        }
        void* p = nullptr;
        if (tb_host_alloc(&p, need) == TB_OK) {
            j.raw = static_cast<std::byte*>(p);
            j.cap = need;
        }
    }

    void give_back(Job& j) {
        std::lock_guard<std::mutex> lk(mu_);
        if (j.raw) pool_.emplace_back(j.raw, j.cap);
        j.raw = nullptr;
    }

public:
    /// The caller is done with a finished job (written or skipped): its
    /// outputs are dropped and the reader may read one tensor further ahead.
    void release(Job& j) {
        j.result = Pruned{};
        std::lock_guard<std::mutex> lk(mu_);
        --in_flight_;
        cv_room_.notify_one();
    }

private:

    void work(int dev) {
        const bool device_ok = tb_set_device(dev) == TB_OK;
        for (;;) {
            std::size_t i;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_ready_.wait(lk, [&] { return !ready_.empty() || reader_done_; });
                if (ready_.empty()) return;
                i = ready_.front();
                ready_.pop_front();
            }
            Job& j = jobs_[i];
            if (j.read_ok && device_ok) run(j);
            else j.read_ok = false;
            give_back(j);
            {
                std::lock_guard<std::mutex> lk(mu_);
                j.done = true;
            }
            cv_done_.notify_all();
        }
    }

    // Widen on the device (src/main.cpp:213-245), then gradients = 0.01 * w
    // (src/main.cpp:253-259, the same float product on the device), then the
    // pruner sequence.
    void run(Job& j) {
        const auto& meta = *j.meta;
        const std::size_t n = meta.numel;
        const int dt = meta.dtype == loader::STDtype::kF32 ? TB_F32 : meta.dtype == loader::STDtype::kBF16 ? TB_BF16 : TB_F16;
        TensorDense<uint8_t> draw(std::span<const std::size_t>(&meta.length, 1), DeviceLocation::kDevice);
        TensorDense<float> w(std::span<const std::size_t>(meta.shape.data(), meta.shape.size()), DeviceLocation::kDevice);
        if (w.size() != n || (n && (tb_memcpy_h2d(draw.data(), j.raw, meta.length, nullptr) ||
                                    tb_decode_to_f32(draw.data(), dt, w.data(), n, nullptr) || tb_stream_sync(nullptr)))) {
            j.read_ok = false;
            return;
        }
        TensorDense<float> g(w.shape(), DeviceLocation::kDevice);
        if (n && (!scaled_copy(w, 0.01f, g) || tb_stream_sync(nullptr))) {
            j.skip_silently = true;
            return;
        }
        j.stage = w.empty() ? Stage::kEhap : prune_tensor(o_, w, g, j.result);
    }

    const Options& o_;
    loader::SafeTensorsFile& sf_;
    std::vector<Job>& jobs_;
    int gpus_;
    std::thread reader_;
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_room_, cv_ready_, cv_done_;
    std::deque<std::size_t> ready_;
    std::vector<std::pair<std::byte*, std::size_t>> pool_;
    std::size_t in_flight_ = 0;
    bool reader_done_ = false;
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
    std::vector<Job> jobs;
    for (const auto& meta : metas)
        if (meta.dtype == loader::STDtype::kF32 || meta.dtype == loader::STDtype::kBF16 ||
            meta.dtype == loader::STDtype::kF16) {
            jobs.emplace_back();
            jobs.back().meta = &meta;
        }
    Pipeline pipe(o, sf, jobs, o.gpus);
    pipe.start();
    for (std::size_t i = 0; i < jobs.size(); ++i) {
        Job& j = pipe.wait(i);
        struct Release {
            Pipeline& p;
            Job& j;
            ~Release() { p.release(j); }
        } release{pipe, j};
        const auto& meta = *j.meta;
        if (!j.read_ok) { TENSORBIT_LOG_WARN("  SKIP {}: read error", meta.name); continue; }
        if (j.skip_silently) continue;
        TENSORBIT_LOG_INFO("  [{}] {} — {} elements", count, meta.name, meta.numel);
        const Pruned& p = j.result;
        if (j.stage == Stage::kEhap) { TENSORBIT_LOG_WARN("    SKIP (EHAP failed)"); continue; }
        if (j.stage == Stage::kCoring) { TENSORBIT_LOG_WARN("    SKIP (CORING failed)"); continue; }
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
    pipe.join();
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
        else if (a == "--gpus") parse_number(next(), o.gpus);
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
    if (o.gpus < 1 || o.gpus > ndev) {
        TENSORBIT_LOG_FATAL("--gpus {} outside 1..{} (visible devices)", o.gpus, ndev);
        return 1;
    }
    TENSORBIT_LOG_INFO("Tensorbit Core v0.2.0 — Pruning Pipeline (B200)");
    return o.use_mock ? run_mock(o) : run_model(o);
}

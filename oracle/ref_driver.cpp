// Oracle harness: extern "C" entry points over the REFERENCE's own CPU code.
//
// Test infrastructure only.  This file is compiled by oracle/Makefile against
// the reference headers where they lie (include/tensorbit/core/*.hpp) and the
// reference CLI translation unit src/main.cpp (pulled in below so its
// anonymous-namespace helpers - mock tensor generator, safetensors decode - are
// reachable).  The resulting oracle/_ref/libtb_ref.so is used only by tests/,
// the golden-fixture generator and bench.py's CPU-baseline leg, never by the
// shipped library.
//
// Every function reproduces one call sequence of the reference library, citing
// the file:line of that sequence.

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <span>
#include <string>
#include <thread>
#include <vector>

#define main tb_prune_reference_main
#include "../src/main.cpp"  // resolved through -I <reference>/include
#undef main

using namespace tensorbit::core;

namespace {

TensorDense<float> host_tensor(const float* src, std::size_t n) {
    TensorDense<float> t(std::span<const std::size_t>(&n, 1), DeviceLocation::kHost);
    if (src) std::memcpy(t.data(), src, n * sizeof(float));
    return t;
}

TensorDense<uint8_t> host_bytes(std::size_t n) {
    return TensorDense<uint8_t>(std::span<const std::size_t>(&n, 1), DeviceLocation::kHost);
}

EHAPConfig ehap_config(float beta, float damping, int mode, int use_fisher, int normalize,
                       float sparsity) {
    EHAPConfig c;
    c.ema_decay = beta;
    c.damping = damping;
    c.importance_mode = static_cast<ImportanceMode>(mode);
    c.use_diagonal_fisher = use_fisher != 0;
    c.normalize_fisher = normalize != 0;
    c.sparsity_ratio = sparsity;
    return c;
}

CORINGConfig coring_config(int n, int m, int strategy, int rounds, int redist, int permute,
                           int hw_layout) {
    CORINGConfig c;
    c.N = n;
    c.M = m;
    c.use_cuda = true;
    c.mask_strategy = static_cast<MaskStrategy>(strategy);
    c.iterative_rounds = rounds;
    c.redist_mode = static_cast<RedistMode>(redist);
    c.permute_weights = permute != 0;
    c.hardware_aware_layout = hw_layout != 0;
    return c;
}

// Feeds S gradient samples ([S, N], sample-major) through accumulate_fisher
// (include/tensorbit/core/ehap.hpp:148-201), one call per sample.
int feed_fisher(EHAPPruner<float>& ehap, const float* grads, std::size_t S, std::size_t N,
                float alpha) {
    for (std::size_t s = 0; s < S; ++s) {
        auto g = host_tensor(grads + s * N, N);
        auto r = ehap.accumulate_fisher(g, alpha);
        if (!r) return 100 + static_cast<int>(r.error());
    }
    return 0;
}

}  // namespace

extern "C" {

// Fisher diagonal after S EMA steps (ehap.hpp:148-201).  Returns 1 if the
// pruner holds no Fisher state (use_diagonal_fisher == false).
int ref_fisher(const float* grads, std::size_t S, std::size_t N, float alpha, float beta,
               int use_fisher, float* F_out) {
    EHAPPruner<float> ehap(ehap_config(beta, 0.01f, 0, use_fisher, 0, 0.5f));
    int rc = feed_fisher(ehap, grads, S, N, alpha);
    if (rc) return rc;
    if (ehap.fisher_diagonal().empty()) return 1;
    std::memcpy(F_out, ehap.fisher_diagonal().data(), N * sizeof(float));
    return 0;
}

// accumulate_fisher x S, then compute_importance (ehap.hpp:206-285).
int ref_importance(const float* grads, std::size_t S, const float* w, std::size_t N, float alpha,
                   float beta, float damping, int mode, int use_fisher, int normalize,
                   float* s_out) {
    EHAPPruner<float> ehap(ehap_config(beta, damping, mode, use_fisher, normalize, 0.5f));
    int rc = feed_fisher(ehap, grads, S, N, alpha);
    if (rc) return rc;
    auto wt = host_tensor(w, N);
    auto st = host_tensor(nullptr, N);
    auto r = ehap.compute_importance(wt, st);
    if (!r) return 100 + static_cast<int>(r.error());
    std::memcpy(s_out, st.data(), N * sizeof(float));
    return 0;
}

// CORINGPruner::generate_nm_mask (coring.hpp:90-165).  mask_out receives the
// whole N-byte buffer the caller allocates (src/main.cpp:396), of which the
// first N/M bytes are the packed groups.
int ref_nm_mask(const float* s, std::size_t N, int n, int m, int strategy, int rounds,
                int permute, int hw_layout, uint8_t* mask_out) {
    CORINGPruner<float> coring(coring_config(n, m, strategy, rounds, 0, permute, hw_layout));
    auto st = host_tensor(s, N);
    auto mk = host_bytes(N);
    auto r = coring.generate_nm_mask(st, mk);
    if (!r) return 100 + static_cast<int>(r.error());
    std::memcpy(mask_out, mk.data(), N);
    return 0;
}

// Empty-tensor / error behaviour of generate_nm_mask: N may be 0.
int ref_nm_mask_status(std::size_t N_scores, std::size_t N_mask, int n, int m) {
    CORINGPruner<float> coring(coring_config(n, m, 0, 3, 0, 0, 0));
    TensorDense<float> st = N_scores ? host_tensor(nullptr, N_scores)
                                     : TensorDense<float>(std::span<const std::size_t>{}, DeviceLocation::kHost);
    TensorDense<uint8_t> mk = N_mask ? host_bytes(N_mask)
                                     : TensorDense<uint8_t>(std::span<const std::size_t>{}, DeviceLocation::kHost);
    auto r = coring.generate_nm_mask(st, mk);
    return r ? 0 : static_cast<int>(r.error());
}

// CORINGPruner::prune (coring.hpp:299-313) followed by the second
// generate_nm_mask the CLI performs for the .tb mask bytes (src/main.cpp:398-409).
int ref_coring_prune(const float* s, float* w_inout, std::size_t N, int n, int m, int strategy,
                     int rounds, int redist, int permute, int hw_layout, uint8_t* mask_out,
                     std::size_t* pruned_out) {
    CORINGPruner<float> coring(coring_config(n, m, strategy, rounds, redist, permute, hw_layout));
    auto st = host_tensor(s, N);
    auto wt = host_tensor(w_inout, N);
    auto r = coring.prune(st, wt);
    if (!r) return 100 + static_cast<int>(r.error());
    auto mk = host_bytes(N);
    auto r2 = coring.generate_nm_mask(st, mk);
    if (!r2) return 200 + static_cast<int>(r2.error());
    std::memcpy(w_inout, wt.data(), N * sizeof(float));
    std::memcpy(mask_out, mk.data(), N / static_cast<std::size_t>(m));
    if (pruned_out) *pruned_out = r.value();
    return 0;
}

// CORINGPruner::apply_mask then redistribute on a caller-supplied mask
// (coring.hpp:170-294), i.e. redistribution with the weights the caller holds.
int ref_apply_redistribute(float* w_inout, const uint8_t* mask, const float* s, std::size_t N,
                           int n, int m, int redist, int do_apply, std::size_t* pruned_out) {
    CORINGPruner<float> coring(coring_config(n, m, 0, 3, redist, 0, 0));
    auto wt = host_tensor(w_inout, N);
    auto st = host_tensor(s, N);
    auto mk = host_bytes(N);
    std::memcpy(mk.data(), mask, N / static_cast<std::size_t>(m));
    if (do_apply) {
        auto r = coring.apply_mask(wt, mk);
        if (!r) return 100 + static_cast<int>(r.error());
        if (pruned_out) *pruned_out = r.value();
    }
    auto r2 = coring.redistribute(wt, mk, st);
    if (!r2) return 200 + static_cast<int>(r2.error());
    std::memcpy(w_inout, wt.data(), N * sizeof(float));
    return 0;
}

// EHAPPruner::select_pruning_mask (ehap.hpp:290-329) on given scores.
int ref_select_mask(const float* s, std::size_t N, float sparsity, uint8_t* mask_out,
                    std::size_t* pruned_out) {
    EHAPPruner<float> ehap(ehap_config(0.99f, 0.01f, 0, 1, 0, sparsity));
    auto st = host_tensor(s, N);
    auto mk = host_bytes(N);
    auto r = ehap.select_pruning_mask(st, mk);
    if (!r) return 100 + static_cast<int>(r.error());
    std::memcpy(mask_out, mk.data(), N);
    if (pruned_out) *pruned_out = r.value();
    return 0;
}

// The whole per-tensor sequence of tb-prune (src/main.cpp:372-418 mock mode,
// :500-525 real mode), generalised over the configuration:
//   accumulate_fisher x S  ->  [store_gradient x K]  ->  [EHAPPruner::prune]
//   -> compute_importance -> CORINGPruner::prune -> generate_nm_mask.
// ehap_strategy < 0 skips the EHAP prune (the score+mask+pack path alone).
// Outputs: F (may be null), scores of the final compute_importance (may be
// null), pruned weights (in place), mask bytes (N/M), prune counts.
int ref_pipeline(float* w_inout, const float* grads, std::size_t S, std::size_t N, float alpha,
                 float beta, float damping, int imp_mode, int use_fisher, int normalize,
                 int ehap_strategy, float sparsity, int prune_rounds, const float* hist,
                 std::size_t K, int n, int m, int mask_strategy, int rounds, int redist,
                 int permute, float* F_out, float* s_out, uint8_t* mask_out,
                 std::size_t* ehap_pruned, std::size_t* coring_pruned) {
    EHAPConfig ec = ehap_config(beta, damping, imp_mode, use_fisher, normalize, sparsity);
    if (ehap_strategy >= 0) ec.prune_strategy = static_cast<PruneStrategy>(ehap_strategy);
    ec.prune_rounds = static_cast<std::size_t>(prune_rounds);
    EHAPPruner<float> ehap(ec);
    int rc = feed_fisher(ehap, grads, S, N, alpha);
    if (rc) return rc;
    for (std::size_t k = 0; k < K; ++k) {
        auto g = host_tensor(hist + k * N, N);
        auto r = ehap.store_gradient(g);
        if (!r) return 150 + static_cast<int>(r.error());
    }
    auto wt = host_tensor(w_inout, N);
    if (ehap_strategy >= 0) {
        auto r = ehap.prune(wt);
        if (!r) return 200 + static_cast<int>(r.error());
        if (ehap_pruned) *ehap_pruned = r.value();
    }
    CORINGPruner<float> coring(coring_config(n, m, mask_strategy, rounds, redist, permute, 1));
    auto imp = host_tensor(nullptr, N);
    auto mk = host_bytes(N);
    auto ri = ehap.compute_importance(wt, imp);
    if (!ri) return 300 + static_cast<int>(ri.error());
    auto rc2 = coring.prune(imp, wt);
    if (!rc2) return 400 + static_cast<int>(rc2.error());
    if (coring_pruned) *coring_pruned = rc2.value();
    auto rm = coring.generate_nm_mask(imp, mk);
    if (!rm) return 500 + static_cast<int>(rm.error());
    std::memcpy(w_inout, wt.data(), N * sizeof(float));
    std::memcpy(mask_out, mk.data(), N / static_cast<std::size_t>(m));
    if (F_out && !ehap.fisher_diagonal().empty())
        std::memcpy(F_out, ehap.fisher_diagonal().data(), N * sizeof(float));
    if (s_out) std::memcpy(s_out, imp.data(), N * sizeof(float));
    return 0;
}

// Block OBS as tb-prune runs it (src/main.cpp:375-386): accumulate_fisher x S,
// store_gradient x K, then EHAPPruner::prune_block_obs (ehap.hpp:502-704).
// block == 0 keeps the config default (128).
int ref_block_obs(float* w_inout, const float* grads, std::size_t S, const float* hist, std::size_t K,
                  std::size_t N, std::size_t block, float sparsity, float damping, float off_alpha,
                  float fisher_alpha, int use_fisher, std::size_t hist_size, std::size_t* pruned_out) {
    EHAPConfig c = ehap_config(0.99f, damping, 0, use_fisher, 0, sparsity);
    c.prune_strategy = PruneStrategy::kBlockOBS;
    if (block) c.obs_block_size = block;
    c.obs_off_diag_alpha = off_alpha;
    c.gradient_history_size = hist_size;
    EHAPPruner<float> ehap(c);
    int rc = feed_fisher(ehap, grads, S, N, fisher_alpha);
    if (rc) return rc;
    for (std::size_t k = 0; k < K; ++k) {
        auto g = host_tensor(hist + k * N, N);
        auto r = ehap.store_gradient(g);
        if (!r) return 150 + static_cast<int>(r.error());
    }
    auto wt = host_tensor(w_inout, N);
    auto r = ehap.prune(wt);
    if (!r) return 200 + static_cast<int>(r.error());
    std::memcpy(w_inout, wt.data(), N * sizeof(float));
    if (pruned_out) *pruned_out = r.value();
    return 0;
}

// EHAPPruner::compensate_weights (ehap.hpp:367-403).
int ref_compensate(float* w_inout, const uint8_t* mask, const float* s, std::size_t N, int mode) {
    EHAPConfig c;
    c.compensation_mode = static_cast<CompensationMode>(mode);
    EHAPPruner<float> ehap(c);
    auto wt = host_tensor(w_inout, N);
    auto st = host_tensor(s, N);
    auto mk = host_bytes(N);
    std::memcpy(mk.data(), mask, N);
    auto r = ehap.compensate_weights(wt, mk, st);
    if (!r) return 100 + static_cast<int>(r.error());
    std::memcpy(w_inout, wt.data(), N * sizeof(float));
    return 0;
}

// TBWriter::write (serialization.hpp:101-151).
int ref_write_tb(const char* path, const float* w, std::size_t N, const uint8_t* masks,
                 std::size_t G, uint32_t n, uint32_t m) {
    TBWriter writer;
    auto r = writer.write(path, std::span<const float>(w, N), std::span<const uint8_t>(masks, G), n, m);
    return r ? 0 : static_cast<int>(r.error());
}

// FP64 variant (precision byte 3, serialization.hpp:129-130).
int ref_write_tb_f64(const char* path, const double* w, std::size_t N, const uint8_t* masks,
                     std::size_t G, uint32_t n, uint32_t m) {
    TBWriter writer;
    auto r = writer.write(path, std::span<const double>(w, N), std::span<const uint8_t>(masks, G), n, m);
    return r ? 0 : static_cast<int>(r.error());
}

// The mock-mode input generator of tb-prune (src/main.cpp:262-276).
void ref_mock_tensor(std::size_t N, float* w_out, float* g_out) {
    auto [w, g] = load_mock_tensor(N);
    std::memcpy(w_out, w.data(), N * sizeof(float));
    std::memcpy(g_out, g.data(), N * sizeof(float));
}

// BF16 / F16 -> FP32 decode of load_safetensor (src/main.cpp:204-250), run on
// a one-tensor .safetensors file written to tmp_path.
int ref_decode_half(const uint16_t* in, std::size_t n, int is_bf16, const char* tmp_path,
                    float* out) {
    std::string hdr = std::string("{\"t\":{\"dtype\":\"") + (is_bf16 ? "BF16" : "F16") +
                      "\",\"shape\":[" + std::to_string(n) + "],\"data_offsets\":[0," +
                      std::to_string(n * 2) + "]}}";
    {
        std::ofstream f(tmp_path, std::ios::binary | std::ios::trunc);
        uint64_t len = hdr.size();
        f.write(reinterpret_cast<const char*>(&len), 8);
        f.write(hdr.data(), static_cast<std::streamsize>(hdr.size()));
        f.write(reinterpret_cast<const char*>(in), static_cast<std::streamsize>(n * 2));
    }
    loader::SafeTensorsFile sf;
    if (!sf.open(tmp_path)) return 1;
    const auto& metas = sf.tensors();
    if (metas.size() != 1) return 2;
    auto w = load_safetensor(sf, metas[0]);
    if (!w) return 3;
    std::memcpy(out, w.value().data(), n * sizeof(float));
    return 0;
}

// Runs the reference tb-prune CLI in-process (src/main.cpp:284-644).
int ref_tb_prune_main(int argc, char** argv) { return tb_prune_reference_main(argc, argv); }

// CPU baseline: the score+mask+pack sequence of ref_pipeline (no EHAP prune)
// over `threads` disjoint contiguous shards of one tensor, each shard an
// independent reference pruner on its own thread - the reference is
// single-threaded, so host cores are used the way its docs shard work, one
// process/pruner per shard (docs/CLOUD.md:162-169).  Shard boundaries fall on
// group boundaries.  Returns 0 on success.
int ref_parallel_pass(float* w_inout, const float* grads, std::size_t S, std::size_t N,
                      float alpha, float beta, float damping, int imp_mode, int n, int m,
                      int mask_strategy, int rounds, int redist, uint8_t* mask_out,
                      int threads) {
    if (threads < 1) threads = 1;
    std::size_t G = N / static_cast<std::size_t>(m);
    std::atomic<int> err{0};
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        std::size_t g0 = G * static_cast<std::size_t>(t) / static_cast<std::size_t>(threads);
        std::size_t g1 = G * static_cast<std::size_t>(t + 1) / static_cast<std::size_t>(threads);
        if (g1 <= g0) continue;
        pool.emplace_back([=, &err] {
            std::size_t e0 = g0 * static_cast<std::size_t>(m), ne = (g1 - g0) * static_cast<std::size_t>(m);
            EHAPPruner<float> ehap(ehap_config(beta, damping, imp_mode, 1, 0, 0.5f));
            for (std::size_t s = 0; s < S; ++s) {
                auto g = host_tensor(nullptr, ne);
                std::memcpy(g.data(), grads + s * N + e0, ne * sizeof(float));
                if (!ehap.accumulate_fisher(g, alpha)) { err = 1; return; }
            }
            auto wt = host_tensor(w_inout + e0, ne);
            auto imp = host_tensor(nullptr, ne);
            auto mk = host_bytes(ne);
            CORINGPruner<float> coring(coring_config(n, m, mask_strategy, rounds, redist, 0, 1));
            if (!ehap.compute_importance(wt, imp)) { err = 2; return; }
            if (!coring.prune(imp, wt)) { err = 3; return; }
            if (!coring.generate_nm_mask(imp, mk)) { err = 4; return; }
            std::memcpy(w_inout + e0, wt.data(), ne * sizeof(float));
            std::memcpy(mask_out + g0, mk.data(), g1 - g0);
        });
    }
    for (auto& th : pool) th.join();
    return err.load();
}

}  // extern "C"

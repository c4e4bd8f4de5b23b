/// @file tb_api_test.cpp
/// @brief Self-checking driver for the C++ host API (run by tests/test_host_api.py).
///
/// Without arguments it runs the checks that need no GPU: the reference's own
/// unit tests (tests/test_ehap.cpp:63-144, tests/test_coring.cpp:62-160: config
/// accessors and error paths), the .tb writer/reader and the safetensors
/// reader.  With --gpu it adds the device paths: Fisher accumulation and
/// reset, importance against the reference expression, the documented
/// [5,1,4,2] -> 0b0101 mask, and host-tensor and device-tensor pruning giving
/// identical bytes.  Prints one line per failed check; exit status = failures.

#include <cmath>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <string>
#include <vector>

#include "tensorbit/core/common.hpp"
#include "tensorbit/core/coring.hpp"
#include "tensorbit/core/ehap.hpp"
#include "tensorbit/core/kernels.hpp"
#include "tensorbit/core/loader.hpp"
#include "tensorbit/core/serialization.hpp"
#include "tensorbit/core/tensor.hpp"

using namespace tensorbit::core;

namespace {

int g_fail = 0, g_pass = 0;

void check(bool ok, const char* what, int line) {
    if (ok) { ++g_pass; return; }
    ++g_fail;
    std::printf("FAIL line %d: %s\n", line, what);
}
#define CHECK(c) check((c), #c, __LINE__)

template <typename T>
TensorDense<T> vec(std::initializer_list<T> v, DeviceLocation d = DeviceLocation::kHost) {
    std::size_t n = v.size();
    TensorDense<T> h(std::span<const std::size_t>(&n, 1), DeviceLocation::kHost);
    std::size_t i = 0;
    for (T x : v) h[i++] = x;
    return d == DeviceLocation::kHost ? std::move(h) : h.to_device();
}

template <typename T>
TensorDense<T> empty_tensor() {
    return TensorDense<T>(std::span<const std::size_t>{}, DeviceLocation::kHost);
}

void cpu_checks() {
    // --- EHAP (tests/test_ehap.cpp:63-144) ---
    {
        EHAPConfig c;
        c.damping = 0.01f;
        c.sparsity_ratio = 0.5f;
        EHAPPruner<float> p(c);
        CHECK(p.config().damping == 0.01f);
        CHECK(p.config().sparsity_ratio == 0.5f);
        CHECK(p.config().use_diagonal_fisher);
        CHECK(p.fisher_diagonal().empty());
        auto e = empty_tensor<float>();
        auto r = p.accumulate_fisher(e, 1.0f);
        CHECK(!r.has_value() && r.error() == EHAPError::kZeroSizeTensor);
        auto ri = p.compute_importance(e, e);
        CHECK(!ri && ri.error() == EHAPError::kZeroSizeTensor);
        auto a3 = vec<float>({1, 2, 3});
        auto b2 = vec<float>({1, 2});
        auto rs = p.compute_importance(a3, b2);
        CHECK(!rs && rs.error() == EHAPError::kShapeMismatch);
        auto em = empty_tensor<uint8_t>();
        auto rm = p.select_pruning_mask(e, em);
        CHECK(!rm && rm.error() == EHAPError::kZeroSizeTensor);
        auto m3 = vec<uint8_t>({0, 0, 0});
        EHAPConfig bad;
        bad.sparsity_ratio = 1.0f;
        EHAPPruner<float> pb(bad);
        auto rb = pb.select_pruning_mask(a3, m3);
        CHECK(!rb && rb.error() == EHAPError::kInvalidConfig);
        auto rp = p.prune(e);
        CHECK(!rp && rp.error() == EHAPError::kZeroSizeTensor);
    }
    // --- CORING (tests/test_coring.cpp:62-160) ---
    {
        CORINGConfig c;
        CORINGPruner<float> p(c);
        CHECK(p.config().N == 2 && p.config().M == 4 && p.config().use_cuda);
        auto e = empty_tensor<float>();
        auto em = empty_tensor<uint8_t>();
        auto r = p.generate_nm_mask(e, em);
        CHECK(!r && r.error() == CORINGError::kZeroSizeTensor);
        auto ra = p.apply_mask(e, em);
        CHECK(!ra && ra.error() == CORINGError::kZeroSizeTensor);
        auto rp = p.prune(e, e);
        CHECK(!rp && rp.error() == CORINGError::kZeroSizeTensor);
        auto s6 = vec<float>({1, 2, 3, 4, 5, 6});
        auto m6 = vec<uint8_t>({0, 0, 0, 0, 0, 0});
        auto rs = p.generate_nm_mask(s6, m6);
        CHECK(!rs && rs.error() == CORINGError::kShapeMismatch);
        CORINGConfig bad;
        bad.N = 4;
        bad.M = 4;
        CORINGPruner<float> pb(bad);
        auto s4 = vec<float>({1, 2, 3, 4});
        auto m4 = vec<uint8_t>({0, 0, 0, 0});
        auto rc = pb.generate_nm_mask(s4, m4);
        CHECK(!rc && rc.error() == CORINGError::kInvalidNMConfig);
        CORINGConfig d;
        d.N = 1;
        d.M = 4;
        CORINGPruner<double> pd(d);
        CHECK(pd.config().N == 1 && pd.config().M == 4);
        auto ed = empty_tensor<double>();
        auto rd = pd.prune(ed, ed);
        CHECK(!rd && rd.error() == CORINGError::kZeroSizeTensor);
    }
    // --- Result<T, E> ---
    {
        Result<int, EHAPError> ok = 3;
        Result<int, EHAPError> er = unexpected(EHAPError::kShapeMismatch);
        CHECK(ok && *ok == 3 && ok.value_or(0) == 3);
        CHECK(!er && er.error() == EHAPError::kShapeMismatch && er.value_or(7) == 7);
        Result<void, TBError> v;
        CHECK(v.has_value());
    }
    // --- .tb writer / reader ---
    {
        const std::string path = (std::filesystem::temp_directory_path() / "tb_api_test.tb").string();
        std::vector<float> w = {1.0f, -2.0f, 0.0f, 3.5f, 4.0f, 0.0f, -1.0f, 0.25f};
        std::vector<uint8_t> m = {0x09, 0x06};
        TBWriter wr;
        CHECK(wr.write<float>(path, w, m, 2, 4).has_value());
        CHECK(std::filesystem::file_size(path) == 4096 + 8 * 4 + 2);
        TBReader rd;
        auto h = rd.open(path);
        CHECK(h && h->magic == kTBMagic && h->version == 1 && h->nm_n == 2 && h->nm_m == 4);
        CHECK(h && h->num_weights == 8 && h->num_mask_bytes == 2 && h->masks_offset == 4096 + 32 && h->precision == 0);
        std::vector<float> w2(8);
        std::vector<uint8_t> m2(2);
        CHECK(rd.read_weights<float>(w2).has_value() && w2 == w);
        CHECK(rd.read_masks(m2).has_value() && m2 == m);
        rd.close();
        std::vector<double> wd = {1.0, 2.0, 3.0, 4.0};
        std::vector<uint8_t> md = {0x03};
        CHECK(wr.write<double>(path, wd, md, 2, 4).has_value());
        TBReader rd2;
        auto h2 = rd2.open(path);
        CHECK(h2 && h2->precision == 3 && h2->masks_offset == 4096 + 32);
        rd2.close();
        {
            std::ofstream f(path, std::ios::binary | std::ios::trunc);
            f << "short";
        }
        TBReader rd3;
        auto h3 = rd3.open(path);
        CHECK(!h3 && h3.error() == TBError::kTruncated);
        {
            std::vector<char> junk(4096, 0);
            std::ofstream f(path, std::ios::binary | std::ios::trunc);
            f.write(junk.data(), 4096);
        }
        TBReader rd4;
        auto h4 = rd4.open(path);
        CHECK(!h4 && h4.error() == TBError::kBadMagic);
        std::filesystem::remove(path);
    }
    // --- safetensors reader ---
    {
        const std::string path = (std::filesystem::temp_directory_path() / "tb_api_test.safetensors").string();
        const std::string hdr =
            "{\"__metadata__\":{\"format\":\"pt\"},\"a/w\":{\"dtype\":\"F32\",\"shape\":[2,2],\"data_offsets\":[0,16]},"
            "\"b\":{\"dtype\":\"BF16\",\"shape\":[4],\"data_offsets\":[16,24]},\"c\":{\"dtype\":\"I64\",\"shape\":[1],"
            "\"data_offsets\":[24,32]}}";
        {
            std::ofstream f(path, std::ios::binary | std::ios::trunc);
            const uint64_t n = hdr.size();
            f.write(reinterpret_cast<const char*>(&n), 8);
            f << hdr;
            std::vector<char> data(32, 1);
            f.write(data.data(), 32);
        }
        loader::SafeTensorsFile sf;
        CHECK(sf.open(path).has_value());
        const auto& t = sf.tensors();
        CHECK(t.size() == 4);
        CHECK(t.size() == 4 && t[0].name == "__metadata__" && t[0].dtype == loader::STDtype::kUnknown);
        CHECK(t.size() == 4 && t[1].name == "a/w" && t[1].numel == 4 && t[1].length == 16 && t[1].offset == 0);
        CHECK(t.size() == 4 && t[2].dtype == loader::STDtype::kBF16 && t[2].offset == 16 && t[2].length == 8);
        CHECK(sf.find("c") && sf.find("c")->dtype == loader::STDtype::kI64);
        std::vector<std::byte> buf(16);
        CHECK(sf.read_tensor_data(t[1], buf).has_value());
        sf.close();
        loader::SafeTensorsFile bad;
        CHECK(!bad.open("/nonexistent/file").has_value());
        std::filesystem::remove(path);
    }
}

void gpu_checks() {
    // Reset (tests/test_ehap.cpp:78-96) with a host gradient.
    {
        EHAPConfig c;
        EHAPPruner<float> p(c);
        auto g = vec<float>({1.0f, 2.0f, 3.0f, 4.0f});
        CHECK(p.accumulate_fisher(g, 1.0f).has_value());
        CHECK(!p.fisher_diagonal().empty() && p.fisher_diagonal()[3] == 16.0f);
        p.reset();
        CHECK(p.fisher_diagonal().empty() && p.step_count() == 0);
    }
    // Importance against the reference expression w*w*(F+damp) (ehap.hpp:268-270).
    {
        EHAPConfig c;
        EHAPPruner<float> p(c);
        auto g1 = vec<float>({0.1f, -0.2f, 0.3f, 0.05f});
        auto g2 = vec<float>({0.2f, 0.1f, -0.1f, 0.4f});
        CHECK(p.accumulate_fisher(g1, 0.01f).has_value());
        CHECK(p.accumulate_fisher(g2, 0.01f).has_value());
        auto w = vec<float>({0.5f, -1.5f, 2.0f, 0.01f});
        auto s = vec<float>({0, 0, 0, 0});
        CHECK(p.compute_importance(w, s).has_value());
        const float gg1[4] = {0.1f, -0.2f, 0.3f, 0.05f}, gg2[4] = {0.2f, 0.1f, -0.1f, 0.4f}, ww[4] = {0.5f, -1.5f, 2.0f, 0.01f};
        bool same = true;
        for (int i = 0; i < 4; ++i) {
            float F = 0.01f * gg1[i] * gg1[i];
            const float contrib = 0.01f * (1.0f - 0.99f);
            F = 0.99f * F + contrib * gg2[i] * gg2[i];
            const float ref = ww[i] * ww[i] * (F + 0.01f);
            same = same && std::memcmp(&ref, &s[i], 4) == 0;
        }
        CHECK(same);
    }
    // docs/TODO.md:101: [5,1,4,2] -> 0b0101, host and device tensors, all strategies.
    for (auto strat : {MaskStrategy::kTopN, MaskStrategy::kOptimal, MaskStrategy::kIterative}) {
        CORINGConfig c;
        c.mask_strategy = strat;
        CORINGPruner<float> p(c);
        auto s = vec<float>({5, 1, 4, 2});
        auto m = vec<uint8_t>({0, 0, 0, 0});
        CHECK(p.generate_nm_mask(s, m).has_value() && m[0] == 0x05);
        auto sd = vec<float>({5, 1, 4, 2}, DeviceLocation::kDevice);
        auto md = vec<uint8_t>({0, 0, 0, 0}, DeviceLocation::kDevice);
        CHECK(p.generate_nm_mask(sd, md).has_value() && md.to_host()[0] == 0x05);
    }
    // One-shot EHAP + CORING on host tensors and on device tensors: same bytes.
    {
        const std::size_t n = 4096;
        std::vector<float> hw(n), hg(n);
        for (std::size_t i = 0; i < n; ++i) {
            hw[i] = std::sin(0.37f * static_cast<float>(i)) * 0.05f;
            hg[i] = std::cos(0.11f * static_cast<float>(i)) * 0.01f;
        }
        auto run = [&](DeviceLocation where, std::vector<float>& wout, std::vector<uint8_t>& mout) {
            TensorDense<float> w(std::span<const std::size_t>(&n, 1), DeviceLocation::kHost);
            TensorDense<float> g(std::span<const std::size_t>(&n, 1), DeviceLocation::kHost);
            std::memcpy(w.data(), hw.data(), n * 4);
            std::memcpy(g.data(), hg.data(), n * 4);
            if (where == DeviceLocation::kDevice) { w = w.to_device(); g = g.to_device(); }
            EHAPPruner<float> e(EHAPConfig{});
            CHECK(e.accumulate_fisher(g, 0.01f).has_value());
            auto pr = e.prune(w);
            CHECK(pr && pr.value() == n / 2);
            CORINGConfig cc;
            cc.redist_mode = RedistMode::kProportional;
            CORINGPruner<float> c(cc);
            TensorDense<float> imp(w.shape(), where);
            TensorDense<uint8_t> mk(w.shape(), where);
            CHECK(e.compute_importance(w, imp).has_value());
            auto cr = c.prune(imp, w);
            CHECK(cr && cr.value() == n / 2);
            CHECK(c.generate_nm_mask(imp, mk).has_value());
            auto wh = where == DeviceLocation::kDevice ? w.to_host() : std::move(w);
            auto mh = where == DeviceLocation::kDevice ? mk.to_host() : std::move(mk);
            wout.assign(wh.data(), wh.data() + n);
            mout.assign(mh.data(), mh.data() + n / 4);
        };
        std::vector<float> w1, w2;
        std::vector<uint8_t> m1, m2;
        run(DeviceLocation::kHost, w1, m1);
        run(DeviceLocation::kDevice, w2, m2);
        CHECK(w1.size() == n && std::memcmp(w1.data(), w2.data(), n * 4) == 0 && m1 == m2);
    }
    // The seven legacy launchers through kernels.hpp.
    {
        auto F = vec<float>({0, 0, 0, 0}, DeviceLocation::kDevice);
        auto g = vec<float>({1, 2, 3, 4}, DeviceLocation::kDevice);
        kernels::launch_fisher_accumulate(F.data(), g.data(), 4, 1.0f, nullptr);
        kernels::launch_fisher_beta_decay(F.data(), 0.5f, 4, nullptr);
        auto h = F.to_host();
        CHECK(h[0] == 0.5f && h[3] == 8.0f);
    }
}

}  // namespace

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::string(argv[1]) == "--gpu";
    cpu_checks();
    if (gpu) gpu_checks();
    std::printf("tb-api-test: %d passed, %d failed%s\n", g_pass, g_fail, gpu ? " (with GPU checks)" : "");
    return g_fail;
}

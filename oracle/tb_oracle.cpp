// CPU restatement ("port" oracle) of the reference pruning path.
//
// TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
// CPU-baseline leg of bench.py as the checker; never linked into the shipped
// library.  Each function restates one reference routine in scalar FP32 with
// the reference's expression trees (built with -ffp-contract=off, so no fused
// multiply-add), citing the reference file:line it follows.  Where the
// reference calls a standard-library algorithm whose tie behaviour is
// implementation-defined (std::nth_element, std::sort), this restatement calls
// the same standard-library routine with the same comparator, so both agree
// when built by the same toolchain.

#include "tb_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <random>
#include <utility>
#include <vector>

namespace {

enum Err { kShapeMismatch = 1, kZeroSize = 2, kInvalidConfig = 3 };

// Fisher state of one EHAPPruner: F plus its step counter
// (include/tensorbit/core/ehap.hpp:734-736).
struct Fisher {
    std::vector<float> F;
    std::size_t steps = 0;
};

// accumulate_fisher, host branch (ehap.hpp:148-165,186-200).
int fisher_step(Fisher& st, const float* g, std::size_t N, float alpha, float beta,
                bool use_fisher) {
    if (N == 0) return kZeroSize;
    if (!use_fisher) return 0;
    if (st.F.empty()) { st.F.assign(N, 0.0f); st.steps = 0; }
    if (st.F.size() != N) return kShapeMismatch;
    const float one_m_beta = 1.0f - beta;
    if (st.steps == 0) {
        for (std::size_t i = 0; i < N; ++i) st.F[i] = (alpha * g[i]) * g[i];
    } else {
        const float contrib = alpha * one_m_beta;
        for (std::size_t i = 0; i < N; ++i) st.F[i] = beta * st.F[i] + (contrib * g[i]) * g[i];
    }
    ++st.steps;
    return 0;
}

// apply_fisher_normalization (ehap.hpp:720-731): sequential float sum.
void normalize_fisher(Fisher& st) {
    if (st.F.empty()) return;
    float norm = 0.0f;
    for (float v : st.F) norm += v * v;
    norm = std::sqrt(norm);
    if (norm > 0.0f) {
        const float inv = 1.0f / norm;
        for (float& v : st.F) v *= inv;
    }
}

// compute_importance, host branch (ehap.hpp:206-221,256-284).
int importance(Fisher& st, const float* w, float* s, std::size_t N, float damping, int mode,
               bool normalize) {
    if (N == 0) return kZeroSize;
    const float damp = damping;
    const bool have_f = !st.F.empty();
    if (have_f && normalize) normalize_fisher(st);
    if (!have_f) {
        for (std::size_t i = 0; i < N; ++i) s[i] = w[i] * w[i];
        return 0;
    }
    const float* F = st.F.data();
    for (std::size_t i = 0; i < N; ++i) {
        const float x = w[i];
        switch (mode) {
        case 0: s[i] = x * x * (F[i] + damp); break;                       // kOBD
        case 1: s[i] = (x * x) / (F[i] + damp); break;                     // kOBS
        default: s[i] = (x * x * (F[i] + damp)) / (1.0f + x * x); break;   // kNormalized
        }
    }
    return 0;
}

// generate_topn (coring.hpp:376-392): the reference's nth_element on
// (score, index) pairs ordered by score, descending.
uint8_t topn_group(const float* v, int n, int m) {
    std::pair<float, int> buf[32];
    for (int i = 0; i < m; ++i) buf[i] = {v[i], i};
    std::nth_element(buf, buf + n, buf + m, [](auto& a, auto& b) { return a.first > b.first; });
    uint8_t byte = 0;
    for (int k = 0; k < n; ++k) byte |= static_cast<uint8_t>(1u << buf[k].second);
    return byte;
}

// generate_optimal (coring.hpp:397-422): every N-subset in Gosper order,
// sums accumulated in ascending index order, first strict maximum wins.
uint8_t optimal_group(const float* v, int n, int m) {
    if (m > 16) return topn_group(v, n, m);
    uint32_t best = 0;
    float best_sum = -std::numeric_limits<float>::max();
    uint32_t bits = (1u << n) - 1u;
    const uint32_t limit = 1u << m;
    while (bits < limit) {
        float sum = 0.0f;
        for (int i = 0; i < m; ++i)
            if (bits & (1u << i)) sum += v[i];
        if (sum > best_sum) { best_sum = sum; best = bits; }
        const uint32_t c = bits & (0u - bits);
        const uint32_t r = bits + c;
        bits = (((r ^ bits) >> 2) / c) | r;
    }
    return static_cast<uint8_t>(best);
}

// One swap-refine round of generate_iterative for one group
// (coring.hpp:437-453): first pruned slot (ascending) that beats the first
// kept slot (ascending) swaps with it.  Returns true if the byte changed.
bool refine_group(const float* v, int m, uint8_t& byte) {
    for (int pi = 0; pi < m; ++pi) {
        if (byte & (1u << pi)) continue;
        for (int ki = 0; ki < m; ++ki) {
            if (!(byte & (1u << ki))) continue;
            if (v[pi] > v[ki]) {
                byte = static_cast<uint8_t>(byte & ~(1u << ki));
                byte = static_cast<uint8_t>(byte | (1u << pi));
                return true;
            }
        }
    }
    return false;
}

// apply_permutation (coring.hpp:340-357): per group, values sorted by |s|
// descending with the reference's std::sort call; indices are discarded.
void permute_groups(const float* in, float* out, std::size_t G, int m) {
    std::vector<std::pair<float, int>> buf(static_cast<std::size_t>(m));
    for (std::size_t g = 0; g < G; ++g) {
        const float* v = in + g * static_cast<std::size_t>(m);
        for (int i = 0; i < m; ++i) buf[static_cast<std::size_t>(i)] = {v[i], i};
        std::sort(buf.begin(), buf.end(),
                  [](auto& a, auto& b) { return std::abs(a.first) > std::abs(b.first); });
        for (int i = 0; i < m; ++i) out[g * static_cast<std::size_t>(m) + static_cast<std::size_t>(i)] = buf[static_cast<std::size_t>(i)].first;
    }
}

// generate_nm_mask (coring.hpp:90-165,321-330), host branch.
int nm_mask(const float* s, std::size_t Ns, std::size_t Nm, int n, int m, int strategy, int rounds,
            bool permute, uint8_t* mask) {
    if (Ns == 0 || Nm == 0) return kZeroSize;
    if (Ns != Nm) return kShapeMismatch;
    if (n <= 0 || m <= 0 || n >= m) return kInvalidConfig;
    if (Ns % static_cast<std::size_t>(m) != 0) return kShapeMismatch;
    const std::size_t G = Ns / static_cast<std::size_t>(m);
    std::vector<float> perm;
    if (permute) {
        perm.resize(Ns);
        permute_groups(s, perm.data(), G, m);
        s = perm.data();
    }
    for (std::size_t g = 0; g < G; ++g) {
        const float* v = s + g * static_cast<std::size_t>(m);
        if (strategy == 1) mask[g] = optimal_group(v, n, m);
        else mask[g] = topn_group(v, n, m);
    }
    if (strategy == 2) {
        // Per-group convergence is equivalent to the reference's global
        // early exit: a group that did not change in a round sees the same
        // byte and scores next round, so it cannot change later either.
        for (std::size_t g = 0; g < G; ++g) {
            const float* v = s + g * static_cast<std::size_t>(m);
            for (int r = 0; r < rounds; ++r)
                if (!refine_group(v, m, mask[g])) break;
        }
    }
    return 0;
}

// CORINGPruner::apply_mask, host branch (coring.hpp:170-223).
int coring_apply(float* w, std::size_t Nw, const uint8_t* mask, std::size_t Nm, int n, int m,
                 std::size_t* pruned) {
    if (Nw == 0 || Nm == 0) return kZeroSize;
    if (Nw != Nm) return kShapeMismatch;
    const std::size_t G = Nw / static_cast<std::size_t>(m);
    for (std::size_t g = 0; g < G; ++g)
        for (int i = 0; i < m; ++i)
            if (!((mask[g] >> i) & 1u)) w[g * static_cast<std::size_t>(m) + static_cast<std::size_t>(i)] = 0.0f;
    if (pruned) *pruned = G * static_cast<std::size_t>(m - n);
    return 0;
}

// CORINGPruner::redistribute (coring.hpp:228-294).
void redistribute(float* w, const uint8_t* mask, const float* s, std::size_t N, int m, int mode) {
    if (mode == 0) return;
    const std::size_t G = N / static_cast<std::size_t>(m);
    for (std::size_t g = 0; g < G; ++g) {
        const uint8_t byte = mask[g];
        float* wg = w + g * static_cast<std::size_t>(m);
        const float* sg = s + g * static_cast<std::size_t>(m);
        float pruned_mag = 0.0f, kept_sum = 0.0f;
        int kept = 0;
        for (int i = 0; i < m; ++i) {
            if (!((byte >> i) & 1u)) pruned_mag += std::abs(wg[i]);
            else ++kept;
        }
        if (kept == 0 || pruned_mag <= 0.0f) continue;
        if (mode == 2) {
            const float share = pruned_mag / static_cast<float>(kept);
            for (int i = 0; i < m; ++i)
                if ((byte >> i) & 1u) {
                    const float sign = (wg[i] >= 0.0f) ? 1.0f : -1.0f;
                    wg[i] += sign * share;
                }
        } else {
            for (int i = 0; i < m; ++i)
                if ((byte >> i) & 1u) kept_sum += sg[i];
            if (kept_sum <= 0.0f) continue;
            for (int i = 0; i < m; ++i)
                if ((byte >> i) & 1u) {
                    const float frac = sg[i] / kept_sum;
                    const float sign = (wg[i] >= 0.0f) ? 1.0f : -1.0f;
                    wg[i] += sign * pruned_mag * frac;
                }
        }
    }
}

// CORINGPruner::prune (coring.hpp:299-313).
int coring_prune(const float* s, float* w, std::size_t N, int n, int m, int strategy, int rounds,
                 int redist, bool permute, std::vector<uint8_t>& mask, std::size_t* pruned) {
    mask.assign(N, 0);
    int rc = nm_mask(s, N, N, n, m, strategy, rounds, permute, mask.data());
    if (rc) return rc;
    rc = coring_apply(w, N, mask.data(), N, n, m, pruned);
    if (rc) return rc;
    redistribute(w, mask.data(), s, N, m, redist);
    return 0;
}

// select_pruning_mask (ehap.hpp:290-329): global threshold = the (N-keep)-th
// smallest score by the reference's nth_element; ties at it are all kept.
int select_mask(const float* s, std::size_t N, float sp, uint8_t* mask, std::size_t* pruned) {
    if (N == 0) return kZeroSize;
    if (sp <= 0.0f || sp >= 1.0f) return kInvalidConfig;
    std::size_t keep = static_cast<std::size_t>(sp * static_cast<float>(N));
    if (keep == 0) keep = 1;
    if (keep >= N) {
        std::fill_n(mask, N, uint8_t{1});
        if (pruned) *pruned = 0;
        return 0;
    }
    std::vector<float> copy(s, s + N);
    const std::size_t t = N - keep;
    std::nth_element(copy.begin(), copy.begin() + static_cast<std::ptrdiff_t>(t), copy.end());
    const float thr = copy[t];
    std::size_t p = 0;
    for (std::size_t i = 0; i < N; ++i) {
        const bool k = s[i] >= thr;
        mask[i] = k ? 1 : 0;
        if (!k) ++p;
    }
    if (pruned) *pruned = p;
    return 0;
}

// EHAPPruner::prune_one_shot / prune_iterative (ehap.hpp:425-478), with the
// default CompensationMode::kNone (ehap.hpp:372-373).
int ehap_prune(Fisher& st, float* w, std::size_t N, float damping, int mode, bool normalize,
               int strategy, float sparsity, int rounds, std::size_t* pruned) {
    std::vector<float> imp(N);
    std::vector<uint8_t> msk(N);
    auto one_round = [&](float sp, std::size_t* cnt) -> int {
        int rc = importance(st, w, imp.data(), N, damping, mode, normalize);
        if (rc) return rc;
        rc = select_mask(imp.data(), N, sp, msk.data(), nullptr);
        if (rc) return rc;
        std::size_t z = 0;
        for (std::size_t i = 0; i < N; ++i)
            if (!msk[i]) { w[i] = 0.0f; ++z; }
        *cnt = z;
        return 0;
    };
    if (strategy == 1) {
        float cur_keep = 1.0f;
        std::size_t total = 0;
        for (int r = 0; r < rounds; ++r) {
            const float t = static_cast<float>(r + 1) / static_cast<float>(rounds);
            const float target_keep =
                sparsity + (1.0f - sparsity) * static_cast<float>(std::pow(1.0 - t, 3));
            float round_keep = target_keep / cur_keep;
            if (round_keep < 0.0f) round_keep = 0.0f;
            if (round_keep > 1.0f) round_keep = 1.0f;
            std::size_t c = 0;
            int rc = one_round(round_keep, &c);
            if (rc) return rc;
            total += c;
            cur_keep = round_keep;
        }
        *pruned = total;
        return 0;
    }
    return one_round(sparsity, pruned);
}

}  // namespace

extern "C" {

int port_fisher(const float* grads, size_t S, size_t N, float alpha, float beta, int use_fisher,
                float* F_out) {
    Fisher st;
    for (size_t s = 0; s < S; ++s) {
        int rc = fisher_step(st, grads + s * N, N, alpha, beta, use_fisher != 0);
        if (rc) return 100 + rc;
    }
    if (st.F.empty()) return 1;
    std::memcpy(F_out, st.F.data(), N * sizeof(float));
    return 0;
}

int port_importance(const float* grads, size_t S, const float* w, size_t N, float alpha,
                    float beta, float damping, int mode, int use_fisher, int normalize,
                    float* s_out) {
    Fisher st;
    for (size_t s = 0; s < S; ++s) {
        int rc = fisher_step(st, grads + s * N, N, alpha, beta, use_fisher != 0);
        if (rc) return 100 + rc;
    }
    int rc = importance(st, w, s_out, N, damping, mode, normalize != 0);
    return rc ? 100 + rc : 0;
}

int port_nm_mask(const float* s, size_t N, int n, int m, int strategy, int rounds, int permute,
                 int /*hw_layout: a no-op in the reference, coring.hpp:367-371*/,
                 uint8_t* mask_out) {
    std::vector<uint8_t> mk(N, 0);
    int rc = nm_mask(s, N, N, n, m, strategy, rounds, permute != 0, mk.data());
    if (rc) return 100 + rc;
    std::memcpy(mask_out, mk.data(), N);
    return 0;
}

int port_nm_mask_status(size_t N_scores, size_t N_mask, int n, int m) {
    std::vector<float> s(N_scores, 0.0f);
    std::vector<uint8_t> mk(N_mask, 0);
    return nm_mask(s.data(), N_scores, N_mask, n, m, 0, 3, false, mk.data());
}

int port_coring_prune(const float* s, float* w_inout, size_t N, int n, int m, int strategy,
                      int rounds, int redist, int permute, int /*hw_layout*/, uint8_t* mask_out,
                      size_t* pruned_out) {
    std::vector<uint8_t> mk;
    size_t pruned = 0;
    int rc = coring_prune(s, w_inout, N, n, m, strategy, rounds, redist, permute != 0, mk, &pruned);
    if (rc) return 100 + rc;
    std::vector<uint8_t> mk2(N, 0);
    rc = nm_mask(s, N, N, n, m, strategy, rounds, permute != 0, mk2.data());
    if (rc) return 200 + rc;
    std::memcpy(mask_out, mk2.data(), N / static_cast<size_t>(m));
    if (pruned_out) *pruned_out = pruned;
    return 0;
}

int port_apply_redistribute(float* w_inout, const uint8_t* mask, const float* s, size_t N, int n,
                            int m, int redist, int do_apply, size_t* pruned_out) {
    if (do_apply) {
        int rc = coring_apply(w_inout, N, mask, N, n, m, pruned_out);
        if (rc) return 100 + rc;
    }
    redistribute(w_inout, mask, s, N, m, redist);
    return 0;
}

int port_select_mask(const float* s, size_t N, float sparsity, uint8_t* mask_out,
                     size_t* pruned_out) {
    int rc = select_mask(s, N, sparsity, mask_out, pruned_out);
    return rc ? 100 + rc : 0;
}

// The tb-prune per-tensor sequence (src/main.cpp:372-409, :500-525).  BlockOBS
// (ehap_strategy 2) is not restated here.
int port_pipeline(float* w_inout, const float* grads, size_t S, size_t N, float alpha, float beta,
                  float damping, int imp_mode, int use_fisher, int normalize, int ehap_strategy,
                  float sparsity, int prune_rounds, const float* /*hist*/, size_t /*K*/, int n,
                  int m, int mask_strategy, int rounds, int redist, int permute, float* F_out,
                  float* s_out, uint8_t* mask_out, size_t* ehap_pruned, size_t* coring_pruned) {
    if (ehap_strategy == 2) return -1;
    Fisher st;
    for (size_t s = 0; s < S; ++s) {
        int rc = fisher_step(st, grads + s * N, N, alpha, beta, use_fisher != 0);
        if (rc) return 100 + rc;
    }
    if (ehap_strategy >= 0) {
        if (N == 0) return 200 + kZeroSize;
        size_t p = 0;
        int rc = ehap_prune(st, w_inout, N, damping, imp_mode, normalize != 0, ehap_strategy,
                            sparsity, prune_rounds, &p);
        if (rc) return 200 + rc;
        if (ehap_pruned) *ehap_pruned = p;
    }
    std::vector<float> imp(N);
    int rc = importance(st, w_inout, imp.data(), N, damping, imp_mode, normalize != 0);
    if (rc) return 300 + rc;
    std::vector<uint8_t> mk;
    size_t cp = 0;
    rc = coring_prune(imp.data(), w_inout, N, n, m, mask_strategy, rounds, redist, permute != 0, mk, &cp);
    if (rc) return 400 + rc;
    if (coring_pruned) *coring_pruned = cp;
    std::vector<uint8_t> mk2(N, 0);
    rc = nm_mask(imp.data(), N, N, n, m, mask_strategy, rounds, permute != 0, mk2.data());
    if (rc) return 500 + rc;
    std::memcpy(mask_out, mk2.data(), N / static_cast<size_t>(m));
    if (F_out && !st.F.empty()) std::memcpy(F_out, st.F.data(), N * sizeof(float));
    if (s_out) std::memcpy(s_out, imp.data(), N * sizeof(float));
    return 0;
}

// TBHeader as TBWriter::write fills it (serialization.hpp:30-54,115-134):
// little-endian packed fields, everything else zero.
void port_tb_header(uint8_t out[4096], uint32_t n, uint32_t m, uint64_t num_weights,
                    uint64_t num_mask_bytes, uint32_t elem_size) {
    std::memset(out, 0, 4096);
    auto put32 = [&](size_t off, uint32_t v) { for (int b = 0; b < 4; ++b) out[off + b] = static_cast<uint8_t>(v >> (8 * b)); };
    auto put64 = [&](size_t off, uint64_t v) { for (int b = 0; b < 8; ++b) out[off + b] = static_cast<uint8_t>(v >> (8 * b)); };
    put32(0, 0x31304254u);
    put32(4, 1u);
    put32(8, n);
    put32(12, m);
    put64(16, num_weights);
    put64(24, num_mask_bytes);
    put64(32, 4096u);
    put64(40, 4096u + num_weights * elem_size);
    out[48] = (elem_size == 8) ? 3 : 0;
}

// load_safetensor's BF16 and F16 widening (src/main.cpp:213-245).  The F16
// branch keeps the reference's handling of exponent 0: the 10-bit fraction is
// placed in an FP32 with exponent 0, which is not the IEEE value.
void port_decode_half(const uint16_t* in, size_t n, int is_bf16, float* out) {
    for (size_t i = 0; i < n; ++i) {
        const uint32_t h = in[i];
        uint32_t f;
        if (is_bf16) {
            f = h << 16;
        } else {
            const uint32_t sign = (h >> 15) << 31;
            const uint32_t e = (h >> 10) & 0x1Fu;
            const uint32_t frac = h & 0x3FFu;
            if (e == 0) f = sign | (frac << 13);
            else if (e == 31) f = sign | 0x7F800000u | (frac << 13);
            else f = sign | ((e + 112u) << 23) | (frac << 13);
        }
        std::memcpy(&out[i], &f, 4);
    }
}

// tb-prune's mock tensor (src/main.cpp:262-276): mt19937(42) feeding one
// normal(0, 0.5) distribution, alternating weight and gradient draws.
void port_mock_tensor(size_t N, float* w_out, float* g_out) {
    std::mt19937 rng(42);
    std::normal_distribution<float> dist(0.0f, 0.5f);
    for (size_t i = 0; i < N; ++i) {
        w_out[i] = dist(rng);
        g_out[i] = dist(rng) * 0.1f;
    }
}

// Groups whose N-th and (N+1)-th largest scores differ by at most 1e-6
// relative: |a - b| <= 1e-6 * max(|a|, FLT_MIN).  Exact ties count.
size_t port_near_ties(const float* s, size_t N, int n, int m) {
    size_t G = N / static_cast<size_t>(m), cnt = 0;
    std::vector<float> v(static_cast<size_t>(m));
    for (size_t g = 0; g < G; ++g) {
        std::copy_n(s + g * static_cast<size_t>(m), m, v.begin());
        std::sort(v.begin(), v.end(), [](float a, float b) { return a > b; });
        const float a = v[static_cast<size_t>(n - 1)], b = v[static_cast<size_t>(n)];
        const float scale = std::max(std::abs(a), std::numeric_limits<float>::min());
        if (std::abs(a - b) <= 1e-6f * scale) ++cnt;
    }
    return cnt;
}

// EHAPPruner::compensate_weights (ehap.hpp:367-403) on a 1-byte-per-element mask.
void port_compensate(float* w, const uint8_t* mask, const float* s, size_t N, int mode) {
    if (mode == 0 || N == 0) return;
    if (mode == 1) {
        float delta = 0.0f;
        for (size_t i = 0; i < N; ++i)
            if (!mask[i]) delta += w[i];
        w[N - 1] += delta;
        return;
    }
    for (size_t g = 0; g < N; g += 8) {
        const size_t end = (g + 8 < N) ? g + 8 : N;
        float t_pruned = 0.0f, t_weight = 0.0f;
        for (size_t i = g; i < end; ++i) {
            if (!mask[i]) t_pruned += w[i];
            else t_weight += s[i];
        }
        if (t_weight <= 0.0f) continue;
        for (size_t i = g; i < end; ++i)
            if (mask[i]) w[i] += t_pruned * s[i] / t_weight;
    }
}

// ---- block OBS (ehap.hpp:502-704) -------------------------------------------
// Restated with the operation order of the Eigen stand-in the reference oracle
// is built with (oracle/eigen_subset/Eigen/Dense): products accumulate over the
// inner index from zero, the K x K system is solved by pivoted LDL^T.

namespace {

// Symmetric LDL^T with diagonal pivoting of a K x K column-major matrix and
// solve against the identity: Minv = M^-1.
void ldlt_inverse(std::vector<float>& a, int n, std::vector<float>& inv) {
    auto at = [&](std::vector<float>& m, int i, int j) -> float& { return m[static_cast<size_t>(j * n + i)]; };
    std::vector<int> perm(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) perm[static_cast<size_t>(i)] = i;
    for (int k = 0; k < n; ++k) {
        int p = k;
        float best = std::abs(at(a, k, k));
        for (int i = k + 1; i < n; ++i)
            if (std::abs(at(a, i, i)) > best) { best = std::abs(at(a, i, i)); p = i; }
        if (p != k) {
            std::swap(perm[static_cast<size_t>(k)], perm[static_cast<size_t>(p)]);
            std::vector<float> full = a, sw(a.size());
            auto idx = [&](int i) { return i == k ? p : (i == p ? k : i); };
            for (int j = 0; j < n; ++j)
                for (int i = 0; i < n; ++i) {
                    const int x = idx(i), y = idx(j);
                    if (j < k) at(sw, i, j) = at(full, x, j);
                    else at(sw, i, j) = (x >= y) ? at(full, x, y) : at(full, y, x);
                }
            a = sw;
        }
        const float dk = at(a, k, k);
        if (dk == 0.0f) continue;
        for (int i = k + 1; i < n; ++i) at(a, i, k) /= dk;
        for (int j = k + 1; j < n; ++j)
            for (int i = j; i < n; ++i) at(a, i, j) -= at(a, i, k) * dk * at(a, j, k);
    }
    inv.assign(static_cast<size_t>(n * n), 0.0f);
    std::vector<float> y(static_cast<size_t>(n));
    for (int c = 0; c < n; ++c) {
        for (int i = 0; i < n; ++i) y[static_cast<size_t>(i)] = (perm[static_cast<size_t>(i)] == c) ? 1.0f : 0.0f;
        for (int i = 0; i < n; ++i)
            for (int k = 0; k < i; ++k) y[static_cast<size_t>(i)] -= at(a, i, k) * y[static_cast<size_t>(k)];
        for (int i = 0; i < n; ++i) {
            const float d = at(a, i, i);
            if (d != 0.0f) y[static_cast<size_t>(i)] /= d;
        }
        for (int i = n - 1; i >= 0; --i)
            for (int k = i + 1; k < n; ++k) y[static_cast<size_t>(i)] -= at(a, k, i) * y[static_cast<size_t>(k)];
        for (int i = 0; i < n; ++i) at(inv, perm[static_cast<size_t>(i)], c) = y[static_cast<size_t>(i)];
    }
}

size_t block_obs(float* w, const float* fdiag, const std::vector<const float*>& hist, size_t N, size_t B,
                 float sp, float damp, float alpha) {
    const size_t num_blocks = (N + B - 1) / B;
    const size_t prune_total = N - static_cast<size_t>(sp * static_cast<float>(N));
    if (prune_total == 0) return 0;
    std::vector<float> block_imp(num_blocks, 0.0f);
    for (size_t b = 0; b < num_blocks; ++b) {
        const size_t st = b * B, en = std::min(st + B, N);
        float sum = 0.0f;
        for (size_t i = st; i < en; ++i) {
            float fi = damp;
            if (fdiag) fi += fdiag[i];
            sum += w[i] * w[i] * fi;
        }
        block_imp[b] = sum / static_cast<float>(en - st);
    }
    float mx = 0.0f;
    for (float v : block_imp) if (v > mx) mx = v;
    if (mx <= 0.0f) mx = 1.0f;
    std::vector<float> blk_w(num_blocks);
    const float tau = 4.0f;
    for (size_t b = 0; b < num_blocks; ++b) blk_w[b] = std::exp(-tau * (block_imp[b] / mx));
    std::vector<size_t> target(num_blocks, 0);
    float total_w = 0.0f;
    for (float v : blk_w) total_w += v;
    if (total_w <= 0.0f) total_w = 1.0f;
    size_t allocated = 0;
    for (size_t b = 0; b < num_blocks; ++b) {
        const float share = blk_w[b] / total_w;
        const size_t bs = (b == num_blocks - 1) ? (N - b * B) : B;
        target[b] = static_cast<size_t>(share * static_cast<float>(prune_total));
        if (target[b] >= bs) target[b] = bs > 1 ? bs - 1 : 0;
        allocated += target[b];
    }
    std::ptrdiff_t rem = static_cast<std::ptrdiff_t>(prune_total) - static_cast<std::ptrdiff_t>(allocated);
    for (size_t b = 0; b < num_blocks && rem > 0; ++b) {
        const size_t rb = num_blocks - 1 - b;
        const size_t bs = (rb == num_blocks - 1) ? (N - rb * B) : B;
        while (rem > 0 && target[rb] + 1 < bs) { ++target[rb]; --rem; }
    }
    size_t pruned = 0;
    const int K = hist.empty() ? 1 : static_cast<int>(hist.size());
    for (size_t b = 0; b < num_blocks; ++b) {
        const size_t st = b * B, en = std::min(st + B, N), bs = en - st;
        if (target[b] == 0 || target[b] >= bs) continue;
        std::vector<float> Dinv(bs), U(bs * static_cast<size_t>(K));  // U column-major (i + k*bs)
        for (size_t i = 0; i < bs; ++i) {
            float d = damp;
            if (fdiag) d += fdiag[st + i];
            Dinv[i] = (d > 0.0f) ? (1.0f / d) : 1.0f;
        }
        if (!hist.empty()) {
            for (int k = 0; k < K; ++k) {
                const float age = static_cast<float>(K - 1 - k);
                const float wk = std::exp(-age / 2.0f);
                for (size_t i = 0; i < bs; ++i) U[i + static_cast<size_t>(k) * bs] = wk * hist[static_cast<size_t>(k)][st + i];
            }
        } else {
            for (size_t i = 0; i < bs; ++i) U[i] = std::sqrt(alpha) * w[st + i];
        }
        // M = I + 1e-8 I + (U^T D^-1) U
        std::vector<float> M(static_cast<size_t>(K * K), 0.0f);
        for (int k = 0; k < K; ++k) M[static_cast<size_t>(k * K + k)] = 1.0f;
        for (int k = 0; k < K; ++k) M[static_cast<size_t>(k * K + k)] += 1e-8f;
        for (int j = 0; j < K; ++j)
            for (int i = 0; i < K; ++i) {
                float acc = 0.0f;
                for (size_t x = 0; x < bs; ++x)
                    acc += (U[x + static_cast<size_t>(i) * bs] * Dinv[x]) * U[x + static_cast<size_t>(j) * bs];
                M[static_cast<size_t>(j * K + i)] += acc;
            }
        std::vector<float> Minv;
        ldlt_inverse(M, K, Minv);
        // Hinv = D^-1 - D^-1 S D^-1, S = sum_k1 sum_k2 Minv(k1,k2) u_k1 u_k2^T
        std::vector<float> H(bs * bs);  // column-major
        for (size_t j = 0; j < bs; ++j)
            for (size_t i = 0; i < bs; ++i) {
                float S = 0.0f;
                for (int k1 = 0; k1 < K; ++k1)
                    for (int k2 = 0; k2 < K; ++k2)
                        S += Minv[static_cast<size_t>(k2 * K + k1)] *
                             (U[i + static_cast<size_t>(k1) * bs] * U[j + static_cast<size_t>(k2) * bs]);
                const float h0 = (i == j) ? Dinv[i] : 0.0f;
                H[i + j * bs] = h0 - Dinv[i] * S * Dinv[j];
            }
        std::vector<float> wv(w + st, w + en), col(bs);
        size_t done = 0;
        while (done < target[b]) {
            float min_s = std::numeric_limits<float>::max();
            size_t best = 0;
            for (size_t i = 0; i < bs; ++i) {
                const float hii = H[i + i * bs];
                if (hii <= 0.0f) continue;
                const float sc = (wv[i] * wv[i]) / hii;
                if (sc < min_s) { min_s = sc; best = i; }
            }
            if (min_s >= std::numeric_limits<float>::max() / 2) break;
            const float wi_old = wv[best];
            const float inv_h = 1.0f / H[best + best * bs];
            for (size_t j = 0; j < bs; ++j)
                if (j != best) wv[j] -= wi_old * inv_h * H[j + best * bs];
            wv[best] = 0.0f;
            const float hbb = H[best + best * bs];
            for (size_t i = 0; i < bs; ++i) col[i] = H[i + best * bs];
            for (size_t j = 0; j < bs; ++j)
                for (size_t i = 0; i < bs; ++i) H[i + j * bs] -= (col[i] * col[j]) / hbb;
            ++done;
        }
        std::copy(wv.begin(), wv.end(), w + st);
        pruned += done;
    }
    return pruned;
}

}  // namespace

int port_block_obs(float* w_inout, const float* grads, size_t S, const float* hist, size_t K, size_t N,
                   size_t block, float sparsity, float damping, float off_alpha, float fisher_alpha,
                   int use_fisher, size_t hist_size, size_t* pruned_out) {
    Fisher st;
    for (size_t s = 0; s < S; ++s) {
        int rc = fisher_step(st, grads + s * N, N, fisher_alpha, 0.99f, use_fisher != 0);
        if (rc) return 100 + rc;
    }
    std::vector<const float*> h;
    const size_t keep = hist_size;
    for (size_t k = 0; k < K && keep > 0; ++k) {
        if (h.size() >= keep) h.erase(h.begin());
        h.push_back(hist + k * N);
    }
    if (N == 0) return 200 + kZeroSize;
    const size_t B = block ? block : 128;
    const size_t p = block_obs(w_inout, st.F.empty() ? nullptr : st.F.data(), h, N, B, sparsity, damping, off_alpha);
    if (pruned_out) *pruned_out = p;
    return 0;
}

void port_topn_group(const float* vals, int n, int m, uint8_t* mask_out) {
    *mask_out = topn_group(vals, n, m);
}

}  // extern "C"

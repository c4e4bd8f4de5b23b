// Blockwise OBS with a diagonal + low-rank Hessian, reference semantics
// (EHAPPruner::prune_block_obs, include/tensorbit/core/ehap.hpp:502-704).
//
// Phase 1 (device): per block of B contiguous weights, the mean importance
//   sum_i w_i^2 (lambda + F_i) / |block|, one serial sum per block as the
//   reference writes it (ehap.hpp:522-536).
// Phase 2 (host): max, exp weights, serial total and per-block prune targets
//   with the remainder handed to the last blocks (ehap.hpp:538-577).  These are
//   O(N/B) scalars; the host runs them with the same C library as the
//   reference (std::exp on float) so the targets are identical.
// Phase 3 (device, one CTA per block, one thread per row): D^-1, U (K gradient
//   snapshots or sqrt(alpha) w), M = I + U^T D^-1 U, M^-1 by pivoted LDL^T,
//   then the greedy loop: argmin w_i^2 / H^-1_ii (lowest index on ties), OBS
//   update of the other weights, rank-1 Sherman-Morrison deflation of
//   H^-1 = D^-1 - D^-1 (sum Minv_kl u_k u_l^T) D^-1 (ehap.hpp:582-701), with
//   the deflation applied lazily to the rows the greedy reads.
//
// Every float operation keeps the reference's expression tree (products
// accumulated over the inner index in order from zero, no fused multiply-add);
// the K x K factorisation follows the pivoted LDL^T the reference oracle is
// built with.  The loop is latency-bound CUDA-core work (correctly rounded
// divisions); there is no tensor-core formulation of its serial greedy.
#include <algorithm>
#include <cfloat>
#include <chrono>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "tb_device.cuh"
#include "tb_runtime.h"

namespace tb {
namespace {

constexpr int kMaxK = 16;
constexpr int kMaxBlock = 224;       // one thread per row; the downdate columns must fit in shared memory
constexpr int kObsMaxThreads = 224;  // kMaxBlock rounded up to whole warps

struct ObsParams {
    float* w;
    const float* F;
    const float* hist[kMaxK];
    float wk[kMaxK];
    int K;           // snapshots (0: use sqrt(alpha) * w)
    float sa;        // sqrt(obs_off_diag_alpha)
    float damp;
    size_t N;
    int B;
    const uint32_t* targets;
    const uint32_t* order;   // the block of each CTA
    unsigned long long* pruned;
    int tcap;        // the largest target: rows of the kept downdate columns
};

__global__ void block_importance_kernel(const float* __restrict__ w, const float* __restrict__ F, float damp,
                                        size_t N, int B, size_t nb, float* __restrict__ out) {
    for (size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x; b < nb; b += (size_t)gridDim.x * blockDim.x) {
        const size_t st = b * B, en = st + B < N ? st + B : N;
        float sum = 0.0f;
        for (size_t i = st; i < en; ++i) {
            const float fi = F ? __fadd_rn(damp, F[i]) : damp;
            sum = __fadd_rn(sum, __fmul_rn(__fmul_rn(w[i], w[i]), fi));
        }
        out[b] = __fdiv_rn(sum, static_cast<float>(en - st));
    }
}

// Pivoted LDL^T inverse of the K x K column-major matrix a (in place, K <= 16),
// written to inv; one thread.
__device__ void ldlt_inverse(float* a, int n, float* inv) {
    int perm[kMaxK];
    float sw[kMaxK * kMaxK];
    for (int i = 0; i < n; ++i) perm[i] = i;
    for (int k = 0; k < n; ++k) {
        int p = k;
        float best = fabsf(a[k * n + k]);
        for (int i = k + 1; i < n; ++i)
            if (fabsf(a[i * n + i]) > best) { best = fabsf(a[i * n + i]); p = i; }
        if (p != k) {
            const int t = perm[k]; perm[k] = perm[p]; perm[p] = t;
            for (int j = 0; j < n; ++j)
                for (int i = 0; i < n; ++i) {
                    const int x = i == k ? p : (i == p ? k : i);
                    const int y = j == k ? p : (j == p ? k : j);
                    sw[j * n + i] = (j < k) ? a[j * n + x] : ((x >= y) ? a[y * n + x] : a[x * n + y]);
                }
            for (int e = 0; e < n * n; ++e) a[e] = sw[e];
        }
        const float dk = a[k * n + k];
        if (dk == 0.0f) continue;
        for (int i = k + 1; i < n; ++i) a[k * n + i] = __fdiv_rn(a[k * n + i], dk);
        for (int j = k + 1; j < n; ++j)
            for (int i = j; i < n; ++i)
                a[j * n + i] = __fsub_rn(a[j * n + i], __fmul_rn(__fmul_rn(a[k * n + i], dk), a[k * n + j]));
    }
    float y[kMaxK];
    for (int c = 0; c < n; ++c) {
        for (int i = 0; i < n; ++i) y[i] = (perm[i] == c) ? 1.0f : 0.0f;
        for (int i = 0; i < n; ++i)
            for (int k = 0; k < i; ++k) y[i] = __fsub_rn(y[i], __fmul_rn(a[k * n + i], y[k]));
        for (int i = 0; i < n; ++i) {
            const float d = a[i * n + i];
            if (d != 0.0f) y[i] = __fdiv_rn(y[i], d);
        }
        for (int i = n - 1; i >= 0; --i)
            for (int k = i + 1; k < n; ++k) y[i] = __fsub_rn(y[i], __fmul_rn(a[i * n + k], y[k]));
        for (int i = 0; i < n; ++i) inv[c * n + perm[i]] = y[i];
    }
}

// A candidate of the greedy argmin: its score, row, weight and diagonal entry.
struct ObsCand {
    float v;
    int i;
    float w;
    float h;
};

// smaller score wins, equal scores -> lower row index
__device__ __forceinline__ void cand_merge(ObsCand& a, const ObsCand& b) {
    if (b.v < a.v || (b.v == a.v && b.i < a.i)) a = b;
}

// One CTA per block, one thread per row of the block (blockDim = B rounded up
// to whole warps).  The reference keeps the full B x B inverse and deflates all
// of it after every pruned weight; here the greedy loop keeps only what it
// reads: the diagonal of H^-1 and the weights (each in its row's thread), the
// downdate columns c_s = H^-1[best_s][:] and their pivots h_s.  The one row a
// step needs is formed as the reference's element would have been: H0[best][j]
// (recomputed from U, M^-1 and D^-1 by the same expression tree), minus
// c_s[j] c_s[best] / h_s for every earlier step s in step order -- the same
// operations in the same order, so the same bits, with about a quarter of the
// reference's correctly rounded divisions (they dominate a step) and no B x B
// array, which leaves room for three CTAs per SM.
__global__ void __launch_bounds__(kObsMaxThreads) block_obs_kernel(const ObsParams p) {
    extern __shared__ float smem[];
    const size_t b = p.order[blockIdx.x];
    const size_t st = b * p.B;
    const int bs = static_cast<int>((st + p.B < p.N ? st + p.B : p.N) - st);
    const uint32_t target = p.targets[b];
    if (target == 0 || target >= static_cast<uint32_t>(bs) || target > static_cast<uint32_t>(p.tcap)) return;
    const int K = p.K ? p.K : 1;
    float* U = smem;                      // bs*K, column-major (snapshot k at U + k*bs)
    float* Dinv = U + bs * K;             // bs
    float* M = Dinv + bs;                 // K*K
    float* Minv = M + kMaxK * kMaxK;      // K*K
    float* hs = Minv + kMaxK * kMaxK;     // tcap pivots h_s
    float* Cs = hs + p.tcap;              // tcap x bs downdate columns c_s
    __shared__ ObsCand red[2][kObsMaxThreads / 32];
    const int t = threadIdx.x;
    const int nt = blockDim.x;
    const bool own = t < bs;

    float my_w = 0.0f;
    if (own) {
        const float d = p.F ? __fadd_rn(p.damp, p.F[st + t]) : p.damp;
        Dinv[t] = d > 0.0f ? __fdiv_rn(1.0f, d) : 1.0f;
        my_w = p.w[st + t];
        if (p.K) {
            for (int k = 0; k < K; ++k) U[k * bs + t] = __fmul_rn(p.wk[k], p.hist[k][st + t]);
        } else {
            U[t] = __fmul_rn(p.sa, my_w);
        }
    }
    __syncthreads();
    // M = I + 1e-8 I + (U^T D^-1) U: one thread per entry, inner index in order.
    for (int e = t; e < K * K; e += nt) {
        const int i = e % K, j = e / K;
        float acc = 0.0f;
        for (int x = 0; x < bs; ++x)
            acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(U[i * bs + x], Dinv[x]), U[j * bs + x]));
        const float m0 = (i == j) ? __fadd_rn(1.0f, 1e-8f) : 0.0f;
        M[j * K + i] = __fadd_rn(m0, acc);
    }
    __syncthreads();
    if (t == 0) ldlt_inverse(M, K, Minv);
    __syncthreads();

    const float dt = own ? Dinv[t] : 0.0f;
    // H0[j][t] = D^-1 - D^-1 (sum_k1 sum_k2 Minv(k1,k2) u_k1 u_k2^T) D^-1 at
    // (row t, column j), k1 outer and k2 inner as the full inverse is summed.
    auto h0 = [&](int j) {
        float S = 0.0f;
        for (int k1 = 0; k1 < K; ++k1) {
            const float ui = U[k1 * bs + t];
            for (int k2 = 0; k2 < K; ++k2)
                S = __fadd_rn(S, __fmul_rn(Minv[k2 * K + k1], __fmul_rn(ui, U[k2 * bs + j])));
        }
        const float d0 = (j == t) ? dt : 0.0f;
        return __fsub_rn(d0, __fmul_rn(__fmul_rn(dt, S), Dinv[j]));
    };
    float my_d = own ? h0(t) : 0.0f;

    uint32_t done = 0;
    int par = 0;
    while (done < target) {
        // argmin_i w_i^2 / H_ii over H_ii > 0, first index on ties
        ObsCand c{FLT_MAX, 0x7FFFFFFF, 0.0f, 0.0f};
        if (own && my_d > 0.0f) {
            const float sc = __fdiv_rn(__fmul_rn(my_w, my_w), my_d);
            if (sc < c.v) c = ObsCand{sc, t, my_w, my_d};
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
            ObsCand o;
            o.v = __shfl_down_sync(0xFFFFFFFFu, c.v, off);
            o.i = __shfl_down_sync(0xFFFFFFFFu, c.i, off);
            o.w = __shfl_down_sync(0xFFFFFFFFu, c.w, off);
            o.h = __shfl_down_sync(0xFFFFFFFFu, c.h, off);
            cand_merge(c, o);
        }
        if ((t & 31) == 0) red[par][t >> 5] = c;
        __syncthreads();
        // every thread merges the warps' winners itself (the same total order),
        // so one barrier per step; red[] alternates so the next step's writes
        // never meet this step's reads
        ObsCand r = red[par][0];
        for (int q = 1; q < nt / 32; ++q) cand_merge(r, red[par][q]);
        par ^= 1;
        if (r.v >= FLT_MAX / 2) break;
        const int best = r.i;
        const float wi_old = r.w, hbb = r.h;
        if (own) {
            float x = h0(best);
            const float* cq = Cs;
#pragma unroll 4
            for (uint32_t q = 0; q < done; ++q, cq += bs)
                x = __fsub_rn(x, __fdiv_rn(__fmul_rn(cq[t], cq[best]), hs[q]));
            if (t != best) {
                const float inv_h = __fdiv_rn(1.0f, hbb);
                my_w = __fsub_rn(my_w, __fmul_rn(__fmul_rn(wi_old, inv_h), x));
            } else {
                my_w = 0.0f;
            }
            my_d = __fsub_rn(my_d, __fdiv_rn(__fmul_rn(x, x), hbb));
            Cs[done * bs + t] = x;
        }
        if (t == 0) hs[done] = hbb;
        ++done;
    }
    if (own) p.w[st + t] = my_w;
    if (t == 0) atomicAdd(p.pruned, static_cast<unsigned long long>(done));
}

// dynamic shared memory of block_obs_kernel for blocks of B rows, K snapshots
// and at most tcap pruned weights per block
constexpr size_t obs_smem_bytes(size_t B, size_t K, size_t tcap) {
    return sizeof(float) * (B * K + B + 2 * kMaxK * kMaxK + tcap + tcap * B);
}
static_assert(obs_smem_bytes(kMaxBlock, kMaxK, kMaxBlock - 1) <= 227 * 1024,
              "the largest block's downdate columns must fit in shared memory");

}  // namespace
}  // namespace tb

using namespace tb;

namespace tb {
namespace {
// Phase times of the calling thread's last tb_block_obs call (milliseconds):
// [0] block importance + its copy to the host, [1] host target allocation,
// [2] target/order upload and the greedy kernels, [3] the whole call.
thread_local float g_obs_phase_ms[4] = {0, 0, 0, 0};

struct PhaseEvents {
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    bool ok = false;
    PhaseEvents() {
        ok = true;
        for (auto& e : ev) ok = ok && cudaEventCreate(&e) == cudaSuccess;
    }
    ~PhaseEvents() {
        for (auto& e : ev)
            if (e) cudaEventDestroy(e);
    }
};
}  // namespace
}  // namespace tb

namespace tb {
namespace {
// Launch setup of block_obs_kernel: the kernel's shared-memory limit (one
// value per device, shared by every call) raised once to the largest any call
// can need, and per (device, block, snapshots) the CTAs per SM for every
// target 1..B-1, queried once - so a call makes no attribute or occupancy
// queries after the first of its shape.
struct OccKey {
    int dev, B, K;
    bool operator<(const OccKey& o) const { return std::tie(dev, B, K) < std::tie(o.dev, o.B, o.K); }
};
std::mutex g_occ_mu;
std::map<OccKey, std::vector<int>> g_occ;
std::vector<int> g_obs_smem_set;  // devices whose limit is raised

int obs_occupancy(int B, int K, unsigned threads, const std::vector<int>** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_occ_mu);
    if (std::find(g_obs_smem_set.begin(), g_obs_smem_set.end(), dev) == g_obs_smem_set.end()) {
        e = cudaFuncSetAttribute(block_obs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(obs_smem_bytes(kMaxBlock, kMaxK, kMaxBlock - 1)));
        if (e != cudaSuccess) return cuda_fail(e, "tb_block_obs setup");
        g_obs_smem_set.push_back(dev);
    }
    auto it = g_occ.find({dev, B, K});
    if (it == g_occ.end()) {
        const size_t tcap = B > 1 ? static_cast<size_t>(B - 1) : 0;
        std::vector<int> occ(static_cast<size_t>(B) + 1, 0);
        for (size_t t = 1; t <= tcap && e == cudaSuccess; ++t)
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ[t], block_obs_kernel, static_cast<int>(threads),
                                                              obs_smem_bytes(B, K, t));
        if (e != cudaSuccess) return cuda_fail(e, "tb_block_obs setup");
        it = g_occ.emplace(OccKey{dev, B, K}, std::move(occ)).first;
    }
    *out = &it->second;
    return TB_OK;
}
}  // namespace
}  // namespace tb

extern "C" int tb_block_obs_phase_times(float* ms_out, int n) {
    if (!ms_out || n < 1) return fail(TB_ERR_ARG, "tb_block_obs_phase_times: null or empty output");
    for (int i = 0; i < n && i < 4; ++i) ms_out[i] = g_obs_phase_ms[i];
    return TB_OK;
}

extern "C" int tb_block_obs(float* weights, const float* fisher, const float* const* hist, int K, size_t N,
                            size_t block, float sparsity, float damping, float off_diag_alpha, uint64_t* pruned_out,
                            void* stream) {
    if (N == 0) return fail(TB_ERR_ZERO_SIZE, "empty tensor");
    if (!weights) return fail(TB_ERR_ARG, "tb_block_obs: null weights");
    if (block == 0) return fail(TB_ERR_CONFIG, "obs_block_size 0");
    if (block > static_cast<size_t>(kMaxBlock))
        return fail(TB_ERR_UNSUPPORTED, "obs_block_size %zu > %d (B x B inverse must fit in shared memory)", block, kMaxBlock);
    if (K < 0 || K > kMaxK) return fail(TB_ERR_UNSUPPORTED, "gradient history of %d snapshots > %d", K, kMaxK);
    if (K > 0 && !hist) return fail(TB_ERR_ARG, "tb_block_obs: null history");
    if (!(sparsity >= 0.0f && sparsity <= 1.0f)) return fail(TB_ERR_CONFIG, "sparsity_ratio %g outside [0, 1]", sparsity);
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const size_t B = block;
    const size_t nb = (N + B - 1) / B;
    const size_t prune_total = N - static_cast<size_t>(sparsity * static_cast<float>(N));  // ehap.hpp:519
    if (prune_total == 0) {
        if (pruned_out) *pruned_out = 0;
        return TB_OK;
    }
    // Phase 1: block importance on the device.
    const auto t_call = std::chrono::steady_clock::now();
    PhaseEvents pe;
    if (pe.ok) cudaEventRecord(pe.ev[0], st);
    float* d_imp = nullptr;
    uint32_t* d_tgt = nullptr;
    unsigned long long* d_cnt = nullptr;
    // one scratch block: importances [nb] f32, targets then launch order
    // [2 nb] u32, the pruned counter (8-byte aligned)
    const size_t o_tgt = nb * sizeof(float), o_cnt = (o_tgt + 2 * nb * sizeof(uint32_t) + 7) / 8 * 8;
    char* scratch = nullptr;
    if ((rc = scratch_alloc(reinterpret_cast<void**>(&scratch), o_cnt + sizeof(unsigned long long), st))) return rc;
    d_imp = reinterpret_cast<float*>(scratch);
    d_tgt = reinterpret_cast<uint32_t*>(scratch + o_tgt);
    d_cnt = reinterpret_cast<unsigned long long*>(scratch + o_cnt);
    cudaError_t e = cudaSuccess;
    auto release = [&] { scratch_free(scratch, st); };
    block_importance_kernel<<<static_cast<unsigned>(std::min<size_t>((nb + 255) / 256, 148 * 16)), 256, 0, st>>>(
        weights, fisher, damping, N, static_cast<int>(B), nb, d_imp);
    std::vector<float> imp(nb);
    e = cudaMemcpyAsync(imp.data(), d_imp, nb * sizeof(float), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { release(); return cuda_fail(e, "tb_block_obs block importance"); }
    if (pe.ok) cudaEventRecord(pe.ev[1], st);
    const auto t_host = std::chrono::steady_clock::now();
    // Phase 2: targets (ehap.hpp:538-577), host scalars.
    float mx = 0.0f;
    for (float v : imp) if (v > mx) mx = v;
    if (mx <= 0.0f) mx = 1.0f;
    const float tau = 4.0f;
    std::vector<float> bw(nb);
    for (size_t b = 0; b < nb; ++b) {
        const float rel = imp[b] / mx;
        bw[b] = std::exp(-tau * rel);
    }
    float total_w = 0.0f;
    for (float v : bw) total_w += v;
    if (total_w <= 0.0f) total_w = 1.0f;
    std::vector<uint32_t> tgt(nb);
    std::vector<size_t> tg(nb);
    size_t allocated = 0;
    for (size_t b = 0; b < nb; ++b) {
        const float share = bw[b] / total_w;
        const size_t bs = (b == nb - 1) ? (N - b * B) : B;
        tg[b] = static_cast<size_t>(share * static_cast<float>(prune_total));
        if (tg[b] >= bs) tg[b] = bs > 1 ? bs - 1 : 0;
        allocated += tg[b];
    }
    std::ptrdiff_t rem = static_cast<std::ptrdiff_t>(prune_total) - static_cast<std::ptrdiff_t>(allocated);
    for (size_t b = 0; b < nb && rem > 0; ++b) {
        const size_t rb = nb - 1 - b;
        const size_t bs = (rb == nb - 1) ? (N - rb * B) : B;
        while (rem > 0 && tg[rb] + 1 < bs) { ++tg[rb]; --rem; }
    }
    for (size_t b = 0; b < nb; ++b) tgt[b] = static_cast<uint32_t>(tg[b]);
    // Phase 3: per-block greedy OBS.
    ObsParams p{};
    p.w = weights;
    p.F = fisher;
    p.K = K;
    for (int k = 0; k < K; ++k) {
        p.hist[k] = hist[k];
        const float age = static_cast<float>(K - 1 - k);
        p.wk[k] = std::exp(-age / 2.0f);  // ehap.hpp:606-607
    }
    p.sa = std::sqrt(off_diag_alpha);     // ehap.hpp:615
    p.damp = damping;
    p.N = N;
    p.B = static_cast<int>(B);
    p.targets = d_tgt;
    p.pruned = d_cnt;
    uint32_t tmax = 0;
    for (uint32_t x : tgt) tmax = std::max(tmax, x);
    const unsigned threads = static_cast<unsigned>((B + 31) / 32 * 32);
    // CTAs per SM for each target: the downdate columns in shared memory grow
    // with it, so blocks that prune fewer weights fit more CTAs on an SM
    const std::vector<int>* occp = nullptr;
    if ((rc = obs_occupancy(static_cast<int>(B), K ? K : 1, threads, &occp))) { release(); return rc; }
    const std::vector<int>& occ = *occp;
    // Within each slice of at most 2^30 blocks (block ids stay 32-bit), the
    // blocks run in descending order of target (counting sort, block id order
    // within a target; target-0 blocks are left out), one launch per run of
    // targets with the same CTAs per SM, each sized for its own largest target.
    struct Launch {
        size_t b0, first, count;
        uint32_t tcap;
    };
    std::vector<Launch> launches;
    std::vector<uint32_t> order(nb);
    const size_t slice = (size_t)1 << 30;
    for (size_t b0 = 0; b0 < nb; b0 += slice) {
        const size_t ns = std::min(slice, nb - b0);
        std::vector<size_t> start(tmax + 2, 0);  // start[t]: first position of target t
        for (size_t b = b0; b < b0 + ns; ++b) ++start[tgt[b]];
        size_t pos = 0;
        for (uint32_t t = tmax; t >= 1; --t) {
            const size_t c = start[t];
            start[t] = pos;
            pos += c;
        }
        const size_t nrun = pos;
        for (size_t b = b0; b < b0 + ns; ++b)
            if (tgt[b]) order[b0 + start[tgt[b]]++] = static_cast<uint32_t>(b - b0);
        size_t first = 0;
        for (uint32_t t = tmax; t >= 1 && first < nrun; --t) {
            const size_t c = (t == tmax ? start[t] : start[t] - start[t + 1]);
            if (c == 0) continue;
            if (!launches.empty() && launches.back().b0 == b0 && occ[launches.back().tcap] == occ[t]) {
                launches.back().count += c;
            } else {
                launches.push_back({b0, first, c, t});
            }
            first += c;
        }
    }
    const auto t_host_end = std::chrono::steady_clock::now();
    if (pe.ok) cudaEventRecord(pe.ev[2], st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_tgt, tgt.data(), nb * sizeof(uint32_t), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_tgt + nb, order.data(), nb * sizeof(uint32_t), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_cnt, 0, sizeof(unsigned long long), st);
    if (e != cudaSuccess) { release(); return cuda_fail(e, "tb_block_obs setup"); }
    for (const Launch& l : launches) {
        ObsParams q = p;
        q.w = p.w + l.b0 * B;
        if (p.F) q.F = p.F + l.b0 * B;
        for (int k = 0; k < K; ++k) q.hist[k] = p.hist[k] + l.b0 * B;
        q.N = N - l.b0 * B;
        q.targets = p.targets + l.b0;
        q.order = d_tgt + nb + l.b0 + l.first;
        q.tcap = static_cast<int>(l.tcap);
        block_obs_kernel<<<static_cast<unsigned>(l.count), threads, obs_smem_bytes(B, K ? K : 1, l.tcap), st>>>(q);
    }
    if ((rc = check_launch("block_obs_kernel"))) { release(); return rc; }
    if (pe.ok) cudaEventRecord(pe.ev[3], st);
    unsigned long long cnt = 0;
    e = cudaMemcpyAsync(&cnt, d_cnt, sizeof(cnt), cudaMemcpyDeviceToHost, st);
    release();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "tb_block_obs result");
    if (pruned_out) *pruned_out = cnt;
    using ms = std::chrono::duration<float, std::milli>;
    g_obs_phase_ms[1] = ms(t_host_end - t_host).count();
    g_obs_phase_ms[3] = ms(std::chrono::steady_clock::now() - t_call).count();
    if (pe.ok) {
        cudaEventElapsedTime(&g_obs_phase_ms[0], pe.ev[0], pe.ev[1]);
        cudaEventElapsedTime(&g_obs_phase_ms[2], pe.ev[2], pe.ev[3]);
    }
    return TB_OK;
}

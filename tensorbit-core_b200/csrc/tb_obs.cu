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
// Phase 3 (device, one CTA per block): D^-1, U (K gradient snapshots or
//   sqrt(alpha) w), M = I + U^T D^-1 U, M^-1 by pivoted LDL^T, the full B x B
//   H^-1 = D^-1 - D^-1 (sum Minv_kl u_k u_l^T) D^-1 in shared memory, then the
//   greedy loop: argmin w_i^2 / H^-1_ii (lowest index on ties), OBS update of
//   the other weights, rank-1 Sherman-Morrison deflation of H^-1
//   (ehap.hpp:582-701).
//
// Every float operation keeps the reference's expression tree (products
// accumulated over the inner index in order from zero, no fused multiply-add);
// the K x K factorisation follows the pivoted LDL^T the reference oracle is
// built with.  The loop is latency-bound CUDA-core work (B^2 divisions per
// pruned weight); there is no tensor-core formulation of its serial greedy.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <vector>

#include "tb_device.cuh"
#include "tb_runtime.h"

namespace tb {
namespace {

constexpr int kMaxK = 16;
constexpr int kObsThreads = 256;
constexpr int kMaxBlock = 224;  // B x B floats must fit in shared memory
constexpr int kLazyChunk = 16;  // earlier downdates whose terms one pass of the lazy row computes

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
    unsigned long long* pruned;
    int tcap;        // the largest target: rows of the kept downdate columns (lazy form)
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

// argmin over (value, index): smaller value wins, equal values -> lower index.
__device__ __forceinline__ void argmin_merge(float& v, int& i, float v2, int i2) {
    if (v2 < v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

// LAZY: H stays the initial inverse H0; the greedy loop keeps only its diagonal
// and the downdate columns c_s, h_s, and forms the one row it needs each step,
// H0[best][j] minus the block's earlier downdates c_s[j] c_s[best] / h_s in
// step order -- the same operations, in the same order, as the element of the
// updated H would have seen, so the results are the same bits, with ~1/4 of
// the correctly rounded divisions (those dominate a step).
template <bool LAZY>
__global__ void __launch_bounds__(kObsThreads) block_obs_kernel(const ObsParams p) {
    extern __shared__ float smem[];
    const size_t b = blockIdx.x;
    const size_t st = b * p.B;
    const int bs = static_cast<int>((st + p.B < p.N ? st + p.B : p.N) - st);
    const uint32_t target = p.targets[b];
    if (target == 0 || target >= static_cast<uint32_t>(bs)) return;
    const int K = p.K ? p.K : 1;
    float* H = smem;                      // bs*bs, column-major
    float* U = H + bs * bs;               // bs*K, column-major
    float* Dinv = U + bs * K;             // bs
    float* wv = Dinv + bs;                // bs
    float* col = wv + bs;                 // bs
    float* M = col + bs;                  // K*K
    float* Minv = M + kMaxK * kMaxK;      // K*K
    __shared__ float red_v[kObsThreads / 32];
    __shared__ int red_i[kObsThreads / 32];
    __shared__ float s_min;
    __shared__ int s_best;
    const int t = threadIdx.x;

    for (int i = t; i < bs; i += kObsThreads) {
        const float d = p.F ? __fadd_rn(p.damp, p.F[st + i]) : p.damp;
        Dinv[i] = d > 0.0f ? __fdiv_rn(1.0f, d) : 1.0f;
        const float wi = p.w[st + i];
        wv[i] = wi;
        if (p.K) {
            for (int k = 0; k < K; ++k) U[k * bs + i] = __fmul_rn(p.wk[k], p.hist[k][st + i]);
        } else {
            U[i] = __fmul_rn(p.sa, wi);
        }
    }
    __syncthreads();
    // M = I + 1e-8 I + (U^T D^-1) U: one thread per entry, inner index in order.
    if (t < K * K) {
        const int i = t % K, j = t / K;
        float acc = 0.0f;
        for (int x = 0; x < bs; ++x)
            acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(U[i * bs + x], Dinv[x]), U[j * bs + x]));
        const float m0 = (i == j) ? __fadd_rn(1.0f, 1e-8f) : 0.0f;
        M[j * K + i] = __fadd_rn(m0, acc);
    }
    __syncthreads();
    if (t == 0) ldlt_inverse(M, K, Minv);
    __syncthreads();
    // H^-1 = D^-1 - D^-1 S D^-1 with S = sum_k1 sum_k2 Minv(k1,k2) u_k1 u_k2^T.
    for (int e = t; e < bs * bs; e += kObsThreads) {
        const int i = e % bs, j = e / bs;
        float S = 0.0f;
        for (int k1 = 0; k1 < K; ++k1)
            for (int k2 = 0; k2 < K; ++k2)
                S = __fadd_rn(S, __fmul_rn(Minv[k2 * K + k1], __fmul_rn(U[k1 * bs + i], U[k2 * bs + j])));
        const float h0 = (i == j) ? Dinv[i] : 0.0f;
        H[e] = __fsub_rn(h0, __fmul_rn(__fmul_rn(Dinv[i], S), Dinv[j]));
    }
    __syncthreads();

    // the rank-1 updates: ung column sets of bs rows each, row ui of set ug
    const int ung = kObsThreads / bs > 0 ? kObsThreads / bs : 1;
    const int ui = (t < ung * bs) ? t % bs : -1, ug = (t < ung * bs) ? t / bs : 0;
    // (bs <= kMaxBlock < kObsThreads, so every row has a thread)
    float* diag = Minv + kMaxK * kMaxK;  // LAZY: the current diagonal of H
    float* Cs = diag + bs;               // LAZY: tcap x bs downdate columns
    float* hs = Cs + p.tcap * bs;        // LAZY: their pivots
    float* terms = hs + p.tcap;          // LAZY: kLazyChunk x bs downdate terms of one row
    if constexpr (LAZY) {
        for (int i = t; i < bs; i += kObsThreads) diag[i] = H[i * bs + i];
        __syncthreads();
    }
    uint32_t done = 0;
    while (done < target) {
        // argmin_i w_i^2 / H_ii over H_ii > 0, first index on ties
        float v = FLT_MAX;
        int bi = 0x7FFFFFFF;
        for (int i = t; i < bs; i += kObsThreads) {
            const float hii = LAZY ? diag[i] : H[i * bs + i];
            if (hii <= 0.0f) continue;
            const float sc = __fdiv_rn(__fmul_rn(wv[i], wv[i]), hii);
            if (sc < v) { v = sc; bi = i; }   // ascending i per thread: first wins
        }
        for (int off = 16; off; off >>= 1) {
            const float v2 = __shfl_down_sync(0xFFFFFFFFu, v, off);
            const int i2 = __shfl_down_sync(0xFFFFFFFFu, bi, off);
            argmin_merge(v, bi, v2, i2);
        }
        if ((t & 31) == 0) { red_v[t >> 5] = v; red_i[t >> 5] = bi; }
        __syncthreads();
        if (t == 0) {
            float vv = red_v[0];
            int ii = red_i[0];
            for (int q = 1; q < kObsThreads / 32; ++q) argmin_merge(vv, ii, red_v[q], red_i[q]);
            s_min = vv;
            s_best = ii;
        }
        __syncthreads();
        if (s_min >= FLT_MAX / 2) break;
        const int best = s_best;
        const float hbb = LAZY ? diag[best] : H[best * bs + best];
        const float wi_old = wv[best];
        const float inv_h = __fdiv_rn(1.0f, hbb);
        if constexpr (LAZY) {
            // The terms of up to kLazyChunk earlier steps at once on every thread,
            // then each row element subtracts them in step order.
            float x = (t < bs) ? H[best * bs + t] : 0.0f;
            for (uint32_t q0 = 0; q0 < done; q0 += kLazyChunk) {
                const int nq = static_cast<int>(min(static_cast<uint32_t>(kLazyChunk), done - q0));
                if (ui >= 0)
                    for (int q = ug; q < nq; q += ung) {
                        const float* cq = Cs + (q0 + q) * bs;
                        terms[q * bs + ui] = __fdiv_rn(__fmul_rn(cq[ui], cq[best]), hs[q0 + q]);
                    }
                __syncthreads();
                if (t < bs)
                    for (int q = 0; q < nq; ++q) x = __fsub_rn(x, terms[q * bs + t]);
                __syncthreads();
            }
            if (t < bs) col[t] = x;
            __syncthreads();
            for (int j = t; j < bs; j += kObsThreads) {
                const float cj = col[j];
                if (j != best) wv[j] = __fsub_rn(wv[j], __fmul_rn(__fmul_rn(wi_old, inv_h), cj));
                diag[j] = __fsub_rn(diag[j], __fdiv_rn(__fmul_rn(cj, cj), hbb));
                Cs[done * bs + j] = cj;
            }
            if (t == 0) {
                wv[best] = 0.0f;
                hs[done] = hbb;
            }
            __syncthreads();
            ++done;
            continue;
        }
        for (int j = t; j < bs; j += kObsThreads) {
            col[j] = H[best * bs + j];
            if (j != best) wv[j] = __fsub_rn(wv[j], __fmul_rn(__fmul_rn(wi_old, inv_h), H[best * bs + j]));
        }
        __syncthreads();
        if (t == 0) wv[best] = 0.0f;
        // H -= col col^T / h_bb: thread (row ui, column set ug) walks its columns
        if (ui >= 0) {
            const float ci = col[ui];
            for (int j = ug; j < bs; j += ung) {
                float* h = H + j * bs + ui;
                *h = __fsub_rn(*h, __fdiv_rn(__fmul_rn(ci, col[j]), hbb));
            }
        }
        __syncthreads();
        ++done;
    }
    for (int i = t; i < bs; i += kObsThreads) p.w[st + i] = wv[i];
    if (t == 0) atomicAdd(p.pruned, static_cast<unsigned long long>(done));
}

size_t obs_smem_bytes(int B, int K) {
    return sizeof(float) * (static_cast<size_t>(B) * B + static_cast<size_t>(B) * K + 3 * B + 2 * kMaxK * kMaxK);
}

}  // namespace
}  // namespace tb

using namespace tb;

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
    float* d_imp = nullptr;
    uint32_t* d_tgt = nullptr;
    unsigned long long* d_cnt = nullptr;
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d_imp), nb * sizeof(float), st);
    if (e == cudaSuccess) e = cudaMallocAsync(reinterpret_cast<void**>(&d_tgt), nb * sizeof(uint32_t), st);
    if (e == cudaSuccess) e = cudaMallocAsync(reinterpret_cast<void**>(&d_cnt), sizeof(unsigned long long), st);
    if (e != cudaSuccess) return cuda_fail(e, "tb_block_obs scratch");
    auto release = [&] {
        cudaFreeAsync(d_imp, st);
        cudaFreeAsync(d_tgt, st);
        cudaFreeAsync(d_cnt, st);
    };
    block_importance_kernel<<<static_cast<unsigned>(std::min<size_t>((nb + 255) / 256, 148 * 16)), 256, 0, st>>>(
        weights, fisher, damping, N, static_cast<int>(B), nb, d_imp);
    std::vector<float> imp(nb);
    e = cudaMemcpyAsync(imp.data(), d_imp, nb * sizeof(float), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) { release(); return cuda_fail(e, "tb_block_obs block importance"); }
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
    // the lazy form where its downdate columns fit in shared memory beside H0
    const size_t smem_eager = obs_smem_bytes(static_cast<int>(B), K ? K : 1);
    const size_t smem_lazy =
        smem_eager + sizeof(float) * (B + static_cast<size_t>(tmax) * B + tmax + static_cast<size_t>(kLazyChunk) * B);
    const bool lazy = smem_lazy <= 227 * 1024;
    const size_t smem = lazy ? smem_lazy : smem_eager;
    p.tcap = static_cast<int>(tmax);
    e = lazy ? cudaFuncSetAttribute(block_obs_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem))
             : cudaFuncSetAttribute(block_obs_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem));
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_tgt, tgt.data(), nb * sizeof(uint32_t), cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_cnt, 0, sizeof(unsigned long long), st);
    if (e != cudaSuccess) { release(); return cuda_fail(e, "tb_block_obs setup"); }
    // Blocks beyond 2^31-1 are launched in slices.
    const size_t slice = (size_t)1 << 30;
    for (size_t b0 = 0; b0 < nb; b0 += slice) {
        ObsParams q = p;
        const size_t nslice = std::min(slice, nb - b0);
        q.w = p.w + b0 * B;
        if (p.F) q.F = p.F + b0 * B;
        for (int k = 0; k < K; ++k) q.hist[k] = p.hist[k] + b0 * B;
        q.N = N - b0 * B;
        q.targets = p.targets + b0;
        if (lazy)
            block_obs_kernel<true><<<static_cast<unsigned>(nslice), kObsThreads, smem, st>>>(q);
        else
            block_obs_kernel<false><<<static_cast<unsigned>(nslice), kObsThreads, smem, st>>>(q);
    }
    if ((rc = check_launch("block_obs_kernel"))) { release(); return rc; }
    unsigned long long cnt = 0;
    e = cudaMemcpyAsync(&cnt, d_cnt, sizeof(cnt), cudaMemcpyDeviceToHost, st);
    release();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "tb_block_obs result");
    if (pruned_out) *pruned_out = cnt;
    return TB_OK;
}

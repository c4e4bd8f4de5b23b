// Fused score -> N:M mask -> pack pass (stages 1 and 2 of the pruning path).
//
// One read of W, the S gradient samples and (optionally) the prior Fisher
// state; one write of the FP32 pruned weights and the packed mask bytes - the
// .tb weight and mask sections (serialization.hpp:101-151).  Per element it
// runs the reference's EMA recurrence over the samples in registers
// (ehap.hpp:186-200), scores it (ehap.hpp:256-284), and per group selects,
// applies and redistributes exactly as CORINGPruner::prune (coring.hpp:299-313).
//
// Layout in HBM: W [N] (FP32/BF16/F16), G [S][g_stride] sample-major, outputs
// W' [N] FP32 and mask [N/M] u8.  Each thread owns 16 consecutive elements:
// per sample a warp reads 32 x 32 B (BF16) contiguous with 16-byte
// non-L1-allocating loads, so a CTA streams all samples of its 4096-element
// column slab with every load independent of the FP chain.  The pass is
// HBM-bound (about 2S+6 bytes per parameter against ~3 FP ops per
// parameter-sample).
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <vector>

#include "tb_device.cuh"
#include "tb_runtime.h"
#include "tb_threshold.h"

namespace tb {
namespace {

constexpr int kThreads = 256;
constexpr int kEpt = 16;  // elements per thread in the vector kernel
// Gradient samples of a 16-bit type whose loads a thread keeps in flight in
// the vector kernel (two 16-byte loads each), and the CTAs per SM its register
// budget is set for.  Measured on B200 against 4 and 3 (80 registers): 8 in
// flight at 2 CTAs (94 registers) and 4 or 2 at 4 CTAs (64 registers, with
// spills) were 2-11 % slower on the 7B pass and the 70B sweep.
#ifndef TB_SAMPLES_IN_FLIGHT
#define TB_SAMPLES_IN_FLIGHT 4
#endif
#ifndef TB_VEC_MIN_CTAS
#define TB_VEC_MIN_CTAS (TB_SAMPLES_IN_FLIGHT > 4 ? 2 : 3)
#endif
constexpr int kU16 = TB_SAMPLES_IN_FLIGHT;
constexpr int kVecMinCtas = TB_VEC_MIN_CTAS;
constexpr int kMaxParts = 8;  // partial Fisher sums of a sample-split pass (ranks of one node)

// Variants of the pass (template argument of the vector kernel, p.variant in
// the scalar one).
constexpr int kVarPlain = 0;      // score -> mask -> pack
constexpr int kVarPeer = 1;       // Fisher state = sum of peer partials (sample split)
constexpr int kVarScores = 2;     // Fisher and importance only: writes fout / sout, no mask
constexpr int kVarThreshold = 3;  // EHAP one-shot keep (s >= *thr) before CORING (tb-prune sequence)

struct FusedParams {
    const void* w;
    const void* g;
    const float* fin;
    float* wout;
    uint8_t* mout;
    float* fout;
    float* sout;
    unsigned long long* ties;
    const uint8_t* lut;
    size_t N;        // elements in this launch
    size_t S;        // samples actually read (0 when the Fisher is off)
    size_t gstride;  // elements between samples
    float alpha, beta, contrib, damp;
    int mode;
    int have_f;      // a Fisher state exists after this pass
    int first;       // sample 0 initialises F (no prior state)
    int use_fin;     // F starts from fin
    int n, strategy, rounds, redist, permute;
    int wdt, gdt;    // dtypes (generic kernel)
    int nparts;      // > 0: F starts as the sum of parts[0..nparts) (sample split)
    const float* parts[kMaxParts];
    int variant;     // kVar*
    const float* thr;              // kVarThreshold: device address of the EHAP threshold
    unsigned long long* thr_pruned;  // kVarThreshold: counter of weights the threshold zeroes
    int prefetch;    // vector kernel: batches of samples prefetched into L2 ahead of the loads (0: none)
};

// --- 16-element vector loads --------------------------------------------------
template <int DT> struct Vec16;
template <> struct Vec16<TB_F32> {
    static constexpr int kWords = 4;  // uint4 per 16 elements
    __device__ static void decode(const uint4 (&b)[kWords], float (&x)[kEpt]) {
#pragma unroll
        for (int k = 0; k < kWords; ++k) {
            x[4 * k + 0] = __uint_as_float(b[k].x);
            x[4 * k + 1] = __uint_as_float(b[k].y);
            x[4 * k + 2] = __uint_as_float(b[k].z);
            x[4 * k + 3] = __uint_as_float(b[k].w);
        }
    }
};
template <> struct Vec16<TB_BF16> {
    static constexpr int kWords = 2;
    __device__ static void decode(const uint4 (&b)[kWords], float (&x)[kEpt]) {
#pragma unroll
        for (int k = 0; k < kWords; ++k) {
            const uint32_t u[4] = {b[k].x, b[k].y, b[k].z, b[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                x[8 * k + 2 * j + 0] = __uint_as_float(u[j] << 16);
                x[8 * k + 2 * j + 1] = __uint_as_float(u[j] & 0xFFFF0000u);
            }
        }
    }
};
template <> struct Vec16<TB_F16> {
    static constexpr int kWords = 2;
    __device__ static void decode(const uint4 (&b)[kWords], float (&x)[kEpt]) {
#pragma unroll
        for (int k = 0; k < kWords; ++k) {
            const uint32_t u[4] = {b[k].x, b[k].y, b[k].z, b[k].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                x[8 * k + 2 * j + 0] = f16ref_to_f32(u[j] & 0xFFFFu);
                x[8 * k + 2 * j + 1] = f16ref_to_f32(u[j] >> 16);
            }
        }
    }
};

template <int DT>
__device__ __forceinline__ void load16(const void* base, size_t e0, float (&x)[kEpt]) {
    constexpr int W = Vec16<DT>::kWords;
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const char*>(base) + e0 * Dtype<DT>::kBytes);
    uint4 b[W];
#pragma unroll
    for (int k = 0; k < W; ++k) b[k] = ldg_stream(p + k);
    Vec16<DT>::decode(b, x);
}

__device__ __forceinline__ void store16(float* base, size_t e0, const float (&x)[kEpt]) {
    float4* p = reinterpret_cast<float4*>(base + e0);
#pragma unroll
    for (int k = 0; k < 4; ++k) stg_stream(p + k, make_float4(x[4 * k], x[4 * k + 1], x[4 * k + 2], x[4 * k + 3]));
}

// 16 FP32 values of one partial Fisher sum, which may live in a peer GPU's
// memory: coherent streaming loads (ld.global.cs), not the read-only path.
__device__ __forceinline__ void load16_part(const float* base, size_t e0, float (&x)[kEpt]) {
    const float4* q = reinterpret_cast<const float4*>(base + e0);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float4 v = __ldcs(q + k);
        x[4 * k + 0] = v.x;
        x[4 * k + 1] = v.y;
        x[4 * k + 2] = v.z;
        x[4 * k + 3] = v.w;
    }
}

// Adds the active lanes' counts to a device counter with one atomic per warp.
__device__ __forceinline__ void warp_add_count(unsigned long long* counter, int local) {
    const unsigned active = __activemask();
    const int total = __reduce_add_sync(active, local);
    if (total && (threadIdx.x & 31) == (__ffs(active) - 1))
        atomicAdd(counter, static_cast<unsigned long long>(total));
}

// Stage 2 on one thread's 16 scores: select, apply, redistribute; returns the
// packed mask bytes (group k in byte k).
template <int M>
__device__ __forceinline__ uint64_t groups16(const FusedParams& p, const float (&s)[kEpt], float (&w)[kEpt],
                                             int& ties) {
    uint64_t packed = 0;
#pragma unroll
    for (int q = 0; q < kEpt / M; ++q) {
        float v[M], sg[M], wg[M];
#pragma unroll
        for (int k = 0; k < M; ++k) { v[k] = s[q * M + k]; sg[k] = v[k]; }
        if (p.ties) ties += near_tie<M>(v, p.n) ? 1 : 0;
        const uint32_t byte = select_group<M>(v, p.n, p.strategy, p.rounds, p.permute != 0, p.lut);
#pragma unroll
        for (int k = 0; k < M; ++k) wg[k] = ((byte >> k) & 1u) ? w[q * M + k] : 0.0f;
        redistribute_group<M>(wg, sg, byte, p.redist);
#pragma unroll
        for (int k = 0; k < M; ++k) w[q * M + k] = wg[k];
        packed |= static_cast<uint64_t>(byte & 0xFFu) << (8 * q);
    }
    return packed;
}

// Vector kernel: 16 elements per thread, all pointers 16-byte aligned and
// g_stride * sizeof(G) a multiple of 16 (checked on the host).  Three 256-thread
// CTAs per SM (<= 85 registers) keep more loads in flight than two.  The
// sample recurrence issues its products as packed f32x2 (ema_next2, exact);
// at the power-capped clock the pass is partly issue-bound, so fewer FP32
// instructions per element show up as bandwidth.
//
// VAR selects a variant (kVar*); the plain instantiations compile without the
// other variants' code.  kVarPeer: the Fisher state starts as the sum of the
// p.nparts partial sums of a sample-split pass (tb_score_mask_pack_peer).
// kVarScores: stage 1 and the importance only.  kVarThreshold: the EHAP
// one-shot keep rule s >= threshold zeroes weights before the importance that
// CORING ranks is recomputed (tb_prune_one_shot_nm).
template <int WDT, int GDT, int M, int VAR>
__global__ void __launch_bounds__(kThreads, kVecMinCtas) fused_vec_kernel(const FusedParams p) {
    constexpr int GW = Vec16<GDT>::kWords;
    constexpr int U = (GW == 2) ? kU16 : 2;  // samples in flight per thread
    const uint64_t beta2 = pack2(p.beta, p.beta), c2 = pack2(p.contrib, p.contrib);
    const size_t nchunks = p.N / kEpt;
    const size_t gstride_b = p.gstride * Dtype<GDT>::kBytes;
    int ties = 0;
    int zeroed = 0;  // kVarThreshold
    for (size_t c = blockIdx.x * (size_t)kThreads + threadIdx.x; c < nchunks; c += (size_t)gridDim.x * kThreads) {
        const size_t e0 = c * kEpt;
        float F[kEpt];
        // ---- stage 1: Fisher EMA over the samples, in registers ----
        const char* gb = static_cast<const char*>(p.g) + e0 * Dtype<GDT>::kBytes;
        size_t s = 0;
        const char* wb = static_cast<const char*>(p.w) + e0 * Dtype<WDT>::kBytes;
        const size_t ahead = static_cast<size_t>(p.prefetch) * U;  // samples prefetched ahead
        if (ahead) {
            // Each thread prefetches its own bytes (a warp's prefetches cover
            // its rows): here the batches after the first, up to `ahead`
            // samples, and the weights if that window reaches the last sample;
            // the batch loop keeps the window `ahead` samples in front.
            const size_t s1 = (p.first && p.S > 0) ? 1 : 0;
            for (size_t t = s1 + U; t < s1 + ahead && t < p.S; ++t) prefetch_l2(gb + t * gstride_b);
            if (s1 + ahead >= p.S) prefetch_l2(wb);
        }
        if (p.first && p.S > 0) {
            uint4 b[GW];
#pragma unroll
            for (int k = 0; k < GW; ++k) b[k] = ldg_stream(reinterpret_cast<const uint4*>(gb) + k);
            float x[kEpt];
            Vec16<GDT>::decode(b, x);
#pragma unroll
            for (int i = 0; i < kEpt; ++i) F[i] = ema_first(p.alpha, x[i]);
            s = 1;
        } else if (VAR == kVarPeer) {
            load16_part(p.parts[0], e0, F);
            for (int k = 1; k < p.nparts; ++k) {
                float x[kEpt];
                load16_part(p.parts[k], e0, x);
#pragma unroll
                for (int i = 0; i < kEpt; ++i) F[i] = __fadd_rn(F[i], x[i]);
            }
        } else if (p.use_fin) {
            load16<TB_F32>(p.fin, e0, F);
        } else {
#pragma unroll
            for (int i = 0; i < kEpt; ++i) F[i] = 0.0f;
        }
        for (; s + U <= p.S; s += U) {
            uint4 b[U][GW];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int k = 0; k < GW; ++k)
                    b[u][k] = ldg_stream(reinterpret_cast<const uint4*>(gb + (s + u) * gstride_b) + k);
            if (ahead) {
                const size_t t0 = s + ahead;
                if (t0 < p.S) {
#pragma unroll
                    for (int u = 0; u < U; ++u)
                        if (t0 + u < p.S) prefetch_l2(gb + (t0 + u) * gstride_b);
                    if (t0 + U >= p.S) prefetch_l2(wb);
                }
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float x[kEpt];
                Vec16<GDT>::decode(b[u], x);
#pragma unroll
                for (int i = 0; i < kEpt; i += 2) ema_next2(F[i], F[i + 1], beta2, c2, x[i], x[i + 1]);
            }
        }
        for (; s < p.S; ++s) {
            uint4 b[GW];
#pragma unroll
            for (int k = 0; k < GW; ++k) b[k] = ldg_stream(reinterpret_cast<const uint4*>(gb + s * gstride_b) + k);
            float x[kEpt];
            Vec16<GDT>::decode(b, x);
#pragma unroll
            for (int i = 0; i < kEpt; i += 2) ema_next2(F[i], F[i + 1], beta2, c2, x[i], x[i + 1]);
        }
        // ---- importance ----
        float w[kEpt], sc[kEpt];
        load16<WDT>(wb, 0, w);
        const bool have_f = p.have_f != 0;
        if (VAR == kVarScores) {
#pragma unroll
            for (int i = 0; i < kEpt; ++i) sc[i] = importance(w[i], F[i], p.damp, p.mode, have_f);
            if (p.fout && have_f) store16(p.fout, e0, F);
            store16(p.sout, e0, sc);
            continue;
        }
        if (VAR == kVarThreshold) {
            // select_pruning_mask + apply_mask (ehap.hpp:313-362): keep where
            // s >= threshold, others become +0 (NaN scores are not kept).
            const float thr = *p.thr;
#pragma unroll
            for (int i = 0; i < kEpt; ++i) {
                const bool keep = importance(w[i], F[i], p.damp, p.mode, have_f) >= thr;
                w[i] = keep ? w[i] : 0.0f;
                zeroed += keep ? 0 : 1;
            }
        }
#pragma unroll
        for (int i = 0; i < kEpt; ++i) sc[i] = importance(w[i], F[i], p.damp, p.mode, have_f);
        // ---- stage 2: select, apply, redistribute, pack ----
        const uint64_t packed = groups16<M>(p, sc, w, ties);
        store16(p.wout, e0, w);
        constexpr int kMaskBytes = kEpt / M;
        if (kMaskBytes == 8) *reinterpret_cast<uint64_t*>(p.mout + c * 8) = packed;
        else if (kMaskBytes == 4) *reinterpret_cast<uint32_t*>(p.mout + c * 4) = static_cast<uint32_t>(packed);
        else *reinterpret_cast<uint16_t*>(p.mout + c * 2) = static_cast<uint16_t>(packed);
        if (p.fout && have_f) store16(p.fout, e0, F);
        if (p.sout) store16(p.sout, e0, sc);
    }
    if (p.ties) warp_add_count(p.ties, ties);
    if (VAR == kVarThreshold) warp_add_count(p.thr_pruned, zeroed);
}

// ---- sample split: partial Fisher sums pushed to the ranks that own them ------
constexpr int kMaxScatterRanks = 8;
constexpr int kMaxPartialSamples = 128;

struct PartialSpec {
    const void* g;
    size_t S, gstride, N;
    float c[kMaxPartialSamples];           // per-sample weights of the regrouped EMA
    int nranks;
    size_t start[kMaxScatterRanks + 1];    // owner r holds elements [start[r], start[r + 1])
    float* dest[kMaxScatterRanks];         // element start[r] of this partial lands at dest[r][0]
    size_t rot;                            // vector chunks are visited from chunk `rot` on, cyclically
};

__device__ __forceinline__ int owner_of(const PartialSpec& q, size_t e) {
    int r = 0;
    for (int k = 1; k < q.nranks; ++k) r += (e >= q.start[k]) ? 1 : 0;
    return r;
}

// a += (c * x) * x for two lanes, the two products packed (mul.rn.f32x2,
// exact) and the sums scalar round-to-nearest, as ema_next2 does.
__device__ __forceinline__ void wsum_next2(float& a0, float& a1, uint64_t c2, float x0, float x1) {
    float t0, t1;
    asm("{\n\t.reg .b64 G, T;\n\t"
        "mov.b64 G, {%2, %3};\n\t"
        "mul.rn.f32x2 T, %4, G;\n\tmul.rn.f32x2 T, T, G;\n\t"
        "mov.b64 {%0, %1}, T;\n\t}"
        : "=f"(t0), "=f"(t1)
        : "f"(x0), "f"(x1), "l"(c2));
    a0 = __fadd_rn(a0, t0);
    a1 = __fadd_rn(a1, t1);
}

// 16 consecutive elements per thread, U samples' loads in flight as in the
// fused vector kernel: sum_t c_t g_t^2 per element in registers (from +0,
// samples in order: the arithmetic of tb_fisher_weighted_sum, bit for bit),
// each 8-element half stored to its owner (a peer's memory over NVLink, or
// this GPU's own).  Range starts are multiples of 8, so no half straddles two
// owners.  Requires 16-byte aligned gradients, rows and destinations.
template <int GDT>
__global__ void __launch_bounds__(kThreads, 3) partial_vec_kernel(const PartialSpec q) {
    constexpr int GW = Vec16<GDT>::kWords;
    constexpr int U = (GW == 2) ? 4 : 2;
    const size_t nchunks = q.N / kEpt;
    const size_t gstride_b = q.gstride * Dtype<GDT>::kBytes;
    for (size_t i = blockIdx.x * (size_t)kThreads + threadIdx.x; i < nchunks; i += (size_t)gridDim.x * kThreads) {
        // Ranks start at different owners' ranges, so that their remote
        // stores do not all converge on one peer's links at a time.
        const size_t c = i + q.rot < nchunks ? i + q.rot : i + q.rot - nchunks;
        const size_t e0 = c * kEpt;
        float acc[kEpt];
#pragma unroll
        for (int i = 0; i < kEpt; ++i) acc[i] = 0.0f;
        const char* gb = static_cast<const char*>(q.g) + e0 * Dtype<GDT>::kBytes;
        size_t s = 0;
        for (; s + U <= q.S; s += U) {
            uint4 b[U][GW];
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int k = 0; k < GW; ++k)
                    b[u][k] = ldg_stream(reinterpret_cast<const uint4*>(gb + (s + u) * gstride_b) + k);
#pragma unroll
            for (int u = 0; u < U; ++u) {
                float x[kEpt];
                Vec16<GDT>::decode(b[u], x);
                const uint64_t c2 = pack2(q.c[s + u], q.c[s + u]);
#pragma unroll
                for (int i = 0; i < kEpt; i += 2) wsum_next2(acc[i], acc[i + 1], c2, x[i], x[i + 1]);
            }
        }
        for (; s < q.S; ++s) {
            uint4 b[GW];
#pragma unroll
            for (int k = 0; k < GW; ++k) b[k] = ldg_stream(reinterpret_cast<const uint4*>(gb + s * gstride_b) + k);
            float x[kEpt];
            Vec16<GDT>::decode(b, x);
            const uint64_t c2 = pack2(q.c[s], q.c[s]);
#pragma unroll
            for (int i = 0; i < kEpt; i += 2) wsum_next2(acc[i], acc[i + 1], c2, x[i], x[i + 1]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const size_t e = e0 + 8 * h;
            const int r = owner_of(q, e);
            float4* d = reinterpret_cast<float4*>(q.dest[r] + (e - q.start[r]));
            __stcs(d, make_float4(acc[8 * h], acc[8 * h + 1], acc[8 * h + 2], acc[8 * h + 3]));
            __stcs(d + 1, make_float4(acc[8 * h + 4], acc[8 * h + 5], acc[8 * h + 6], acc[8 * h + 7]));
        }
    }
    // The pushed partials are visible to their owners once the kernel ends: the
    // CTA's stores are collected by the barrier and one system-scope fence
    // (cumulative) per CTA, not one per thread waiting on its remote stores.
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// Elements [e_begin, N) one per thread: any alignment, and the vector
// kernel's ragged tail.
__global__ void __launch_bounds__(kThreads) partial_scalar_kernel(const PartialSpec q, int gdt, size_t e_begin) {
    for (size_t i = e_begin + blockIdx.x * (size_t)kThreads + threadIdx.x; i < q.N; i += (size_t)gridDim.x * kThreads) {
        float acc = 0.0f;
        for (size_t s = 0; s < q.S; ++s) {
            const float x = load_any(q.g, gdt, s * q.gstride + i);
            acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(q.c[s], x), x));
        }
        const int r = owner_of(q, i);
        q.dest[r][i - q.start[r]] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
}

// Generic kernel: one group of M elements per thread, scalar loads; covers any
// alignment, M in [2, 8], and the tail of the vector kernel.
template <int M>
__global__ void __launch_bounds__(kThreads) fused_group_kernel(const FusedParams p) {
    const size_t G = p.N / M;
    int ties = 0;
    int zeroed = 0;
    for (size_t g = blockIdx.x * (size_t)kThreads + threadIdx.x; g < G; g += (size_t)gridDim.x * kThreads) {
        const size_t e0 = g * M;
        float F[M], w[M], sc[M], v[M];
#pragma unroll
        for (int k = 0; k < M; ++k) {
            const size_t e = e0 + k;
            float f = 0.0f;
            size_t s = 0;
            if (p.first && p.S > 0) { f = ema_first(p.alpha, load_any(p.g, p.gdt, e)); s = 1; }
            else if (p.nparts) {
                f = __ldcs(p.parts[0] + e);
                for (int q = 1; q < p.nparts; ++q) f = __fadd_rn(f, __ldcs(p.parts[q] + e));
            } else if (p.use_fin) f = p.fin[e];
            for (; s < p.S; ++s) f = ema_next(f, p.beta, p.contrib, load_any(p.g, p.gdt, s * p.gstride + e));
            F[k] = f;
            w[k] = load_any(p.w, p.wdt, e);
            if (p.variant == kVarThreshold) {
                const bool keep = importance(w[k], f, p.damp, p.mode, p.have_f != 0) >= *p.thr;
                zeroed += keep ? 0 : 1;
                w[k] = keep ? w[k] : 0.0f;
            }
            sc[k] = importance(w[k], f, p.damp, p.mode, p.have_f != 0);
            v[k] = sc[k];
        }
        if (p.variant == kVarScores) {
#pragma unroll
            for (int k = 0; k < M; ++k) {
                if (p.fout && p.have_f) p.fout[e0 + k] = F[k];
                p.sout[e0 + k] = sc[k];
            }
            continue;
        }
        if (p.ties) ties += near_tie<M>(v, p.n) ? 1 : 0;
        const uint32_t byte = select_group<M>(v, p.n, p.strategy, p.rounds, p.permute != 0, p.lut);
#pragma unroll
        for (int k = 0; k < M; ++k) w[k] = ((byte >> k) & 1u) ? w[k] : 0.0f;
        redistribute_group<M>(w, sc, byte, p.redist);
#pragma unroll
        for (int k = 0; k < M; ++k) {
            p.wout[e0 + k] = w[k];
            if (p.fout && p.have_f) p.fout[e0 + k] = F[k];
            if (p.sout) p.sout[e0 + k] = sc[k];
        }
        p.mout[g] = static_cast<uint8_t>(byte);
    }
    if (p.ties) warp_add_count(p.ties, ties);
    if (p.variant == kVarThreshold) warp_add_count(p.thr_pruned, zeroed);
}

unsigned grid_for(size_t items) {
    size_t b = (items + kThreads - 1) / kThreads;
    return static_cast<unsigned>(std::max<size_t>(1, std::min<size_t>(b, (size_t)1 << 30)));
}

template <int WDT, int GDT, int VAR = kVarPlain>
void launch_vec_m(int m, unsigned grid, cudaStream_t st, const FusedParams& p) {
    if (m == 2) fused_vec_kernel<WDT, GDT, 2, VAR><<<grid, kThreads, 0, st>>>(p);
    else if (m == 4) fused_vec_kernel<WDT, GDT, 4, VAR><<<grid, kThreads, 0, st>>>(p);
    else fused_vec_kernel<WDT, GDT, 8, VAR><<<grid, kThreads, 0, st>>>(p);
}

template <int WDT, int VAR>
void launch_vec_g(int gdt, int m, unsigned grid, cudaStream_t st, const FusedParams& p) {
    if (gdt == TB_F32) launch_vec_m<WDT, TB_F32, VAR>(m, grid, st, p);
    else if (gdt == TB_BF16) launch_vec_m<WDT, TB_BF16, VAR>(m, grid, st, p);
    else launch_vec_m<WDT, TB_F16, VAR>(m, grid, st, p);
}

// Variants that read no gradient samples (S == 0) are instantiated for one
// gradient type only.
template <int VAR>
void launch_vec_nosamples(int m, unsigned grid, cudaStream_t st, const FusedParams& p) {
    if (p.wdt == TB_F32) launch_vec_m<TB_F32, TB_BF16, VAR>(m, grid, st, p);
    else if (p.wdt == TB_BF16) launch_vec_m<TB_BF16, TB_BF16, VAR>(m, grid, st, p);
    else launch_vec_m<TB_F16, TB_BF16, VAR>(m, grid, st, p);
}

// Batches of gradient samples the vector kernel prefetches into L2 ahead of its
// register loads, so that while a thread decodes one batch its next loads (and,
// near the end, its weights) are already on the way.  Measured on B200 over
// distances 0-6: with 32 BF16 samples per element (OBS scores, iterative 2:4,
// 2:8, 4:8 on 70B-class tensors) two batches ahead raised the pass from 84-86 %
// to 88-91 % of the HBM copy bandwidth; with 64 samples (OBD, optimal 2:4) and
// 128 (Normalized) every distance lowered it (96 % to 93 %, 98 % to 93-95 %):
// the prefetches add power under the 1 kW cap (SM clock 1450 -> 1300 MHz) and
// those passes have little load latency left to hide.
// TB_L2_PREFETCH_BATCHES=<n> in the environment fixes the distance (for such
// measurements).
int prefetch_batches(size_t S) {
    static const int forced = [] {
        const char* e = std::getenv("TB_L2_PREFETCH_BATCHES");
        return e && *e ? std::max(0, std::min(8, std::atoi(e))) : -1;
    }();
    if (forced >= 0) return forced;
    return (S > 0 && S <= 48) ? 2 : 0;
}

void launch_vec(FusedParams p, int m, cudaStream_t st) {
    const unsigned grid = grid_for(p.N / kEpt);
    p.prefetch = prefetch_batches(p.S);
    if (p.variant == kVarPeer) return launch_vec_nosamples<kVarPeer>(m, grid, st, p);
    if (p.variant == kVarThreshold) return launch_vec_nosamples<kVarThreshold>(m, grid, st, p);
    if (p.variant == kVarScores) {
        if (p.wdt == TB_F32) launch_vec_g<TB_F32, kVarScores>(p.gdt, m, grid, st, p);
        else if (p.wdt == TB_BF16) launch_vec_g<TB_BF16, kVarScores>(p.gdt, m, grid, st, p);
        else launch_vec_g<TB_F16, kVarScores>(p.gdt, m, grid, st, p);
        return;
    }
    if (p.wdt == TB_F32) launch_vec_g<TB_F32, kVarPlain>(p.gdt, m, grid, st, p);
    else if (p.wdt == TB_BF16) launch_vec_g<TB_BF16, kVarPlain>(p.gdt, m, grid, st, p);
    else launch_vec_g<TB_F16, kVarPlain>(p.gdt, m, grid, st, p);
}

void launch_group(const FusedParams& p, int m, cudaStream_t st) {
    const unsigned grid = grid_for(p.N / m);
    switch (m) {
    case 2: fused_group_kernel<2><<<grid, kThreads, 0, st>>>(p); break;
    case 3: fused_group_kernel<3><<<grid, kThreads, 0, st>>>(p); break;
    case 4: fused_group_kernel<4><<<grid, kThreads, 0, st>>>(p); break;
    case 5: fused_group_kernel<5><<<grid, kThreads, 0, st>>>(p); break;
    case 6: fused_group_kernel<6><<<grid, kThreads, 0, st>>>(p); break;
    case 7: fused_group_kernel<7><<<grid, kThreads, 0, st>>>(p); break;
    default: fused_group_kernel<8><<<grid, kThreads, 0, st>>>(p); break;
    }
}

int dtype_bytes(int dt) { return dt == TB_F32 ? 4 : 2; }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool parts_aligned16(const FusedParams& p) {
    for (int k = 0; k < p.nparts; ++k)
        if (!aligned16(p.parts[k])) return false;
    return true;
}

// Validates args in the order the reference sequence would fail
// (accumulate_fisher, compute_importance, generate_nm_mask) and fills the
// kernel parameters.
int prepare(const tb_prune_args* a, FusedParams& p) {
    if (!a) return fail(TB_ERR_ARG, "null args");
    if (a->struct_size < sizeof(tb_prune_args)) return fail(TB_ERR_ARG, "tb_prune_args.struct_size too small");
    const int n = a->nm_n, m = a->nm_m;
    if (a->N == 0) return fail(TB_ERR_ZERO_SIZE, "empty tensor");
    if (n <= 0 || m <= 0 || n >= m) return fail(TB_ERR_CONFIG, "invalid N:M %d:%d", n, m);
    if (a->N % static_cast<uint64_t>(m) != 0) return fail(TB_ERR_SHAPE, "numel %llu not divisible by M=%d",
                                                           (unsigned long long)a->N, m);
    if (m > 8) return fail(TB_ERR_UNSUPPORTED, "M=%d > 8: masks hold one byte per group", m);
    if (a->w_dtype < TB_F32 || a->w_dtype > TB_BF16 || a->g_dtype < TB_F32 || a->g_dtype > TB_BF16)
        return fail(TB_ERR_ARG, "bad dtype");
    if (a->importance_mode < TB_IMP_OBD || a->importance_mode > TB_IMP_NORMALIZED)
        return fail(TB_ERR_ARG, "bad importance mode %d", a->importance_mode);
    if (a->mask_strategy < TB_MASK_TOPN || a->mask_strategy > TB_MASK_ITERATIVE)
        return fail(TB_ERR_ARG, "bad mask strategy %d", a->mask_strategy);
    if (a->redist_mode < TB_REDIST_NONE || a->redist_mode > TB_REDIST_UNIFORM)
        return fail(TB_ERR_ARG, "bad redistribution mode %d", a->redist_mode);
    if (!a->weights || !a->w_out || !a->mask_out) return fail(TB_ERR_ARG, "null weights/outputs");
    const bool use_f = a->use_fisher != 0;
    if (use_f && a->S > 0 && !a->grads) return fail(TB_ERR_ARG, "null gradients with S > 0");
    if (use_f && a->fisher_steps_in > 0 && !a->fisher_in) return fail(TB_ERR_ARG, "fisher_steps_in > 0 without fisher_in");
    const uint64_t gstride = a->g_stride ? a->g_stride : a->N;
    if (gstride < a->N) return fail(TB_ERR_ARG, "g_stride < N");

    p = FusedParams{};
    p.w = a->weights;
    p.g = a->grads;
    p.fin = a->fisher_in;
    p.wout = a->w_out;
    p.mout = a->mask_out;
    p.fout = a->fisher_out;
    p.sout = a->scores_out;
    p.ties = a->near_ties;
    p.N = a->N;
    p.S = use_f ? a->S : 0;
    p.gstride = gstride;
    p.alpha = a->alpha;
    p.beta = a->beta;
    const float one_m_beta = 1.0f - a->beta;  // ehap.hpp:165
    p.contrib = a->alpha * one_m_beta;        // ehap.hpp:195
    p.damp = a->damping;
    p.mode = a->importance_mode;
    p.use_fin = use_f && a->fisher_steps_in > 0;
    p.first = use_f && a->fisher_steps_in == 0 && a->S > 0;
    p.have_f = use_f && (a->S > 0 || a->fisher_steps_in > 0);
    p.n = n;
    p.strategy = a->mask_strategy;
    p.rounds = a->iterative_rounds;
    p.redist = a->redist_mode;
    p.permute = a->permute;
    p.wdt = a->w_dtype;
    p.gdt = a->g_dtype;
    return TB_OK;
}

int launch_fused(FusedParams p, int m, cudaStream_t st) {
    int rc = require_device(nullptr);
    if (rc) return rc;
    if (p.strategy != TB_MASK_OPTIMAL && (rc = topn_table(p.n, m, &p.lut))) return rc;
    const bool vec_m = (m == 2 || m == 4 || m == 8);
    const bool vec_ok = vec_m && aligned16(p.w) && aligned16(p.wout) && (!p.S || aligned16(p.g)) &&
                        (!p.use_fin || aligned16(p.fin)) && (!p.fout || aligned16(p.fout)) &&
                        (!p.sout || aligned16(p.sout)) &&
                        (reinterpret_cast<uintptr_t>(p.mout) % (kEpt / m) == 0) &&
                        ((p.gstride * dtype_bytes(p.gdt)) % 16 == 0) && parts_aligned16(p);
    const size_t nvec = vec_ok ? (p.N / kEpt) * kEpt : 0;
    if (nvec) {
        FusedParams q = p;
        q.N = nvec;
        launch_vec(q, m, st);
        if ((rc = check_launch("fused_vec_kernel"))) return rc;
    }
    if (nvec < p.N) {
        // Remaining elements (a multiple of M): offset every pointer.
        FusedParams t = p;
        t.N = p.N - nvec;
        t.w = static_cast<const char*>(p.w) + nvec * dtype_bytes(p.wdt);
        if (p.S) t.g = static_cast<const char*>(p.g) + nvec * dtype_bytes(p.gdt);
        if (p.fin) t.fin = p.fin + nvec;
        for (int k = 0; k < p.nparts; ++k) t.parts[k] = p.parts[k] + nvec;
        if (p.wout) t.wout = p.wout + nvec;
        if (p.mout) t.mout = p.mout + nvec / m;
        if (p.fout) t.fout = p.fout + nvec;
        if (p.sout) t.sout = p.sout + nvec;
        launch_group(t, m, st);
        if ((rc = check_launch("fused_group_kernel"))) return rc;
    }
    return TB_OK;
}

// ---- host-buffer pipeline ----------------------------------------------------
// Per-device staging for tb_score_mask_pack_host: kSlots independent
// (stream, buffers) slots; chunk k goes to slot k % kSlots, so the H2D copy of
// one chunk, the kernel of another and the D2H copy of a third overlap.  A call
// holds its device's call lock from the first copy until its outputs are in
// host memory, so calls from several host threads on one device run one after
// another and never share the slots or the tie counter; calls on different
// devices run in parallel.
constexpr int kSlots = 3;

struct Slot {
    cudaStream_t st = nullptr;
    char* dbuf = nullptr;
    size_t cap = 0;
};

struct HostPipe {
    int dev = -1;
    std::mutex call_mu;  // held for a whole tb_score_mask_pack_host call
    Slot slot[kSlots];
    unsigned long long* ties = nullptr;
};

std::mutex g_pipe_mu;
std::vector<HostPipe*> g_pipes;

// The device's pipe (streams and tie counter created on first use).
int get_pipe(int dev, HostPipe** out) {
    std::lock_guard<std::mutex> lk(g_pipe_mu);
    for (auto* x : g_pipes)
        if (x->dev == dev) {
            *out = x;
            return TB_OK;
        }
    auto* hp = new HostPipe;
    hp->dev = dev;
    for (auto& s : hp->slot) {
        cudaError_t e = cudaStreamCreateWithFlags(&s.st, cudaStreamNonBlocking);
        if (e != cudaSuccess) return cuda_fail(e, "cudaStreamCreate");
    }
    cudaError_t e = cudaMalloc(&hp->ties, sizeof(unsigned long long));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(tie counter)");
    g_pipes.push_back(hp);
    *out = hp;
    return TB_OK;
}

// Grows every slot to `need` bytes.  Called with hp->call_mu held, after the
// previous call drained the slot streams, so no copy or kernel uses a buffer
// that is freed here.
int grow_slots(HostPipe* hp, size_t need) {
    for (auto& s : hp->slot) {
        if (s.cap >= need) continue;
        if (s.dbuf) {
            cudaStreamSynchronize(s.st);
            cudaFree(s.dbuf);
            s.dbuf = nullptr;
            s.cap = 0;
        }
        cudaError_t e = cudaMalloc(&s.dbuf, need);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(host-path staging)");
        s.cap = need;
    }
    return TB_OK;
}

// Waits for every slot stream when a call returns, also on an error path, so
// no copy into or out of the caller's host buffers is left in flight.
struct DrainSlots {
    HostPipe* hp;
    ~DrainSlots() {
        for (auto& s : hp->slot) cudaStreamSynchronize(s.st);
    }
};

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

int tb_fisher_partial_scatter(const void* gradients, int g_dtype, size_t S, size_t g_stride, size_t N,
                              const float* weights, int n_ranks, const uint64_t* starts, float* const* dest,
                              int start_owner, void* stream) {
    if (N == 0) return TB_OK;
    if (n_ranks < 1 || n_ranks > kMaxScatterRanks)
        return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: %d ranks (1..%d)", n_ranks, kMaxScatterRanks);
    if (S > static_cast<size_t>(kMaxPartialSamples))
        return fail(TB_ERR_CAPACITY, "tb_fisher_partial_scatter: %zu samples in one call (at most %d)", S,
                    kMaxPartialSamples);
    if (!starts || !dest || (S && (!gradients || !weights)))
        return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: null pointer");
    if (g_dtype < TB_F32 || g_dtype > TB_BF16) return fail(TB_ERR_ARG, "bad gradient dtype %d", g_dtype);
    const size_t stride = g_stride ? g_stride : N;
    if (stride < N) return fail(TB_ERR_ARG, "g_stride < N");
    if (starts[0] != 0 || starts[n_ranks] != N)
        return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: ranges must cover [0, N)");
    PartialSpec q{};
    q.g = gradients;
    q.S = S;
    q.gstride = stride;
    q.N = N;
    for (size_t k = 0; k < S; ++k) q.c[k] = weights[k];
    q.nranks = n_ranks;
    bool aligned = true;
    for (int r = 0; r <= n_ranks; ++r) {
        q.start[r] = starts[r];
        if (r > 0 && starts[r] < starts[r - 1]) return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: ranges out of order");
        if (r > 0 && r < n_ranks && starts[r] % 8) return fail(TB_ERR_ARG, "range start %llu not a multiple of 8",
                                                               (unsigned long long)starts[r]);
    }
    for (int r = 0; r < n_ranks; ++r) {
        if (starts[r + 1] > starts[r] && !dest[r]) return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: null dest %d", r);
        q.dest[r] = dest[r];
        aligned = aligned && aligned16(dest[r]);
    }
    if (start_owner < 0 || start_owner >= n_ranks)
        return fail(TB_ERR_ARG, "tb_fisher_partial_scatter: start_owner %d outside 0..%d", start_owner, n_ranks - 1);
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const bool vec = S > 0 && aligned && aligned16(gradients) && (stride * dtype_bytes(g_dtype)) % 16 == 0;
    const size_t nvec = vec ? N / kEpt * kEpt : 0;
    q.rot = nvec ? std::min(starts[start_owner] / kEpt, nvec / kEpt - 1) : 0;
    if (nvec) {
        const unsigned grid = grid_for(nvec / kEpt);
        if (g_dtype == TB_BF16) partial_vec_kernel<TB_BF16><<<grid, kThreads, 0, st>>>(q);
        else if (g_dtype == TB_F16) partial_vec_kernel<TB_F16><<<grid, kThreads, 0, st>>>(q);
        else partial_vec_kernel<TB_F32><<<grid, kThreads, 0, st>>>(q);
        if ((rc = check_launch("partial_vec_kernel"))) return rc;
    }
    const size_t done = nvec;
    if (done < N) {
        partial_scalar_kernel<<<grid_for(N - done), kThreads, 0, st>>>(q, g_dtype, done);
        if ((rc = check_launch("partial_scalar_kernel"))) return rc;
    }
    return TB_OK;
}

int tb_score_mask_pack(const tb_prune_args* args, void* stream) {
    FusedParams p;
    int rc = prepare(args, p);
    if (rc) return rc;
    return launch_fused(p, args->nm_m, static_cast<cudaStream_t>(stream));
}

int tb_score_mask_pack_peer(const tb_prune_args* args, const float* const* partials, int n_partials,
                            void* stream) {
    if (!args) return fail(TB_ERR_ARG, "null args");
    if (n_partials < 1 || n_partials > kMaxParts)
        return fail(TB_ERR_ARG, "tb_score_mask_pack_peer: %d partials (1..%d)", n_partials, kMaxParts);
    if (!partials) return fail(TB_ERR_ARG, "tb_score_mask_pack_peer: null partials");
    for (int k = 0; k < n_partials; ++k)
        if (!partials[k]) return fail(TB_ERR_ARG, "tb_score_mask_pack_peer: partial %d is null", k);
    if (args->S != 0 || args->fisher_in)
        return fail(TB_ERR_ARG, "tb_score_mask_pack_peer: the partials are the Fisher state (S must be 0, "
                                "fisher_in NULL)");
    if (!args->use_fisher || args->fisher_steps_in == 0)
        return fail(TB_ERR_ARG, "tb_score_mask_pack_peer: use_fisher with fisher_steps_in > 0 required");
    tb_prune_args a = *args;
    a.fisher_in = partials[0];  // passes the stateful-entry checks; replaced by the sum below
    FusedParams p;
    int rc = prepare(&a, p);
    if (rc) return rc;
    p.use_fin = 0;
    p.fin = nullptr;
    p.nparts = n_partials;
    p.variant = kVarPeer;
    for (int k = 0; k < n_partials; ++k) p.parts[k] = partials[k];
    return launch_fused(p, args->nm_m, static_cast<cudaStream_t>(stream));
}

// The one-shot sequence; the threshold and EHAP count go to host values
// (thr_host / pruned_host, with a host wait when either is asked for) and/or
// are copied, stream-ordered, to device-accessible thr_dst / pruned_dst.
static int one_shot(const tb_prune_args* args, float sparsity, float* thr_host, uint64_t* pruned_host, float* thr_dst,
             uint64_t* pruned_dst, uint64_t* coring_pruned_out, void* stream) {
    if (!args) return fail(TB_ERR_ARG, "null args");
    // EHAP's checks come first, as in the reference sequence (the global select
    // runs before CORING sees the tensor).
    size_t keep = 0;
    int rc = threshold_args(args->N, sparsity, &keep);
    if (rc) return rc;
    FusedParams p;
    if ((rc = prepare(args, p))) return rc;
    if (!args->scores_out) return fail(TB_ERR_ARG, "tb_prune_one_shot_nm: scores_out is required");
    if (p.have_f && !args->fisher_out)
        return fail(TB_ERR_ARG, "tb_prune_one_shot_nm: fisher_out is required when a Fisher state exists");
    const int m = args->nm_m;
    const size_t N = args->N;
    auto st = static_cast<cudaStream_t>(stream);
    // Pass 1: Fisher EMA and the importance the global select ranks.
    FusedParams a = p;
    a.variant = kVarScores;
    a.wout = nullptr;
    a.mout = nullptr;
    a.ties = nullptr;
    a.fout = p.have_f ? args->fisher_out : nullptr;
    a.sout = args->scores_out;
    if ((rc = launch_fused(a, m, st))) return rc;
    // The threshold's three digit passes over the scores (keep < N).
    SelectState* sel = nullptr;
    if (keep < N) {
        if ((rc = scratch_alloc(reinterpret_cast<void**>(&sel), sizeof(SelectState), st))) return rc;
        if ((rc = threshold_digits(args->scores_out, N, keep, sel, st))) {
            scratch_free(sel, st);
            return rc;
        }
    }
    // Pass 2: threshold keep, recomputed importance, CORING, .tb sections.
    FusedParams b = p;
    b.S = 0;
    b.g = nullptr;
    b.first = 0;
    b.use_fin = p.have_f;
    b.fin = p.have_f ? args->fisher_out : nullptr;
    b.fout = nullptr;
    b.sout = args->scores_out;
    if (sel) {
        b.variant = kVarThreshold;
        b.thr = &sel->threshold;
        b.thr_pruned = &sel->pruned;
    }
    rc = launch_fused(b, m, st);
    if (rc == TB_OK && (thr_dst || pruned_dst)) {
        if (!sel) {  // everything kept: threshold 0, nothing pruned
            if ((rc = scratch_alloc(reinterpret_cast<void**>(&sel), sizeof(SelectState), st))) return rc;
            rc = threshold_clear(sel, st);
        }
        cudaError_t e = cudaSuccess;
        if (rc == TB_OK && thr_dst)
            e = cudaMemcpyAsync(thr_dst, &sel->threshold, sizeof(float), cudaMemcpyDefault, st);
        if (rc == TB_OK && e == cudaSuccess && pruned_dst)
            e = cudaMemcpyAsync(pruned_dst, &sel->pruned, sizeof(uint64_t), cudaMemcpyDefault, st);
        if (rc == TB_OK && e != cudaSuccess) rc = cuda_fail(e, "tb_prune_one_shot_nm_async result copy");
    }
    if (rc == TB_OK) rc = threshold_finish(N, keep, sel, thr_host, pruned_host, st);
    scratch_free(sel, st);
    if (rc == TB_OK && coring_pruned_out)
        *coring_pruned_out = static_cast<uint64_t>(N / m) * static_cast<uint64_t>(m - args->nm_n);  // coring.hpp:192,222
    return rc;
}

int tb_prune_one_shot_nm(const tb_prune_args* args, float sparsity, float* threshold_out,
                         uint64_t* ehap_pruned_out, uint64_t* coring_pruned_out, void* stream) {
    return one_shot(args, sparsity, threshold_out, ehap_pruned_out, nullptr, nullptr, coring_pruned_out, stream);
}

int tb_prune_one_shot_nm_async(const tb_prune_args* args, float sparsity, float* threshold_dst,
                               uint64_t* ehap_pruned_dst, uint64_t* coring_pruned_out, void* stream) {
    return one_shot(args, sparsity, nullptr, nullptr, threshold_dst, ehap_pruned_dst, coring_pruned_out, stream);
}

int tb_score_mask_pack_host(const tb_prune_args* a) {
    FusedParams p;
    int rc = prepare(a, p);
    if (rc) return rc;
    int dev = 0;
    if ((rc = require_device(&dev))) return rc;
    const int m = a->nm_m;
    const size_t N = a->N, S = p.S;
    const int wb = dtype_bytes(a->w_dtype), gb = dtype_bytes(a->g_dtype);
    // Chunk: a multiple of 16 elements and of M, about 64 MB of gradients.
    size_t chunk = (64ull << 20) / std::max<size_t>(1, S * gb + wb + 8);
    chunk = std::max<size_t>(chunk / 16 / m * 16 * m, static_cast<size_t>(16 * m));
    chunk = std::min(chunk, round_up(N, static_cast<size_t>(16 * m)));
    // Staging layout per slot: [W][G (S rows of chunk)][F_in][W'][mask][F_out][s_out]
    const size_t o_w = 0;
    const size_t o_g = round_up(o_w + chunk * wb, 256);
    const size_t o_fi = round_up(o_g + S * chunk * gb, 256);
    const size_t o_wo = round_up(o_fi + (p.use_fin ? chunk * 4 : 0), 256);
    const size_t o_m = round_up(o_wo + chunk * 4, 256);
    const size_t o_fo = round_up(o_m + chunk / m, 256);
    const size_t o_so = round_up(o_fo + (p.fout ? chunk * 4 : 0), 256);
    const size_t need = round_up(o_so + (p.sout ? chunk * 4 : 0), 256);
    HostPipe* hp = nullptr;
    if ((rc = get_pipe(dev, &hp))) return rc;
    std::lock_guard<std::mutex> call_lock(hp->call_mu);
    DrainSlots drain{hp};
    if ((rc = grow_slots(hp, need))) return rc;
    if (p.ties) {
        cudaError_t e = cudaMemsetAsync(hp->ties, 0, sizeof(unsigned long long), hp->slot[0].st);
        if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
        // Every slot stream must see the zeroed counter.
        cudaStreamSynchronize(hp->slot[0].st);
    }
    const char* hw = static_cast<const char*>(a->weights);
    const char* hg = static_cast<const char*>(a->grads);
    const size_t gstride = p.gstride;
    size_t k = 0;
    for (size_t e0 = 0; e0 < N; e0 += chunk, ++k) {
        const size_t len = std::min(chunk, N - e0);
        Slot& sl = hp->slot[k % kSlots];
        char* d = sl.dbuf;
        cudaError_t e = cudaMemcpyAsync(d + o_w, hw + e0 * wb, len * wb, cudaMemcpyHostToDevice, sl.st);
        if (e == cudaSuccess && S)
            e = cudaMemcpy2DAsync(d + o_g, len * gb, hg + e0 * gb, gstride * gb, len * gb, S, cudaMemcpyHostToDevice, sl.st);
        if (e == cudaSuccess && p.use_fin)
            e = cudaMemcpyAsync(d + o_fi, a->fisher_in + e0, len * 4, cudaMemcpyHostToDevice, sl.st);
        if (e != cudaSuccess) return cuda_fail(e, "host-path H2D copy");
        FusedParams q = p;
        q.N = len;
        q.w = d + o_w;
        q.g = S ? d + o_g : nullptr;
        q.gstride = len;
        q.fin = p.use_fin ? reinterpret_cast<const float*>(d + o_fi) : nullptr;
        q.wout = reinterpret_cast<float*>(d + o_wo);
        q.mout = reinterpret_cast<uint8_t*>(d + o_m);
        q.fout = p.fout ? reinterpret_cast<float*>(d + o_fo) : nullptr;
        q.sout = p.sout ? reinterpret_cast<float*>(d + o_so) : nullptr;
        q.ties = p.ties ? hp->ties : nullptr;
        if ((rc = launch_fused(q, m, sl.st))) return rc;
        e = cudaMemcpyAsync(a->w_out + e0, q.wout, len * 4, cudaMemcpyDeviceToHost, sl.st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(a->mask_out + e0 / m, q.mout, len / m, cudaMemcpyDeviceToHost, sl.st);
        if (e == cudaSuccess && q.fout) e = cudaMemcpyAsync(a->fisher_out + e0, q.fout, len * 4, cudaMemcpyDeviceToHost, sl.st);
        if (e == cudaSuccess && q.sout) e = cudaMemcpyAsync(a->scores_out + e0, q.sout, len * 4, cudaMemcpyDeviceToHost, sl.st);
        if (e != cudaSuccess) return cuda_fail(e, "host-path D2H copy");
    }
    for (auto& sl : hp->slot) {
        cudaError_t e = cudaStreamSynchronize(sl.st);
        if (e != cudaSuccess) return cuda_fail(e, "host-path synchronise");
    }
    if (p.ties) {
        unsigned long long t = 0;
        cudaError_t e = cudaMemcpy(&t, hp->ties, sizeof(t), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) return cuda_fail(e, "tie counter D2H");
        *a->near_ties += t;
    }
    return TB_OK;
}

}  // extern "C"

// ---- host-buffer pass without device allocation ----------------------------
// Some callers cannot let this library call cudaMalloc: a process whose GPU
// memory is already fully reserved by another allocator (a framework's caching
// pool, or a serving process that pins its budget at start-up) would see the
// allocation fail or fragment its pool.  tb_score_mask_pack_host_noalloc stages
// through the fixed array below instead.  The array is a file-scope device
// variable, so every GPU that loads this library holds its 16 MiB until the
// process exits.  Host code must not take its address directly (in host code
// the name is only a stand-in); the device address comes from
// cudaGetSymbolAddress, once per device, with that device current.
static __device__ __align__(256) unsigned char g_tb_noalloc_staging[16u << 20];

namespace tb {
namespace {

constexpr size_t kNoAllocBytes = sizeof(g_tb_noalloc_staging);
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
char* g_noalloc_addr[kMaxDevices] = {};

// Device address of the staging array on `dev` (the current device); the
// first call per device resolves and caches it.
int noalloc_staging(int dev, char** out) {
    if (dev < 0 || dev >= kMaxDevices) return fail(TB_ERR_UNSUPPORTED, "device ordinal %d >= %d", dev, kMaxDevices);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_tb_noalloc_staging);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc staging)");
        g_noalloc_addr[dev] = static_cast<char*>(p);
    }
    *out = g_noalloc_addr[dev];
    return TB_OK;
}

}  // namespace
}  // namespace tb

extern "C" int tb_score_mask_pack_host_noalloc(const tb_prune_args* a) {
    FusedParams p;
    int rc = prepare(a, p);
    if (rc) return rc;
    int dev = 0;
    if ((rc = require_device(&dev))) return rc;
    const int m = a->nm_m;
    if (p.strategy != TB_MASK_OPTIMAL && !topn_table_ready(p.n, m))
        return fail(TB_ERR_UNSUPPORTED,
                    "top-N tie table for %d:%d is not on this device yet and building it would allocate; "
                    "call tb_prepare_nm(%d, %d) once where allocation is allowed, or use TB_MASK_OPTIMAL",
                    p.n, m, p.n, m);
    char* base = nullptr;
    if ((rc = noalloc_staging(dev, &base))) return rc;
    const size_t N = a->N, S = p.S;
    const size_t wb = dtype_bytes(a->w_dtype), gb = dtype_bytes(a->g_dtype);
    // Bytes one element occupies across the staging regions, and the fixed
    // overhead: the tie counter and up to 256 bytes of alignment per region.
    const size_t per_elem = wb + S * gb + (p.use_fin ? 4 : 0) + 4 + 1 + (p.fout ? 4 : 0) + (p.sout ? 4 : 0);
    const size_t fixed = 256 + 8 * 256;
    const size_t unit = static_cast<size_t>(16 * m);
    size_t chunk = kNoAllocBytes > fixed ? (kNoAllocBytes - fixed) / per_elem / unit * unit : 0;
    if (chunk == 0)
        return fail(TB_ERR_CAPACITY,
                    "tb_score_mask_pack_host_noalloc: one %zu-element chunk with %zu samples needs %zu bytes; "
                    "the static staging array holds %zu bytes",
                    unit, S, fixed + unit * per_elem, kNoAllocBytes);
    chunk = std::min(chunk, round_up(N, unit));
    unsigned long long* ties = reinterpret_cast<unsigned long long*>(base);
    const size_t o_w = 256;
    const size_t o_g = round_up(o_w + chunk * wb, 256);
    const size_t o_fi = round_up(o_g + S * chunk * gb, 256);
    const size_t o_wo = round_up(o_fi + (p.use_fin ? chunk * 4 : 0), 256);
    const size_t o_m = round_up(o_wo + chunk * 4, 256);
    const size_t o_fo = round_up(o_m + chunk / m, 256);
    const size_t o_so = round_up(o_fo + (p.fout ? chunk * 4 : 0), 256);
    if (round_up(o_so + (p.sout ? chunk * 4 : 0), 256) > kNoAllocBytes)
        return fail(TB_ERR_CAPACITY, "tb_score_mask_pack_host_noalloc: staging layout exceeds %zu bytes", kNoAllocBytes);
    // One sequential pass on the legacy default stream.  The array keeps the
    // previous call's contents; only the tie counter must start at zero.
    cudaStream_t st = 0;
    cudaError_t e = cudaSuccess;
    if (p.ties) e = cudaMemsetAsync(ties, 0, sizeof(*ties), st);
    if (e != cudaSuccess) return cuda_fail(e, "no-alloc tie counter reset");
    const char* hw = static_cast<const char*>(a->weights);
    const char* hg = static_cast<const char*>(a->grads);
    for (size_t e0 = 0; e0 < N; e0 += chunk) {
        const size_t len = std::min(chunk, N - e0);
        e = cudaMemcpyAsync(base + o_w, hw + e0 * wb, len * wb, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess && S)
            e = cudaMemcpy2DAsync(base + o_g, len * gb, hg + e0 * gb, p.gstride * gb, len * gb, S,
                                  cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess && p.use_fin)
            e = cudaMemcpyAsync(base + o_fi, a->fisher_in + e0, len * 4, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return cuda_fail(e, "no-alloc H2D copy");
        FusedParams q = p;
        q.N = len;
        q.w = base + o_w;
        q.g = S ? base + o_g : nullptr;
        q.gstride = len;
        q.fin = p.use_fin ? reinterpret_cast<const float*>(base + o_fi) : nullptr;
        q.wout = reinterpret_cast<float*>(base + o_wo);
        q.mout = reinterpret_cast<uint8_t*>(base + o_m);
        q.fout = p.fout ? reinterpret_cast<float*>(base + o_fo) : nullptr;
        q.sout = p.sout ? reinterpret_cast<float*>(base + o_so) : nullptr;
        q.ties = p.ties ? ties : nullptr;
        if ((rc = launch_fused(q, m, st))) return rc;
        e = cudaMemcpyAsync(a->w_out + e0, q.wout, len * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaMemcpyAsync(a->mask_out + e0 / m, q.mout, len / m, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess && q.fout) e = cudaMemcpyAsync(a->fisher_out + e0, q.fout, len * 4, cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess && q.sout) e = cudaMemcpyAsync(a->scores_out + e0, q.sout, len * 4, cudaMemcpyDeviceToHost, st);
        if (e != cudaSuccess) return cuda_fail(e, "no-alloc D2H copy");
    }
    unsigned long long t = 0;
    if (p.ties) e = cudaMemcpyAsync(&t, ties, sizeof(t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "no-alloc synchronise");
    if (p.ties) *a->near_ties += t;
    return TB_OK;
}

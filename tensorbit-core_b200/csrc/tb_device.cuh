// Device building blocks shared by the pruning kernels.
//
// Arithmetic contract: every float operation that reproduces a reference
// expression goes through the round-to-nearest intrinsics (__fmul_rn,
// __fadd_rn, __fdiv_rn), which the compiler never fuses into FMA.  The
// reference is built with FP contraction off (ISO C++20, CMakeLists.txt:33-35),
// so its host loops round every product and sum separately; these helpers keep
// the same expression trees and therefore the same bits.
#pragma once

#include <cstdint>
#include <cfloat>
#include <cuda_runtime.h>

#include "tb_kernels.h"

namespace tb {

// ---------------------------------------------------------------------------
// Element decode (src/main.cpp:213-245)
// ---------------------------------------------------------------------------

// BF16 -> FP32: the 16 bits become the high half of the FP32 word.
__device__ __forceinline__ float bf16_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// F16 -> FP32 exactly as the reference loader widens it.  Exponent 0 keeps the
// 10-bit fraction in an FP32 with exponent 0 (not the IEEE subnormal value);
// exponent 31 maps to FP32 Inf/NaN; otherwise the exponent is rebiased.
__device__ __forceinline__ float f16ref_to_f32(uint32_t h) {
    const uint32_t sign = (h >> 15) << 31;
    const uint32_t e = (h >> 10) & 0x1Fu;
    const uint32_t frac = (h & 0x3FFu) << 13;
    uint32_t f;
    if (e == 0) f = sign | frac;
    else if (e == 31) f = sign | 0x7F800000u | frac;
    else f = sign | ((e + 112u) << 23) | frac;
    return __uint_as_float(f);
}

template <int DT> struct Dtype;
template <> struct Dtype<TB_F32> {
    static constexpr int kBytes = 4;
    __device__ static float load(const void* p, size_t i) { return static_cast<const float*>(p)[i]; }
};
template <> struct Dtype<TB_BF16> {
    static constexpr int kBytes = 2;
    __device__ static float load(const void* p, size_t i) { return bf16_to_f32(static_cast<const uint16_t*>(p)[i]); }
};
template <> struct Dtype<TB_F16> {
    static constexpr int kBytes = 2;
    __device__ static float load(const void* p, size_t i) { return f16ref_to_f32(static_cast<const uint16_t*>(p)[i]); }
};

__device__ __forceinline__ float load_any(const void* p, int dt, size_t i) {
    if (dt == TB_F32) return Dtype<TB_F32>::load(p, i);
    if (dt == TB_BF16) return Dtype<TB_BF16>::load(p, i);
    return Dtype<TB_F16>::load(p, i);
}

// Streaming 16-byte load that bypasses L1 allocation (each byte is read once).
__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void stg_stream(float4* p, float4 v) { __stcs(p, v); }

// Hint: bring the line holding p into L2 (no register result, no wait).
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// ---------------------------------------------------------------------------
// Stage 1 arithmetic (include/tensorbit/core/ehap.hpp)
// ---------------------------------------------------------------------------

// accumulate_fisher, first step: fo[i] = alpha * gi[i] * gi[i]   (ehap.hpp:190-192)
__device__ __forceinline__ float ema_first(float alpha, float g) {
    return __fmul_rn(__fmul_rn(alpha, g), g);
}
// accumulate_fisher, later steps: decay * fo[i] + contrib * gi[i] * gi[i] (ehap.hpp:194-197)
__device__ __forceinline__ float ema_next(float F, float beta, float contrib, float g) {
    return __fadd_rn(__fmul_rn(beta, F), __fmul_rn(__fmul_rn(contrib, g), g));
}

// Two lanes of ema_next with the three products in packed FP32 (sm_100
// mul.rn.f32x2) and the sum in scalar round-to-nearest: 5 instructions per
// pair instead of 8, bit-identical to two ema_next calls.  The sum must stay
// scalar: with a packed add after the packed products, the compiler fused the
// pair into multiply-adds despite .rn and -fmad=false (measured: 1-ulp
// differences in 20-87 % of elements), while each packed op on its own and
// this form match the scalar results exactly.  beta2 / c2 hold the scalar in
// both halves (pack2).
__device__ __forceinline__ uint64_t pack2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void ema_next2(float& f0, float& f1, uint64_t beta2, uint64_t c2, float g0, float g1) {
    float t0, t1, u0, u1;
    asm("{\n\t.reg .b64 F, G, T, U;\n\t"
        "mov.b64 F, {%4, %5};\n\tmov.b64 G, {%6, %7};\n\t"
        "mul.rn.f32x2 T, %9, G;\n\tmul.rn.f32x2 T, T, G;\n\t"
        "mul.rn.f32x2 U, %8, F;\n\t"
        "mov.b64 {%0, %1}, T;\n\tmov.b64 {%2, %3}, U;\n\t}"
        : "=f"(t0), "=f"(t1), "=f"(u0), "=f"(u1)
        : "f"(f0), "f"(f1), "f"(g0), "f"(g1), "l"(beta2), "l"(c2));
    f0 = __fadd_rn(u0, t0);
    f1 = __fadd_rn(u1, t1);
}

// compute_importance (ehap.hpp:260-282).  have_f == false is the "no Fisher
// state" branch (s = w * w).
__device__ __forceinline__ float importance(float w, float F, float damp, int mode, bool have_f) {
    const float w2 = __fmul_rn(w, w);
    if (!have_f) return w2;
    const float fd = __fadd_rn(F, damp);
    if (mode == TB_IMP_OBD) return __fmul_rn(w2, fd);
    if (mode == TB_IMP_OBS) return __fdiv_rn(w2, fd);
    return __fdiv_rn(__fmul_rn(w2, fd), __fadd_rn(1.0f, w2));
}

// ---------------------------------------------------------------------------
// Stage 2: per-group N:M selection (include/tensorbit/core/coring.hpp)
// ---------------------------------------------------------------------------

// Top-N of one group as the reference's std::nth_element picks it
// (coring.hpp:376-392).  When the N-th and (N+1)-th largest scores differ the
// kept set is unique and any correct selection returns it.  When they tie,
// the reference's choice depends only on the weak order of the M scores
// (nth_element only compares), so the group's "greater-than counts"
// gt[i] = #{j : v[j] > v[i]} - which encode that weak order - index a table
// recorded from the same std::nth_element call on the host (tb_lut.cpp).
template <int M>
__device__ __forceinline__ uint32_t select_topn(const float (&v)[M], int n, const uint8_t* __restrict__ lut) {
    int gt[M];
#pragma unroll
    for (int i = 0; i < M; ++i) gt[i] = 0;
#pragma unroll
    for (int i = 0; i < M; ++i)
#pragma unroll
        for (int j = i + 1; j < M; ++j) {
            gt[j] += (v[i] > v[j]) ? 1 : 0;
            gt[i] += (v[j] > v[i]) ? 1 : 0;
        }
    uint32_t bits = 0;
    int cnt = 0;
#pragma unroll
    for (int i = 0; i < M; ++i)
        if (gt[i] < n) { bits |= 1u << i; ++cnt; }
    if (cnt == n) return bits;
    uint32_t key = 0, scale = 1;
#pragma unroll
    for (int i = 0; i < M; ++i) { key += static_cast<uint32_t>(gt[i]) * scale; scale *= M; }
    return lut[key];
}

// Exhaustive C(M,N) search (coring.hpp:397-422): subsets in Gosper order,
// each sum accumulated in ascending index order from +0, first strict maximum
// kept, initial best = -FLT_MAX with an empty mask.
template <int M>
__device__ __forceinline__ uint32_t select_optimal(const float (&v)[M], int n) {
    uint32_t best = 0;
    float best_sum = -FLT_MAX;
    uint32_t bits = (1u << n) - 1u;
    const uint32_t limit = 1u << M;
    while (bits < limit) {
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < M; ++i)
            if (bits & (1u << i)) sum = __fadd_rn(sum, v[i]);
        if (sum > best_sum) { best_sum = sum; best = bits; }
        const uint32_t c = bits & (0u - bits);
        const uint32_t r = bits + c;
        // c is a power of two, so the reference's division by c is this shift.
        bits = (((r ^ bits) >> 2) >> (__ffs(c) - 1)) | r;
    }
    return best;
}

// Swap-refine rounds of generate_iterative (coring.hpp:427-457) for one group.
// A group that does not change in a round cannot change in a later one (same
// byte, same scores), so stopping per group equals the reference's global
// early exit.
template <int M>
__device__ __forceinline__ uint32_t refine(const float (&v)[M], uint32_t byte, int rounds) {
    for (int r = 0; r < rounds; ++r) {
        bool changed = false;
#pragma unroll
        for (int pi = 0; pi < M; ++pi) {
            if (changed || (byte & (1u << pi))) continue;
#pragma unroll
            for (int ki = 0; ki < M; ++ki) {
                if (changed || !(byte & (1u << ki))) continue;
                if (v[pi] > v[ki]) {
                    byte = (byte & ~(1u << ki)) | (1u << pi);
                    changed = true;
                }
            }
        }
        if (!changed) break;
    }
    return byte;
}

// apply_permutation (coring.hpp:340-357): the group's scores reordered by |s|
// descending.  The reference sorts M <= 16 pairs with std::sort, which for so
// few elements is an insertion sort and therefore stable; this computes the
// same stable order by rank.
template <int M>
__device__ __forceinline__ void permute_by_magnitude(float (&v)[M]) {
    int rank[M];
#pragma unroll
    for (int i = 0; i < M; ++i) {
        const float ai = fabsf(v[i]);
        int r = 0;
#pragma unroll
        for (int j = 0; j < M; ++j) {
            const float aj = fabsf(v[j]);
            r += (aj > ai || (j < i && !(ai > aj) && !(aj > ai))) ? 1 : 0;
        }
        rank[i] = r;
    }
    float out[M];
#pragma unroll
    for (int p = 0; p < M; ++p) {
        float x = 0.0f;
#pragma unroll
        for (int i = 0; i < M; ++i) x = (rank[i] == p) ? v[i] : x;
        out[p] = x;
    }
#pragma unroll
    for (int p = 0; p < M; ++p) v[p] = out[p];
}

// generate_nm_mask for one group (coring.hpp:141-162).  The hardware-aware
// 2:4 layout hook is a no-op in the reference (coring.hpp:367-371).
template <int M>
__device__ __forceinline__ uint32_t select_group(float (&v)[M], int n, int strategy, int rounds,
                                                 bool permute, const uint8_t* __restrict__ lut) {
    if (permute) permute_by_magnitude<M>(v);
    if (strategy == TB_MASK_OPTIMAL) return select_optimal<M>(v, n);
    uint32_t byte = select_topn<M>(v, n, lut);
    // A swap needs a pruned score greater than a kept one.  The top-N byte
    // keeps every score with fewer than N strictly greater ones (ties at the
    // boundary resolved by the table), so a pruned score above a kept one
    // would have at least N + 1 scores above that kept one: impossible unless
    // a comparison is undefined, i.e. the group holds a NaN.  Only such
    // groups run the rounds, with the reference's comparisons.
    if (strategy == TB_MASK_ITERATIVE) {
        bool nan = false;
#pragma unroll
        for (int i = 0; i < M; ++i) nan |= (v[i] != v[i]);
        if (nan) byte = refine<M>(v, byte, rounds);
    }
    return byte;
}

// Near-tie test of one group: |s_(N) - s_(N+1)| <= 1e-6 * max(|s_(N)|, FLT_MIN)
// over the scores sorted descending.  Exact ties count.
template <int M>
__device__ __forceinline__ bool near_tie(const float (&v)[M], int n) {
    int gt[M];
#pragma unroll
    for (int i = 0; i < M; ++i) gt[i] = 0;
#pragma unroll
    for (int i = 0; i < M; ++i)
#pragma unroll
        for (int j = i + 1; j < M; ++j) {
            gt[j] += (v[i] > v[j]) ? 1 : 0;
            gt[i] += (v[j] > v[i]) ? 1 : 0;
        }
    int cnt = 0;
    float a = FLT_MAX, b = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        if (gt[i] < n) { ++cnt; a = fminf(a, v[i]); }
        else b = fmaxf(b, v[i]);
    }
    if (cnt != n) return true;
    const float scale = fmaxf(fabsf(a), FLT_MIN);
    return fabsf(__fsub_rn(a, b)) <= __fmul_rn(1e-6f, scale);
}

// CORINGPruner::redistribute for one group (coring.hpp:245-291) on the
// weights as they are (after apply_mask the pruned ones are +0, so the pruned
// magnitude is 0 and the group is skipped, exactly as in the reference).
template <int M>
__device__ __forceinline__ void redistribute_group(float (&w)[M], const float (&s)[M], uint32_t byte,
                                                   int mode) {
    if (mode == TB_REDIST_NONE) return;
    float pruned_mag = 0.0f;
    int kept = 0;
#pragma unroll
    for (int i = 0; i < M; ++i) {
        if (!((byte >> i) & 1u)) pruned_mag = __fadd_rn(pruned_mag, fabsf(w[i]));
        else ++kept;
    }
    if (kept == 0 || pruned_mag <= 0.0f) return;
    if (mode == TB_REDIST_UNIFORM) {
        const float share = __fdiv_rn(pruned_mag, static_cast<float>(kept));
#pragma unroll
        for (int i = 0; i < M; ++i)
            if ((byte >> i) & 1u) {
                const float sign = (w[i] >= 0.0f) ? 1.0f : -1.0f;
                w[i] = __fadd_rn(w[i], __fmul_rn(sign, share));
            }
        return;
    }
    float ksum = 0.0f;
#pragma unroll
    for (int i = 0; i < M; ++i)
        if ((byte >> i) & 1u) ksum = __fadd_rn(ksum, s[i]);
    if (ksum <= 0.0f) return;
#pragma unroll
    for (int i = 0; i < M; ++i)
        if ((byte >> i) & 1u) {
            const float frac = __fdiv_rn(s[i], ksum);
            const float sign = (w[i] >= 0.0f) ? 1.0f : -1.0f;
            w[i] = __fadd_rn(w[i], __fmul_rn(__fmul_rn(sign, pruned_mag), frac));
        }
}

}  // namespace tb

// tcgen05 NT GEMM for sm_100a (see tb_umma.cuh for the contract).
//
// Descriptor encodings follow the sm100 UMMA definitions (matrix descriptor:
// start address >> 4 in bits 0-13, leading byte offset >> 4 in 16-29, stride
// byte offset >> 4 in 32-45, version 1 in 46-47, layout type in 61-63 with
// 2 = 128-byte swizzle; instruction descriptor: D format bits 4-5, A/B formats
// bits 7-9 / 10-12, K-major bits 15/16 = 0, N >> 3 in bits 17-22, M >> 4 in
// bits 24-28).  Operand tiles are 128 rows x 128 bytes loaded by TMA with the
// 128-byte swizzle, which is the canonical K-major SW128 layout: 8-row groups
// 1024 bytes apart (SBO = 64), and each 32-byte K step of one MMA is a +2
// advance of the descriptor's start address.
#include <cuda.h>

#include <algorithm>
#include <cstdio>
#include <mutex>

#include "tb_pdl.cuh"
#include "tb_runtime.h"
#include "tb_umma.cuh"

namespace tb {
namespace umma {
namespace {

constexpr int kTile = 128;              // rows of A / B per tile, M = N = 128
// Operand K-slices are 128 rows x SW bytes, loaded by TMA with the SW-byte
// swizzle (SW = 128 or 64): the canonical K-major layouts whose 8-row atoms
// sit 8 * SW bytes apart.
constexpr uint64_t kWaitNs = 2000000000ull;  // bounded waits: 2 s

__device__ int g_umma_error;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Bounded wait for the barrier phase `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer();
    while (true) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar), "r"(parity)
            : "memory");
        if (ok) return true;
        if (globaltimer() - t0 > kWaitNs) return false;
    }
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
template <int SW>
__device__ __forceinline__ uint64_t sw_desc(uint32_t addr) {
    constexpr uint64_t kLayout = (SW == 128) ? 2ull : 4ull;  // 128-byte / 64-byte swizzle
    constexpr uint64_t kSbo = (8ull * SW) >> 4;              // 8-row atom stride
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (1ull << 16) | (kSbo << 32) | (1ull << 46) | (kLayout << 61);
}
template <int KIND>
__device__ __forceinline__ void mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    if constexpr (KIND == kTF32x3) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
            ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
            ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u));
    }
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ float tf32_hi(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Warps 0-3 accumulate and store the tile (warp w owns TMEM lanes / rows
// 32w..32w+31), warp 4 lane 0 issues TMA, warp 5 lane 0 issues tcgen05.mma.
// The tensor core's FP32 accumulation truncates, so the K loop is cut into
// groups of 128 K elements: each group accumulates in one of two TMEM
// buffers, and warps 0-3 add the finished buffer into FP32 registers (round to
// nearest) while the next group runs in the other buffer.
constexpr int kThreadsGemm = 192;
constexpr int kStagePitch = kTile + 4;  // epilogue staging pitch (floats): float4 rows without bank conflicts

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Epilogue of one warp: acc holds row `row0 + lane` of a TN-column output
// tile starting at column col0.  The 32 x TN block is staged in shared memory
// (sbuf, pitch TN + 4) and handled 128/TN output rows per step with TN/4 lanes
// per row, each on 4 columns, so every global load and store covers whole
// rows.  With cbuf (a second staging block), the warp's 32 Cin rows are
// fetched with asynchronous copies while the accumulator is staged, one round
// trip in all; without it they are loaded in batches.
template <int TN>
__device__ __forceinline__ void store_rows(const GemmOut& out, const float (&acc)[TN], float* sbuf, float* cbuf,
                                           long long row0, long long col0, int lane) {
    constexpr int kPitch = TN + 4;
    constexpr int kLanesRow = TN / 4;        // lanes per output row
    constexpr int kRowsStep = 32 / kLanesRow; // rows per step
    const int sub = lane / kLanesRow, cl = lane % kLanesRow;
    const long long gcol = col0 + 4 * cl;
    const bool prefetch = cbuf != nullptr && out.beta != 0.0f;
    if (prefetch) {
#pragma unroll 8
        for (int rr = sub; rr < 32; rr += kRowsStep)
            cp_async16(cbuf + rr * kPitch + 4 * cl, out.Cin + (row0 + rr) * out.ldcin + gcol);
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
#pragma unroll
    for (int c = 0; c < TN / 4; ++c)
        *reinterpret_cast<float4*>(sbuf + lane * kPitch + 4 * c) =
            make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
    if (prefetch) asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    constexpr int kBatch = 8;  // rows (per lane) whose Cin loads are in flight together
    for (int rb = 0; rb < 32 / kRowsStep; rb += kBatch) {
        float4 cin[kBatch];
        if (prefetch) {
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                cin[u] = *reinterpret_cast<const float4*>(cbuf + ((rb + u) * kRowsStep + sub) * kPitch + 4 * cl);
        } else if (out.beta != 0.0f) {
#pragma unroll
            for (int u = 0; u < kBatch; ++u)
                cin[u] = *reinterpret_cast<const float4*>(out.Cin + (row0 + (rb + u) * kRowsStep + sub) * out.ldcin + gcol);
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
            const int rr = (rb + u) * kRowsStep + sub;
            const long long grow = row0 + rr;
            float4* sp = reinterpret_cast<float4*>(sbuf + rr * kPitch + 4 * cl);
            const float4 a = *sp;
            float o[4] = {out.alpha * a.x, out.alpha * a.y, out.alpha * a.z, out.alpha * a.w};
            if (out.beta != 0.0f) {
                o[0] += out.beta * cin[u].x;
                o[1] += out.beta * cin[u].y;
                o[2] += out.beta * cin[u].z;
                o[3] += out.beta * cin[u].w;
            }
            const float4 ov = make_float4(o[0], o[1], o[2], o[3]);
            if (out.C) *reinterpret_cast<float4*>(out.C + grow * out.ldc + gcol) = ov;
            if (out.C_hi) {
                float h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    h[e] = tf32_hi(o[e]);
                    l[e] = o[e] - h[e];
                }
                *reinterpret_cast<float4*>(out.C_hi + grow * out.ld_split + gcol) = make_float4(h[0], h[1], h[2], h[3]);
                *reinterpret_cast<float4*>(out.C_lo + grow * out.ld_split + gcol) = make_float4(l[0], l[1], l[2], l[3]);
            }
            if (out.Ct || out.Ct_hi) *sp = ov;  // final values back for the transposed copy
        }
    }
    if (out.Ct || out.Ct_hi) {  // Ct[col][row]: lane = row again, 32 consecutive rows per store
        __syncwarp();
#pragma unroll 4
        for (int c = 0; c < TN / 4; ++c) {
            const float4 x = *reinterpret_cast<const float4*>(sbuf + lane * kPitch + 4 * c);
            const float v[4] = {x.x, x.y, x.z, x.w};
            const long long col = col0 + 4 * c;
            const long long row = row0 + lane;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const long long g = (col + e) * out.ldct + row;
                if (out.Ct) out.Ct[g] = v[e];
                if (out.Ct_hi) {
                    const float h = tf32_hi(v[e]);
                    out.Ct_hi[g] = h;
                    out.Ct_lo[g] = v[e] - h;
                }
            }
        }
    }
}

template <int KIND, int STAGES, int SW, int TN>
__global__ void __launch_bounds__(kThreadsGemm, 1)
gemm_nt_kernel(const __grid_constant__ CUtensorMap tA0, const __grid_constant__ CUtensorMap tA1,
               const __grid_constant__ CUtensorMap tB0, const __grid_constant__ CUtensorMap tB1, const int nk,
               const GemmOut out) {
    const int tm = blockIdx.y, tn = blockIdx.x;  // 128-row tile, TN-column tile
    if (out.lower_only && tn * TN / kTile > tm) return;  // 128 x 128 coverage of the lower triangle
    constexpr int kOps = (KIND == kTF32x3) ? 4 : 2;
    constexpr int kElems = SW / ((KIND == kTF32x3) ? 4 : 2);  // K elements per slice
    constexpr int kABytes = kTile * SW;                      // A operand slice (128 rows)
    constexpr int kBBytes = TN * SW;                         // B operand slice (TN rows)
    constexpr int kStageBytes = (kOps / 2) * (kABytes + kBBytes);
    constexpr int kSteps = SW / 32;                          // 32-byte MMA K steps per slice
    constexpr int kGroup = 128 / kElems * ((KIND == kTF32x3) ? 1 : 2);  // slices per promotion group
    constexpr uint32_t kFmt = (KIND == kTF32x3) ? 2u : 1u;
    constexpr uint32_t kIdesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((TN >> 3) << 17) | ((kTile >> 4) << 24);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * kStageBytes);
    uint64_t* empty = full + STAGES;
    uint64_t* accfull = empty + STAGES;   // [2] group finished in TMEM buffer b
    uint64_t* accempty = accfull + 2;     // [2] buffer b drained by warps 0-3
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // K slices [kc0, kc0 + nkr) of this tile row (all of them unless A is triangular)
    constexpr int kPerTile = kTile / kElems;
    int kc0 = 0, kc1 = nk;
    if (out.tri_a == 1) kc0 = min(nk, tm * kPerTile);
    else if (out.tri_a == 2) kc1 = min(nk, (tm + 1) * kPerTile);
    const int nkr = max(0, kc1 - kc0);
    const int ngroups = (nkr + kGroup - 1) / kGroup;

    if (threadIdx.x == 32 * 4) {  // the TMA thread: fetch the descriptors while the CTA sets up
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tA0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tB0)) : "memory");
        if constexpr (KIND == kTF32x3) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tA1)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tB1)) : "memory");
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&accfull[b]), 1);
            mbar_init(smem_u32(&accempty[b]), 4);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(2 * TN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *tmem_slot;
    // Everything above touched no global memory; the operands and outputs may
    // belong to the kernel before this one in the stream.
    pdl_wait();
    // stage layout: A hi, B hi, A lo, B lo (op 0..3)
    auto tile = [&](int s, int op) {
        return smem_u32(smem + s * kStageBytes + (op >> 1) * (kABytes + kBBytes) + (op & 1) * kABytes);
    };

    if (warp == 4) {
        if (lane == 0) {  // TMA producer
            int issued = 0;
            for (int kc = 0; kc < nkr; ++kc) {
                const int s = kc % STAGES;
                if (kc >= STAGES && !mbar_wait(smem_u32(&empty[s]), ((kc / STAGES) - 1) & 1)) {
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                const uint32_t bar = smem_u32(&full[s]);
                mbar_expect_tx(bar, kStageBytes);
                const int x = (kc0 + kc) * kElems;
                tma_load_2d(tile(s, 0), &tA0, x, tm * kTile, bar);
                tma_load_2d(tile(s, 1), &tB0, x, tn * TN, bar);
                if constexpr (KIND == kTF32x3) {
                    tma_load_2d(tile(s, 2), &tA1, x, tm * kTile, bar);
                    tma_load_2d(tile(s, 3), &tB1, x, tn * TN, bar);
                }
                issued = kc + 1;
            }
            // Bounded drain of loads still in flight after an abort.
            if (*abort_flag)
                for (int kc = std::max(0, issued - STAGES); kc < issued; ++kc)
                    mbar_wait(smem_u32(&full[kc % STAGES]), (kc / STAGES) & 1);
        }
        __syncwarp();
    } else if (warp == 5) {
        if (lane == 0) {  // MMA issuer
            bool ok = true;
            for (int g = 0; g < ngroups && ok; ++g) {
                const int b = g & 1;
                if (g >= 2 && !mbar_wait(smem_u32(&accempty[b]), ((g >> 1) - 1) & 1)) { ok = false; break; }
                fence_after();
                const uint32_t acc_t = tmem + static_cast<uint32_t>(b * TN);
                const int k_end = std::min(nkr, (g + 1) * kGroup);
                for (int kc = g * kGroup; kc < k_end; ++kc) {
                    const int s = kc % STAGES;
                    if (*abort_flag || !mbar_wait(smem_u32(&full[s]), (kc / STAGES) & 1)) { ok = false; break; }
                    fence_after();
                    const uint64_t a0 = sw_desc<SW>(tile(s, 0)), b0 = sw_desc<SW>(tile(s, 1));
#pragma unroll
                    for (int kk = 0; kk < kSteps; ++kk) {
                        const uint64_t adv = static_cast<uint64_t>(kk * 2);  // +32 bytes along K
                        const uint32_t acc = (kc != g * kGroup || kk) ? 1u : 0u;
                        if constexpr (KIND == kTF32x3) {
                            const uint64_t a1 = sw_desc<SW>(tile(s, 2)), b1 = sw_desc<SW>(tile(s, 3));
                            mma<KIND>(acc_t, a0 + adv, b1 + adv, kIdesc, acc);
                            mma<KIND>(acc_t, a1 + adv, b0 + adv, kIdesc, 1u);
                            mma<KIND>(acc_t, a0 + adv, b0 + adv, kIdesc, 1u);
                        } else {
                            mma<KIND>(acc_t, a0 + adv, b0 + adv, kIdesc, acc);
                        }
                    }
                    mma_commit(smem_u32(&empty[s]));
                }
                mma_commit(smem_u32(&accfull[b]));  // arrives when this group's MMAs are done
            }
            if (!ok) {
                *abort_flag = 1;
                // Release any accumulator waiters: commits arrive once issued MMAs complete.
                mma_commit(smem_u32(&accfull[0]));
                mma_commit(smem_u32(&accfull[1]));
            }
        }
        __syncwarp();
    } else {
        // Warps 0-3: promote each finished group into FP32 registers, then store.
        float acc[TN];
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int g = 0; g < ngroups; ++g) {
            const int b = g & 1;
            if (!mbar_wait(smem_u32(&accfull[b]), (g >> 1) & 1) || *abort_flag) { ok = false; break; }
            fence_after();
            const uint32_t base = tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(b * TN);
#pragma unroll
            for (int c = 0; c < TN / 32; ++c) {
                float v[32];
                tmem_ld32(base + static_cast<uint32_t>(c * 32), v);
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[c * 32 + j] = __fadd_rn(acc[c * 32 + j], v[j]);
            }
            fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&accempty[b])) : "memory");
        }
        if (!ok) {
            if (lane == 0) atomicExch(&g_umma_error, 1);
        } else {
            // All MMAs have completed, so the operand ring is free for staging.
            constexpr int kBlk = 32 * (TN + 4);  // one warp's staging block (floats)
            static_assert(4 * kBlk * 4 <= STAGES * kStageBytes, "epilogue staging exceeds the ring");
            // a second staging block for the Cin prefetch where the ring has room
            constexpr bool kCinBuf = 8 * kBlk * 4 <= STAGES * kStageBytes;
            float* sb = reinterpret_cast<float*>(smem);
            store_rows<TN>(out, acc, sb + warp * kBlk, kCinBuf ? sb + (4 + warp) * kBlk : nullptr,
                           static_cast<long long>(tm) * kTile + warp * 32, static_cast<long long>(tn) * TN, lane);
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * TN));
    }
}

// ---- CTA-pair variant (cta_group::2) for large FP32-accurate products --------
// Two CTAs of a cluster compute a 256 x NB tile (NB = 128 or 256) with one
// tcgen05.mma stream: each CTA holds its 128 rows of A and NB/2 of the NB B
// rows in its own shared memory, and its 128 x NB slice of the accumulator in
// its own TMEM.  Wider MMAs pay off: the per-instruction cost is measured at
// ~1.46x for N = 64 versus N = 128 (not 2x), so N = 256 per instruction does
// the same work in fewer, longer MMAs.  The even CTA (rank 0) issues the MMAs
// and owns the full and accumulator-empty barriers: both CTAs' TMA loads
// complete on its full barrier, its commits arrive on both CTAs' barriers,
// and both CTAs' epilogue warps arrive on its accumulator-empty barrier.
// Operand loads carry no multicast.  All waits are bounded; a CTA that gives
// up records the error and both CTAs still meet at the closing cluster barrier.
constexpr uint32_t kPeerMask = 0xFEFFFFFFu;  // shared address of the even CTA's copy
constexpr int kPairA = kTile * 128;           // 128 rows x 128 B

template <int KIND, int NB> struct Pair {
    static constexpr int kParts = (KIND == kTF32x3) ? 2 : 1; // hi/lo or the BF16 operand alone
    static constexpr int kB = (NB / 2) * 128;              // NB/2 rows x 128 B per CTA
    static constexpr int kStage = kParts * (kPairA + kB);
    static constexpr int kStages = (192 * 1024) / kStage;   // 3 or 4 (TF32x3), 6 or 8 (BF16)
    static constexpr int kEpiWarps = NB / 32;               // 4 warps per 128 columns
    static constexpr int kThreads = 32 * (kEpiWarps + 2);   // + TMA warp + MMA warp
    static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStage + 1024 + 256;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t even_bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(even_bar)
        : "memory");
}
template <int KIND>
__device__ __forceinline__ void mma_pair(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    if constexpr (KIND == kTF32x3) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
            ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u));
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
            ::"r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate), "r"(0u));
    }
}
__device__ __forceinline__ void commit_pair(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(bar), "h"(static_cast<uint16_t>(3))
        : "memory");
}

template <int KIND, int NB>
__global__ void __launch_bounds__(Pair<KIND, NB>::kThreads, 1)
gemm_nt_pair_kernel(const __grid_constant__ CUtensorMap tA0, const __grid_constant__ CUtensorMap tA1,
                    const __grid_constant__ CUtensorMap tB0, const __grid_constant__ CUtensorMap tB1, const int nk,
                    const GemmOut out) {
    using P = Pair<KIND, NB>;
    constexpr int kStages = P::kStages;
    constexpr int kEpi = P::kEpiWarps;
    const uint32_t rank = cluster_rank();
    const int tn = blockIdx.x >> 1, tm2 = blockIdx.y;  // NB-column tile, 256-row tile
    constexpr int kSub = NB / kTile;                    // 128-column sub-tiles per tile
    // lower_only: the pair skips together when every 128 x 128 sub-tile lies above the diagonal
    if (out.lower_only && tn * kSub > 2 * tm2 + 1) return;
    constexpr int kElems = (KIND == kTF32x3) ? 32 : 64;  // K elements per 128-byte slice
    constexpr int kGroup = 4;  // slices per promotion group (128 K elements TF32, 256 BF16)
    constexpr uint32_t kFmt = (KIND == kTF32x3) ? 2u : 1u;
    constexpr uint32_t kIdesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((NB >> 3) << 17) | ((2 * kTile >> 4) << 24);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * P::kStage);
    uint64_t* empty = full + kStages;
    uint64_t* accfull = empty + kStages;
    uint64_t* accempty = accfull + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accempty + 2);
    int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // K slices [kc0, kc0 + nkr): a triangular A restricts them to the union of the
    // pair's two 128-row tiles (the extra 128-block is a zero block next to the
    // triangle, written by the producer of A)
    int kc0 = 0, kc1 = nk;
    if (out.tri_a == 1) kc0 = min(nk, 2 * tm2 * (kTile / kElems));
    else if (out.tri_a == 2) kc1 = min(nk, (2 * tm2 + 2) * (kTile / kElems));
    const int nkr = max(0, kc1 - kc0);
    const int ngroups = (nkr + kGroup - 1) / kGroup;

    if (threadIdx.x == 32 * kEpi) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tA0)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tB0)) : "memory");
        if constexpr (KIND == kTF32x3) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tA1)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tB1)) : "memory");
        }
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(smem_u32(&full[s]), 1);
            mbar_init(smem_u32(&empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&accfull[b]), 1);
            mbar_init(smem_u32(&accempty[b]), 2 * kEpi);  // the epilogue warps of both CTAs
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(tmem_slot)), "r"(2 * NB));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    fence_before();
    cluster_sync_all();  // both CTAs' barriers initialised and TMEM allocated
    fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    auto a_tile = [&](int s, int lo) { return smem_u32(smem + s * P::kStage + lo * kPairA); };
    auto b_tile = [&](int s, int lo) { return smem_u32(smem + s * P::kStage + P::kParts * kPairA + lo * P::kB); };

    if (warp == kEpi) {
        if (lane == 0) {  // TMA producer, both CTAs
            const int arow = tm2 * 2 * kTile + static_cast<int>(rank) * kTile;
            const int brow = tn * NB + static_cast<int>(rank) * (NB / 2);
            int issued = 0;
            for (int kc = 0; kc < nkr; ++kc) {
                const int s = kc % kStages;
                if (kc >= kStages && !mbar_wait(smem_u32(&empty[s]), ((kc / kStages) - 1) & 1)) {
                    *abort_flag = 1;
                    break;
                }
                if (*abort_flag) break;
                const uint32_t even_full = smem_u32(&full[s]) & kPeerMask;
                if (rank == 0) mbar_expect_tx(smem_u32(&full[s]), 2 * P::kStage);
                const int x = (kc0 + kc) * kElems;
                tma_load_2d_pair(a_tile(s, 0), &tA0, x, arow, even_full);
                tma_load_2d_pair(b_tile(s, 0), &tB0, x, brow, even_full);
                if constexpr (KIND == kTF32x3) {
                    tma_load_2d_pair(a_tile(s, 1), &tA1, x, arow, even_full);
                    tma_load_2d_pair(b_tile(s, 1), &tB1, x, brow, even_full);
                }
                issued = kc + 1;
            }
            // Bounded drain after an abort: the even CTA's full barrier counts both CTAs' loads.
            if (*abort_flag && rank == 0)
                for (int kc = std::max(0, issued - kStages); kc < issued; ++kc)
                    mbar_wait(smem_u32(&full[kc % kStages]), (kc / kStages) & 1);
        }
        __syncwarp();
    } else if (warp == kEpi + 1) {
        if (lane == 0 && rank == 0) {  // MMA issuer, even CTA only
            bool ok = true;
            for (int g = 0; g < ngroups && ok; ++g) {
                const int b = g & 1;
                if (g >= 2 && !mbar_wait(smem_u32(&accempty[b]), ((g >> 1) - 1) & 1)) { ok = false; break; }
                fence_after();
                const uint32_t acc_t = tmem + static_cast<uint32_t>(b * NB);
                const int k_end = std::min(nkr, (g + 1) * kGroup);
                for (int kc = g * kGroup; kc < k_end; ++kc) {
                    const int s = kc % kStages;
                    if (*abort_flag || !mbar_wait(smem_u32(&full[s]), (kc / kStages) & 1)) { ok = false; break; }
                    fence_after();
                    const uint64_t a0 = sw_desc<128>(a_tile(s, 0)), b0 = sw_desc<128>(b_tile(s, 0));
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t adv = static_cast<uint64_t>(kk * 2);  // +32 bytes along K
                        const uint32_t acc = (kc != g * kGroup || kk) ? 1u : 0u;
                        if constexpr (KIND == kTF32x3) {
                            const uint64_t a1 = sw_desc<128>(a_tile(s, 1)), b1 = sw_desc<128>(b_tile(s, 1));
                            mma_pair<KIND>(acc_t, a0 + adv, b1 + adv, kIdesc, acc);
                            mma_pair<KIND>(acc_t, a1 + adv, b0 + adv, kIdesc, 1u);
                            mma_pair<KIND>(acc_t, a0 + adv, b0 + adv, kIdesc, 1u);
                        } else {
                            mma_pair<KIND>(acc_t, a0 + adv, b0 + adv, kIdesc, acc);
                        }
                    }
                    commit_pair(smem_u32(&empty[s]));  // frees stage s in both CTAs
                }
                commit_pair(smem_u32(&accfull[b]));
            }
            if (!ok) {
                *abort_flag = 1;
                commit_pair(smem_u32(&accfull[0]));
                commit_pair(smem_u32(&accfull[1]));
            }
        }
        __syncwarp();
    } else {
        // Epilogue warps of both CTAs: warp e reads TMEM lanes 32 (e % 4).. and
        // the 128 accumulator columns 128 (e / 4)..; promotes each finished group.
        const int quad = warp & 3, half = warp >> 2;
        float acc[kTile];
#pragma unroll
        for (int j = 0; j < kTile; ++j) acc[j] = 0.0f;
        bool ok = true;
        for (int g = 0; g < ngroups; ++g) {
            const int b = g & 1;
            if (!mbar_wait(smem_u32(&accfull[b]), (g >> 1) & 1) || *abort_flag) { ok = false; break; }
            fence_after();
            const uint32_t base = tmem + (static_cast<uint32_t>(quad * 32) << 16) +
                                  static_cast<uint32_t>(b * NB + half * kTile);
#pragma unroll
            for (int c = 0; c < kTile / 32; ++c) {
                float v[32];
                tmem_ld32(base + static_cast<uint32_t>(c * 32), v);
#pragma unroll
                for (int j = 0; j < 32; ++j) acc[c * 32 + j] = __fadd_rn(acc[c * 32 + j], v[j]);
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(smem_u32(&accempty[b]) & kPeerMask)
                             : "memory");
        }
        const int sub_col = tn * kSub + half;                    // 128-column sub-tile of this warp
        const int sub_row = 2 * tm2 + static_cast<int>(rank);    // 128-row tile of this CTA
        if (!ok) {
            if (lane == 0) atomicExch(&g_umma_error, 1);
        } else if (!(out.lower_only && sub_col > sub_row)) {
            static_assert(kEpi * 32 * kStagePitch * 4 <= kStages * P::kStage, "epilogue staging exceeds the ring");
            store_rows<kTile>(out, acc, reinterpret_cast<float*>(smem) + warp * 32 * kStagePitch, nullptr,
                       static_cast<long long>(sub_row) * kTile + quad * 32, static_cast<long long>(sub_col) * kTile,
                       lane);
        }
    }
    fence_before();
    cluster_sync_all();  // every MMA of the pair is complete and both epilogues are done
    if (warp == 0) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NB));
    }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
    static EncodeFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeFn>(p);
    }();
    return fn;
}

// Row-major [rows, k] operand, 128-row x sw-byte boxes with the sw-byte swizzle.
int make_map(CUtensorMap* map, const void* base, bool bf16, long long rows, long long k, long long ld, int sw,
             int box_rows = kTile) {
    EncodeFn enc = encode_fn();
    if (!enc) return fail(TB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const int esize = bf16 ? 2 : 4;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * esize};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(sw / esize), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     sw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(TB_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return TB_OK;
}

template <int KIND, int STAGES, int SW, int TN>
int launch(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0, const CUtensorMap& b1, int M, int N,
           int nk, const GemmOut& out, cudaStream_t st) {
    constexpr int kOps = (KIND == kTF32x3) ? 4 : 2;
    const size_t smem = static_cast<size_t>(STAGES) * (kOps / 2) * (kTile + TN) * SW + 1024 + 256;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [&] {
        attr = cudaFuncSetAttribute(gemm_nt_kernel<KIND, STAGES, SW, TN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem));
    });
    if (attr != cudaSuccess) return cuda_fail(attr, "cudaFuncSetAttribute(gemm_nt_kernel)");
    const cudaError_t e = launch_pdl(gemm_nt_kernel<KIND, STAGES, SW, TN>, dim3(N / TN, M / kTile),
                                     dim3(kThreadsGemm), smem, st, a0, a1, b0, b1, nk, out);
    return e == cudaSuccess ? check_launch("gemm_nt_kernel") : cuda_fail(e, "gemm_nt_kernel launch");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launches the CTA-pair kernel: clusters of two along x, programmatic
// serialization as for the single-CTA kernel.
template <int KIND, int NB>
int launch_pair(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0, const CUtensorMap& b1, int M,
                int N, int nk, const GemmOut& out, cudaStream_t st) {
    using P = Pair<KIND, NB>;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [&] {
        attr = cudaFuncSetAttribute(gemm_nt_pair_kernel<KIND, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(P::kSmem));
    });
    if (attr != cudaSuccess) return cuda_fail(attr, "cudaFuncSetAttribute(gemm_nt_pair_kernel)");
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * (N / NB), M / (2 * kTile));
    cfg.blockDim = dim3(P::kThreads);
    cfg.dynamicSmemBytes = P::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = pdl_allowed(st) ? 1 : 0;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_nt_pair_kernel<KIND, NB>, a0, a1, b0, b1, nk, out);
    return e == cudaSuccess ? check_launch("gemm_nt_pair_kernel") : cuda_fail(e, "gemm_nt_pair_kernel launch");
}

}  // namespace

int gemm_nt(Kind kind, const Operand& A, const Operand& B, int M, int N, int K, const GemmOut& out,
            cudaStream_t stream) {
    const int kstep = kind == kTF32x3 ? 32 : 64;
    if (M <= 0 || N <= 0 || K <= 0 || M % kTile || N % kTile || K % kstep)
        return fail(TB_ERR_SHAPE, "gemm_nt: M=%d N=%d K=%d must be multiples of 128/128/%d", M, N, K, kstep);
    const int esize = kind == kTF32x3 ? 4 : 2;
    if (!A.hi || !B.hi || (kind == kTF32x3 && (!A.lo || !B.lo)) || !aligned16(A.hi) || !aligned16(B.hi) ||
        (kind == kTF32x3 && (!aligned16(A.lo) || !aligned16(B.lo))) || (A.ld * esize) % 16 || (B.ld * esize) % 16 ||
        A.ld < K || B.ld < K)
        return fail(TB_ERR_ARG, "gemm_nt: operands must be non-null, 16-byte aligned, ld >= K, ld*elem % 16 == 0");
    if ((out.C && (!aligned16(out.C) || out.ldc % 4 || out.ldc < N)) ||
        (out.beta != 0.0f && (!out.Cin || !aligned16(out.Cin) || out.ldcin % 4 || out.ldcin < N)) ||
        (out.C_hi && (!out.C_lo || !aligned16(out.C_hi) || !aligned16(out.C_lo) || out.ld_split % 4 || out.ld_split < N)) ||
        ((out.Ct || out.Ct_hi) && out.ldct < M) || (!out.Ct_hi != !out.Ct_lo))
        return fail(TB_ERR_ARG, "gemm_nt: output pointers must be 16-byte aligned with ld >= N and ld % 4 == 0");
    if (out.tri_a && (out.tri_a > 2 || M != K))
        return fail(TB_ERR_ARG, "gemm_nt: a triangular A must be square (M == K)");
    const bool bf16 = kind == kBF16;
    CUtensorMap a0{}, a1{}, b0{}, b1{};
    // 128-byte slices: three stages for TF32x3, four for BF16.  (64-byte slices
    // with six stages were measured slower: 176 vs 211 TFLOP/s at 4096^3.)
    const int sw = 128;
    // Large products on CTA pairs (256-row tiles).  With a
    // triangular A the pair runs over the union of its two row tiles' K ranges,
    // one 128-block past the triangle, which the caller keeps zero.
    if (M % (2 * kTile) == 0 && K >= 512) {
        CUtensorMap pa0{}, pa1{}, pb0{}, pb1{};
        const int nb = (N % 256 == 0) ? 256 : 128;  // 256-wide MMAs where N allows
        int rc = make_map(&pa0, A.hi, bf16, M, K, A.ld, sw);
        if (!rc) rc = make_map(&pb0, B.hi, bf16, N, K, B.ld, sw, nb / 2);
        if (!rc && !bf16) rc = make_map(&pa1, A.lo, false, M, K, A.ld, sw);
        if (!rc && !bf16) rc = make_map(&pb1, B.lo, false, N, K, B.ld, sw, nb / 2);
        if (rc) return rc;
        if (bf16) { pa1 = pa0; pb1 = pb0; }
        const int nk2 = K / (bf16 ? 64 : 32);
        if (bf16)
            return nb == 256 ? launch_pair<kBF16, 256>(pa0, pa1, pb0, pb1, M, N, nk2, out, stream)
                             : launch_pair<kBF16, 128>(pa0, pa1, pb0, pb1, M, N, nk2, out, stream);
        return nb == 256 ? launch_pair<kTF32x3, 256>(pa0, pa1, pb0, pb1, M, N, nk2, out, stream)
                         : launch_pair<kTF32x3, 128>(pa0, pa1, pb0, pb1, M, N, nk2, out, stream);
    }
    // Products that fill less than one wave of 128 x 128 tiles are latency-bound
    // (one SM writes a whole tile): 128 x 64 tiles halve each CTA's output and
    // hold four K-slices in flight.
    const bool narrow = !bf16 && (static_cast<long long>(M / kTile) * (N / kTile) < 148);
    const int tn_rows = narrow ? kTile / 2 : kTile;
    int rc = make_map(&a0, A.hi, bf16, M, K, A.ld, sw);
    if (!rc) rc = make_map(&b0, B.hi, bf16, N, K, B.ld, sw, tn_rows);
    if (!rc && !bf16) rc = make_map(&a1, A.lo, false, M, K, A.ld, sw);
    if (!rc && !bf16) rc = make_map(&b1, B.lo, false, N, K, B.ld, sw, tn_rows);
    if (rc) return rc;
    if (bf16) { a1 = a0; b1 = b0; }
    const int nk = K / (sw / (bf16 ? 2 : 4));
    if (bf16) return launch<kBF16, 4, 128, 128>(a0, a1, b0, b1, M, N, nk, out, stream);
    return narrow ? launch<kTF32x3, 4, 128, 64>(a0, a1, b0, b1, M, N, nk, out, stream)
                  : launch<kTF32x3, 3, 128, 128>(a0, a1, b0, b1, M, N, nk, out, stream);
}

int gemm_take_error(cudaStream_t stream) {
    int h = 0, zero = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&h, g_umma_error, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(g_umma_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return -1;
    return h;
}

}  // namespace umma
}  // namespace tb

// ---- C ABI --------------------------------------------------------------------
namespace tb {
namespace {
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        uint32_t r;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
        const float h = __uint_as_float(r);
        hi[i] = h;
        lo[i] = v - h;
    }
}
}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_split_tf32(const float* x, float* hi, float* lo, size_t n, void* stream) {
    if (n == 0) return TB_OK;
    if (!x || !hi || !lo) return fail(TB_ERR_ARG, "tb_split_tf32: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((n + 255) / 256, 148u * 32u));
    split_tf32_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, hi, lo, n);
    return check_launch("split_tf32_kernel");
}

extern "C" int tb_gemm_nt_tf32x3(const float* a_hi, const float* a_lo, long long lda, const float* b_hi,
                                 const float* b_lo, long long ldb, int M, int N, int K, float alpha, float beta,
                                 const float* c_in, long long ldcin, float* c, long long ldc, int lower_only,
                                 void* stream) {
    pdl_fence(static_cast<cudaStream_t>(stream));  // the caller may have queued a cross-stream wait
    int rc = require_device(nullptr);
    if (rc) return rc;
    umma::GemmOut o{};
    o.C = c;
    o.ldc = ldc;
    o.Cin = c_in;
    o.ldcin = ldcin;
    o.alpha = alpha;
    o.beta = beta;
    o.lower_only = lower_only;
    return umma::gemm_nt(umma::kTF32x3, {a_hi, a_lo, lda}, {b_hi, b_lo, ldb}, M, N, K, o,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int tb_gemm_nt_bf16(const void* a, long long lda, const void* b, long long ldb, int M, int N, int K,
                               float alpha, float beta, const float* c_in, long long ldcin, float* c, long long ldc,
                               int lower_only, void* stream) {
    pdl_fence(static_cast<cudaStream_t>(stream));  // the caller may have queued a cross-stream wait
    int rc = require_device(nullptr);
    if (rc) return rc;
    umma::GemmOut o{};
    o.C = c;
    o.ldc = ldc;
    o.Cin = c_in;
    o.ldcin = ldcin;
    o.alpha = alpha;
    o.beta = beta;
    o.lower_only = lower_only;
    return umma::gemm_nt(umma::kBF16, {a, nullptr, lda}, {b, nullptr, ldb}, M, N, K, o,
                         static_cast<cudaStream_t>(stream));
}

extern "C" int tb_gemm_status(void* stream) {
    int rc = require_device(nullptr);
    if (rc) return rc;
    const int e = umma::gemm_take_error(static_cast<cudaStream_t>(stream));
    if (e < 0) return fail(TB_ERR_CUDA, "reading the GEMM status failed");
    return e ? fail(TB_ERR_TIMEOUT, "a tcgen05 GEMM pipeline wait expired") : TB_OK;
}

// Exact OBS pruning of one weight matrix against calibration activations, in
// the column-block ("SparseGPT") formulation, for which the reference has no
// implementation (docs/EHAP.md:248-250).  It keeps
// the reference's OBS saliency w^2 / [H^-1]_qq and update
// w -= (w_q / [H^-1]_qq) [H^-1]_{q,:} (ehap.hpp:683-691), taken along the
// Cholesky factor of H^-1 so that each pruned column is eliminated once.
//
//   1. H = X^T X / n over n calibration tokens (BF16 tcgen05, lower tiles).
//   2. lambda = frac * mean(diag H); H += lambda I.
//   3. U = chol_upper(H^-1) without forming H^-1: with P the index reversal,
//      chol_lower(P H P) = L gives H^-1 = (P L^-1 P)^T (P L^-1 P), so
//      U = P L^-1 P.  L comes from a recursive Cholesky whose panel solve is a
//      recursive triangular solve (only 128 x 128 diagonal blocks are inverted,
//      so the factorisation keeps the stability of a triangular solve even when
//      H is rank-deficient plus lambda I), then L^-1 from a recursive
//      triangular inverse; all off-diagonal work is FP32-accurate (3xTF32)
//      tcgen05 GEMMs, the 128 x 128 diagonal blocks are factored in shared
//      memory.
//   4. Column blocks of 128: per row (one warp per row, rows independent), for
//      each group of M columns prune the M-N smallest w^2 / U_qq^2 (lowest index
//      on ties), then for each column q: err = (w_q - kept_q) / U_qq,
//      w_j -= err U_qj (j >= q in the block); the block's errors E then update
//      the remaining columns lazily, W[:, i2:] -= E U[i1:i2, i2:], a tcgen05
//      GEMM.
// All FP32; executed FLOPs are counted by bench.obs_flops (lower-tile XtX,
// the recursions' GEMMs on dense tiles, the in-block and lazy updates).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "tb_device.cuh"
#include "tb_pdl.cuh"
#include "tb_runtime.h"
#include "tb_umma.cuh"

namespace tb {

namespace {

constexpr int kB = 128;  // diagonal / column block

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// diag sum of the lower-tile H (one block reduction, deterministic order per block).
__global__ void diag_sum_kernel(const float* __restrict__ H, int d, double* __restrict__ out) {
    __shared__ double part[1024];
    pdl_wait();
    double s = 0.0;
    for (int i = threadIdx.x; i < d; i += blockDim.x) s += static_cast<double>(H[static_cast<size_t>(i) * d + i]);
    part[threadIdx.x] = s;
    __syncthreads();
    for (int off = blockDim.x / 2; off; off >>= 1) {
        if (threadIdx.x < off) part[threadIdx.x] += part[threadIdx.x + off];
        __syncthreads();
    }
    if (threadIdx.x == 0) *out = part[0];
}

// A = P (H + lambda I) P on the lower triangle, plus its tf32 hi/lo split:
// A[i][j] = H[d-1-j][d-1-i] (j <= i), read from H's lower tiles through a
// 32 x 32 shared-memory transpose so that both the reads and the writes are
// coalesced.  Tiles above the diagonal 128-blocks are never read and are not
// written; inside a diagonal 128-block the upper part is written as zero.
__global__ void __launch_bounds__(256) reverse_damp_kernel(const float* __restrict__ H, int d,
                                                           const double* __restrict__ diag_sum, float frac,
                                                           float* __restrict__ A, float* __restrict__ A_hi,
                                                           float* __restrict__ A_lo) {
    __shared__ float tile[32][33];
    const int I = blockIdx.y, J = blockIdx.x;  // output tile: rows 32I.., columns 32J..
    pdl_wait();
    if (J > I && (J >> 2) != (I >> 2)) return;
    const float lambda = static_cast<float>(frac * (*diag_sum / d));
    const int tx = threadIdx.x, ty = threadIdx.y;
    if (J <= I) {
        const int sr0 = d - 32 * (J + 1), sc0 = d - 32 * (I + 1);  // source rows d-1-j, columns d-1-i
        for (int k = ty; k < 32; k += 8) tile[k][tx] = H[static_cast<size_t>(sr0 + k) * d + sc0 + tx];
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {
        const int i = 32 * I + k, j = 32 * J + tx;
        float v = 0.0f;
        if (j <= i) {
            v = tile[31 - tx][31 - k];
            if (i == j) v += lambda;
        }
        const size_t g = static_cast<size_t>(i) * d + j;
        const float h = tf32_round(v);
        A[g] = v;
        A_hi[g] = h;
        A_lo[g] = v - h;
    }
}

constexpr unsigned kFull = 0xFFFFFFFFu;
constexpr int kP = kB + 4;           // shared-memory pitch of the 128 x 128 blocks (16-byte rows)
constexpr int kBaseThreads = 512;
constexpr int kSP = 36;              // pitch of the 32 x 32 scratch blocks

// ---- 32 x 32 diagonal step of the base kernel, three roles in parallel ----
// Warp 0 factors the diagonal block column by column, lane i holding row i in
// registers relative to a base column (a[k] = D[i][jb+k], shifted by four every
// four columns, so the loop stays rolled with constant register indices).
// After column j it publishes the column (Lc[j][k] = L[j+k][j]) and 1/L_jj in
// shared memory and bumps a counter.  Warp 1 builds L_kk^-1 and warps 2.. solve
// the panel rows below (x L_kk^T = a) by forward substitution, each consuming
// the published columns one step behind, so neither sits on the critical path.
// Columns are read back as eight 128-bit broadcast loads instead of 31 shuffles.
// Waits are bounded: on expiry *bad gets 2 and the warp carries on (the host
// reports a timeout).
constexpr int kSpinLimit = 1 << 22;

__device__ __forceinline__ void wait_columns(const volatile int* ready, int target, int* bad) {
    int spins = 0;
    while (*ready < target) {
        if (++spins > kSpinLimit) {
            atomicExch(bad, 2);
            break;
        }
    }
    __threadfence_block();
}

__device__ __forceinline__ void load_column(const float* Lc, int j, float (&lc)[32]) {
    const float4* p = reinterpret_cast<const float4*>(Lc + j * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 v = p[q];
        lc[4 * q] = v.x; lc[4 * q + 1] = v.y; lc[4 * q + 2] = v.z; lc[4 * q + 3] = v.w;
    }
}

__device__ __forceinline__ void shift4(float (&a)[32]) {
#pragma unroll
    for (int k = 0; k < 28; ++k) a[k] = a[k + 4];
    a[28] = a[29] = a[30] = a[31] = 0.0f;
}

// Warp 0: factor D (pitch kP, Schur-updated, lower part valid) in place.
// Columns are published four at a time (one fence and one counter update per
// group); the column each lane needs for the next pivot comes from its own
// register, so the shared-memory round trip feeds only the other updates.
__device__ __noinline__ void diag_factor(float* D, float* Lc, float* rinv, volatile int* ready, int count0, int lane,
                                         int* bad) {
    float a[32];
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
        const float4 v = *reinterpret_cast<const float4*>(D + lane * kP + k);
        a[k] = (k <= lane) ? v.x : 0.0f;
        a[k + 1] = (k + 1 <= lane) ? v.y : 0.0f;
        a[k + 2] = (k + 2 <= lane) ? v.z : 0.0f;
        a[k + 3] = (k + 3 <= lane) ? v.w : 0.0f;
    }
    bool all_ok = true;
    float my_r = 1.0f;
    float piv = a[0];  // the next pivot, meaningful on the lane of the next column
#pragma unroll 1
    for (int jb = 0; jb < 32; jb += 4) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = jb + jj;
            const float djj = __shfl_sync(kFull, piv, j);
            const bool ok = djj > 0.0f;
            all_ok = all_ok && ok;
            const float rj = ok ? rsqrtf(djj) : 1.0f;
            // Lanes above the diagonal (lane < j) compute garbage from here on, without
            // predicates; their entries are never published nor written back.
            const float l = (lane == j) ? (ok ? djj * rj : 1.0f) : a[jj] * rj;
            a[jj] = l;
            if (lane == j) my_r = rj;
            piv = fmaf(-l, l, a[jj + 1]);  // on lane j + 1: its pivot, ahead of the column's update
            if (lane >= j) Lc[j * 32 + (lane - j)] = l;
            __syncwarp();
            float lc[32];
            load_column(Lc, j, lc);
#pragma unroll
            for (int k = 1; k < 32 - jj; ++k) a[jj + k] = fmaf(-l, lc[k], a[jj + k]);
        }
        // columns jb..jb+3 are final: L into D (zeros above), 1/L_jj, then publish
        *reinterpret_cast<float4*>(D + lane * kP + jb) =
            make_float4(lane >= jb ? a[0] : 0.0f, lane >= jb + 1 ? a[1] : 0.0f, lane >= jb + 2 ? a[2] : 0.0f,
                        lane >= jb + 3 ? a[3] : 0.0f);
        if (lane >= jb && lane < jb + 4) rinv[lane] = my_r;
        __threadfence_block();
        __syncwarp();
        if (lane == 0) *ready = count0 + jb + 4;
        shift4(a);
    }
    if (!all_ok && lane == 0) atomicExch(bad, 1);
}

// Warp 1: column c = lane of L_kk^-1 by forward elimination of L x = e_c,
// written to Q (rows) and QT (transposed), both pitch kP.
__device__ __noinline__ void diag_inverse(const float* Lc, const float* rinv, const volatile int* ready, int count0,
                                          float* Q, float* QT, int lane, int* bad) {
    float x[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) x[k] = (k == lane) ? 1.0f : 0.0f;
#pragma unroll 1
    for (int jb = 0; jb < 32; jb += 4) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = jb + jj;
            if (jj == 0) wait_columns(ready, count0 + jb + 4, bad);
            const float xj = x[jj] * rinv[j];
            Q[j * kP + lane] = xj;
            QT[lane * kP + j] = xj;
            float lc[32];
            load_column(Lc, j, lc);
#pragma unroll
            for (int k = 1; k < 32 - jj; ++k) x[jj + k] = fmaf(-xj, lc[k], x[jj + k]);
        }
        shift4(x);
    }
}

// Warps 2..: one panel row per lane, x L_kk^T = a by forward substitution, in
// place in the row (pitch kP, 16-byte aligned).
__device__ __noinline__ void diag_panel(float* row, const float* Lc, const float* rinv, const volatile int* ready,
                                        int count0, int* bad) {
    float a[32];
#pragma unroll
    for (int k = 0; k < 32; k += 4) {
        const float4 v = *reinterpret_cast<const float4*>(row + k);
        a[k] = v.x; a[k + 1] = v.y; a[k + 2] = v.z; a[k + 3] = v.w;
    }
#pragma unroll 1
    for (int jb = 0; jb < 32; jb += 4) {
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = jb + jj;
            if (jj == 0) wait_columns(ready, count0 + jb + 4, bad);
            const float x = a[jj] * rinv[j];
            row[j] = x;
            float lc[32];
            load_column(Lc, j, lc);
#pragma unroll
            for (int k = 1; k < 32 - jj; ++k) a[jj + k] = fmaf(-x, lc[k], a[jj + k]);
        }
        shift4(a);
    }
}

// Four rows by one column of a row-by-row product: acc[r] = sum_{k<K}
// X[r*px + k] Y[k], with 128-bit shared-memory loads (X broadcast across the
// warp, Y one row per lane); K is a multiple of 4 and the rows 16-byte aligned.
__device__ __forceinline__ void dot4x1(const float* X, int px, const float* Y, int K, float (&acc)[4]) {
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[r] = 0.0f;
#pragma unroll 2
    for (int k = 0; k < K; k += 4) {
        const float4 y = *reinterpret_cast<const float4*>(Y + k);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float4 x = *reinterpret_cast<const float4*>(X + r * px + k);
            acc[r] = fmaf(x.x, y.x, acc[r]);
            acc[r] = fmaf(x.y, y.y, acc[r]);
            acc[r] = fmaf(x.z, y.z, acc[r]);
            acc[r] = fmaf(x.w, y.w, acc[r]);
        }
    }
}

constexpr int kBaseWarps = kBaseThreads / 32;
constexpr int kIdle0 = 5;  // first warp free during a diagonal step (0: factor, 1: inverse, 2-4: panel)

// Block row ib of V = L^-1 is V_ij = -V_ii S_j with S_j = sum_{m=j}^{i-1} L_im V_mj
// (j < i), in 32-blocks.  v_row_s forms S_j^T (from L's row block ib and V^T's
// rows of the final block rows < ib) into sST; v_row_finish forms V_ij and its
// transpose once V_ii exists.  Work is split over nw warps, four rows each.
__device__ __forceinline__ void v_row_s(const float* sA, const float* sVT, float* sST, int ib, int iw, int nw,
                                        int lane) {
#pragma unroll 1
    for (int task = iw; task < ib * 8; task += nw) {
        const int jb = task >> 3, i = 4 * (task & 7);
        float acc[4];
        dot4x1(sA + (32 * ib + i) * kP + 32 * jb, kP, sVT + (32 * jb + lane) * kP + 32 * jb, 32 * (ib - jb), acc);
        *reinterpret_cast<float4*>(sST + (jb * 32 + lane) * kSP + i) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    }
}
__device__ __forceinline__ void v_row_finish(float* sV, float* sVT, const float* sST, int ib, int iw, int nw,
                                             int lane) {
#pragma unroll 1
    for (int task = iw; task < ib * 8; task += nw) {
        const int jb = task >> 3, i = 4 * (task & 7);
        float acc[4];
        dot4x1(sV + (32 * ib + i) * kP + 32 * ib, kP, sST + (jb * 32 + lane) * kSP, 32, acc);
#pragma unroll
        for (int r = 0; r < 4; ++r) sV[(32 * ib + i + r) * kP + 32 * jb + lane] = -acc[r];
        *reinterpret_cast<float4*>(sVT + (32 * jb + lane) * kP + 32 * ib + i) =
            make_float4(-acc[0], -acc[1], -acc[2], -acc[3]);
    }
}

// Cholesky and inverse of one 128 x 128 diagonal block in shared memory,
// blocked by 32: per 32-column step, the diagonal block is factored and
// inverted by one warp (diag32), the panel below is L_ik = A_ik L_kk^-T and
// the trailing lower blocks take the Schur update; then the off-diagonal
// blocks of V = L^-1 are V_ij = -V_ii sum_{k=j}^{i-1} L_ik V_kj, formed by
// the warps a diagonal step leaves idle (block row i's sum during step i, its
// product with V_ii during step i+1; the last row after the loop).  Every
// product is written as rows times rows (V^T and S^T are kept for that), each
// thread computing four rows of one column.
// Writes the tf32 split of V (zeros above the diagonal) and of V^T (zeros
// below), all over the full 128 x 128 block; V itself is V_hi + V_lo exactly.
__global__ void __launch_bounds__(kBaseThreads) base_chol_inv_kernel(const float* __restrict__ A,
                                                                     float* __restrict__ V_hi,
                                                                     float* __restrict__ V_lo,
                                                                     float* __restrict__ VT_hi,
                                                                     float* __restrict__ VT_lo, int ld, int off,
                                                                     int* __restrict__ bad) {
    extern __shared__ __align__(16) float sm[];
    float* sA = sm;                 // 128 x kP: A -> L
    float* sV = sA + kB * kP;       // 128 x kP: V = L^-1
    float* sVT = sV + kB * kP;      // 128 x kP: V^T
    float* sST = sVT + kB * kP;     // 3 x 32 x kSP: S^T blocks
    float* sLc = sST + 3 * 32 * kSP;  // 32 x 32: published columns of the current diagonal block
    float* sRinv = sLc + 32 * 32;     // 32: 1 / L_jj
    int* sReady = reinterpret_cast<int*>(sRinv + 32);  // columns published so far (all steps)
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const size_t base = static_cast<size_t>(off) * ld + off;
    pdl_wait();
    if (t == 0) *sReady = 0;
    {  // the lower triangle of the block, eight 16-byte loads in flight per thread
        constexpr int kChunks = kB * kB / 4 / kBaseThreads;
        float4 v[kChunks];
#pragma unroll
        for (int u = 0; u < kChunks; ++u) {
            const int c = t + u * kBaseThreads, i = c >> 5, j0 = 4 * (c & 31);
            v[u] = j0 <= i ? *reinterpret_cast<const float4*>(A + base + static_cast<size_t>(i) * ld + j0)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
        for (int u = 0; u < kChunks; ++u) {
            const int c = t + u * kBaseThreads, i = c >> 5, j0 = 4 * (c & 31);
            float4 x = v[u];
            if (j0 + 1 > i) x.y = 0.0f;
            if (j0 + 2 > i) x.z = 0.0f;
            if (j0 + 3 > i) x.w = 0.0f;
            *reinterpret_cast<float4*>(sA + i * kP + j0) = x;
            *reinterpret_cast<float4*>(sV + i * kP + j0) = z;
            *reinterpret_cast<float4*>(sVT + i * kP + j0) = z;
        }
    }
    __syncthreads();
#pragma unroll 1
    for (int kb = 0; kb < 4; ++kb) {
        const int o = 32 * kb;
        const int prow = kB - o - 32;  // panel rows below the diagonal block
        volatile int* ready = sReady;
        if (warp == 0) {
            diag_factor(sA + o * kP + o, sLc, sRinv, ready, 32 * kb, lane, bad);
        } else if (warp == 1) {
            diag_inverse(sLc, sRinv, ready, 32 * kb, sV + o * kP + o, sVT + o * kP + o, lane, bad);
        } else if (warp - 2 < prow / 32) {
            diag_panel(sA + (o + 32 + 32 * (warp - 2) + lane) * kP + o, sLc, sRinv, ready, 32 * kb, bad);
        } else if (warp >= kIdle0) {
            // Warps 5..15 are otherwise idle during the diagonal step: they finish
            // block row kb-1 of V (its diagonal inverse came from the previous
            // step) and then form S for block row kb (rows < kb of V are final).
            const int iw = warp - kIdle0;
            if (kb >= 2) v_row_finish(sV, sVT, sST, kb - 1, iw, kBaseWarps - kIdle0, lane);
            asm volatile("bar.sync 1, %0;" ::"r"(32 * (kBaseWarps - kIdle0)) : "memory");
            if (kb >= 1) v_row_s(sA, sVT, sST, kb, iw, kBaseWarps - kIdle0, lane);
        }
        __syncthreads();
        if (prow == 0) break;
        // trailing lower blocks: A[i][j] -= sum_k L[i][o+k] L[j][o+k]
        const int nbt = prow / 32;
        const int ntask = nbt * (nbt + 1) / 2 * 8;  // (block pair, four-row group)
#pragma unroll 1
        for (int task = warp; task < ntask; task += 16) {
            int pair = task >> 3, ib = 0;
            while (pair > ib) { pair -= ib + 1; ++ib; }
            const int jb = pair;
            const int i = o + 32 + 32 * ib + 4 * (task & 7), j = o + 32 + 32 * jb + lane;
            float acc[4];
            dot4x1(sA + i * kP + o, kP, sA + j * kP + o, 32, acc);
#pragma unroll
            for (int r = 0; r < 4; ++r) sA[(i + r) * kP + j] -= acc[r];
        }
        __syncthreads();
    }
    // the last block row of V (its S was formed during the last diagonal step)
    v_row_finish(sV, sVT, sST, 3, warp, kBaseWarps, lane);
    __syncthreads();
    // Write-out: the splits of V and V^T, 16 bytes per store.  The factor of
    // this block is not written back: after its diagonal block is factored
    // nothing reads it (the triangular solves use V_cc, the inverse steps only
    // off-diagonal blocks of L).
#pragma unroll 4
    for (int c = t; c < kB * kB / 4; c += kBaseThreads) {
        const int i = c >> 5, j0 = 4 * (c & 31);
        const size_t g = base + static_cast<size_t>(i) * ld + j0;
        const float4 v = *reinterpret_cast<const float4*>(sV + i * kP + j0);
        const float4 vt = *reinterpret_cast<const float4*>(sVT + i * kP + j0);
        float4 h, l, ht, lt;
        h.x = tf32_round(v.x); l.x = v.x - h.x;  ht.x = tf32_round(vt.x); lt.x = vt.x - ht.x;
        h.y = tf32_round(v.y); l.y = v.y - h.y;  ht.y = tf32_round(vt.y); lt.y = vt.y - ht.y;
        h.z = tf32_round(v.z); l.z = v.z - h.z;  ht.z = tf32_round(vt.z); lt.z = vt.z - ht.z;
        h.w = tf32_round(v.w); l.w = v.w - h.w;  ht.w = tf32_round(vt.w); lt.w = vt.w - ht.w;
        *reinterpret_cast<float4*>(V_hi + g) = h;
        *reinterpret_cast<float4*>(V_lo + g) = l;
        *reinterpret_cast<float4*>(VT_hi + g) = ht;
        *reinterpret_cast<float4*>(VT_lo + g) = lt;
    }
}

// Zeroes the 128-blocks next to the diagonal that no other step writes: the
// split of V's block right of each diagonal block and of V^T's block below it.
// The inverse steps' CTA-pair products read one 128-block past the triangle
// there.  One CTA per (block, row) pair, off the critical path.
__global__ void __launch_bounds__(256) zero_adjacent_kernel(float* __restrict__ V_hi, float* __restrict__ V_lo,
                                                            float* __restrict__ VT_hi, float* __restrict__ VT_lo,
                                                            int d) {
    pdl_wait();
    const int blk = blockIdx.y;  // diagonal block index, 0 .. d/128 - 2
    const size_t off = static_cast<size_t>(blk) * kB;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < kB * kB; e += gridDim.x * blockDim.x) {
        const int i = e >> 7, j = e & 127;
        const size_t gr = (off + i) * d + off + kB + j;  // V[off+i][off+128+j]
        const size_t gb = (off + kB + i) * d + off + j;  // V^T[off+128+i][off+j]
        V_hi[gr] = 0.0f; V_lo[gr] = 0.0f;
        VT_hi[gb] = 0.0f; VT_lo[gb] = 0.0f;
    }
}
constexpr size_t kBaseSmem = (3 * kB * kP + 3 * 32 * kSP + 32 * 32 + 32 + 4) * sizeof(float);

// Ut = (P V P)^T on the lower triangle: Ut[i][j] = V[d-1-j][d-1-i] (the
// factor U = chol(H^-1) transposed, for callers that ask for it).
__global__ void reverse_transpose_kernel(const float* __restrict__ V_hi, const float* __restrict__ V_lo, int d,
                                         float* __restrict__ Ut) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;  // output tile (rows by.., cols bx..)
    pdl_wait();
    // source rows d-1-(bx+..), cols d-1-(by+..)
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int sr = d - 1 - (bx + k), sc = d - 1 - (by + threadIdx.x);
        const size_t g = static_cast<size_t>(sr) * d + sc;
        tile[k][threadIdx.x] = V_hi[g] + V_lo[g];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int i = by + k, j = bx + threadIdx.x;
        const float v = (j <= i) ? tile[threadIdx.x][k] : 0.0f;
        Ut[static_cast<size_t>(i) * d + j] = v;
    }
}

// In-block OBS sweep of columns [i1, i1+128) for every row.  Eight lanes (an
// octet) share a row; lane l of the octet holds groups l, l+8, l+16, l+24 of
// the row (columns 4g..4g+3) in registers, the current one always in slot 0
// (the slots shift down by one group after every eight groups).  Group g is
// handled by its owning lane: it selects the mask, eliminates the group's
// pruned columns inside the group, and hands the pruned columns' errors to
// the octet by shuffle; every lane then applies them to its own later
// columns.  Only pruned columns carry an error, so the update runs over
// exactly the 4 - N pruned ones, in column order, as the sequential sweep
// does: results are those of the plain row-by-row algorithm.  A finished
// group (slot 0 after its eight groups) is written out at once.
// The sweep keeps W and the errors in reversed column order (Wr[:, c] =
// W[:, d-1-c], likewise E), so that the later columns' updates are plain
// products with V = L^-1 of the reversed Hessian; this kernel reads its block
// from Wr, writes the block's final weights to W in natural order (no later
// step touches them), and its errors to E reversed.  Its block of U is
// U[i1+q][i1+j] = V[o+127-q][o+127-j], o = d-i1-128, kept in shared memory
// row by row.  M must be 4 here; N:4 with N in {1, 2, 3}.
constexpr int kUp = kB + 4;                         // pitch of a row of U in shared memory
constexpr int kIbThreads = 256;                     // eight warps of four rows: 32 rows per CTA,
constexpr int kIbRows = 32;                         // so 4096 rows take 128 SMs
constexpr size_t kIbSmem = (kB * kUp + kB) * sizeof(float);

__device__ __forceinline__ uint32_t obs_keep_bits(const float (&w)[4], const float* rv, int n_keep) {
    float s[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float x = w[k] * rv[k];
        s[k] = x * x;
    }
    uint32_t bits = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int rank = 0;
#pragma unroll
        for (int o = 0; o < 4; ++o) rank += (s[o] < s[k] || (o < k && s[o] == s[k])) ? 1 : 0;
        if (rank >= 4 - n_keep) bits |= 1u << k;
    }
    return bits;
}

__global__ void __launch_bounds__(kIbThreads) inblock_kernel(float* __restrict__ W, const float* __restrict__ Wr,
                                                             int r, int d, int i1, const float* __restrict__ V_hi,
                                                             const float* __restrict__ V_lo, int n_keep,
                                                             uint8_t* __restrict__ mask,
                                                             float* __restrict__ E_hi, float* __restrict__ E_lo,
                                                             long long ldE) {
    extern __shared__ float u1[];
    float* rinv = u1 + kB * kUp;
    const int o = d - i1 - kB;  // the block's first column in reversed order
    pdl_wait();
    // U[q][j] = V[o+vr][o+vc] with q = 127-vr, j = 127-vc (j >= q, i.e. vc <= vr),
    // V = V_hi + V_lo (exact), read along V's rows 16 bytes at a time, eight
    // chunks of each part in flight per thread
    constexpr int kIbChunks = kB * kB / 4 / kIbThreads;  // 16
#pragma unroll 1
    for (int u0 = 0; u0 < kIbChunks; u0 += 8) {
        float4 h[8], l[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = threadIdx.x + (u0 + u) * kIbThreads, vr = c >> 5, vc0 = 4 * (c & 31);
            const size_t g = static_cast<size_t>(o + vr) * d + o + vc0;
            const bool in = vc0 <= vr;
            h[u] = in ? *reinterpret_cast<const float4*>(V_hi + g) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            l[u] = in ? *reinterpret_cast<const float4*>(V_lo + g) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int c = threadIdx.x + (u0 + u) * kIbThreads, vr = c >> 5, vc0 = 4 * (c & 31);
            const float x[4] = {h[u].x + l[u].x, h[u].y + l[u].y, h[u].z + l[u].z, h[u].w + l[u].w};
            float* ur = u1 + (127 - vr) * kUp + 127 - vc0;  // U[127-vr][127-vc0-k] = ur[-k]
#pragma unroll
            for (int k = 0; k < 4; ++k) ur[-k] = vc0 + k <= vr ? x[k] : 0.0f;
        }
    }
    __syncthreads();
    if (threadIdx.x < kB) rinv[threadIdx.x] = __frcp_rn(u1[threadIdx.x * kUp + threadIdx.x]);
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ql = lane & 7, oct = lane & ~7;
    const size_t row = static_cast<size_t>(blockIdx.x) * kIbRows + 4 * warp + (lane >> 3);
    if (row >= static_cast<size_t>(r)) return;  // r % 128 == 0: whole octets only
    // slot s (w[4s..4s+3]) = natural columns 4(8s+ql)..+3 = Wr columns o+124-32s-4ql..o+127-32s-4ql
    float w[16];
    const float* wsrc = Wr + row * d + o;
#pragma unroll
    for (int s = 0; s < 4; ++s) {
        const float4 x = *reinterpret_cast<const float4*>(wsrc + 124 - 32 * s - 4 * ql);
        w[4 * s] = x.w; w[4 * s + 1] = x.z; w[4 * s + 2] = x.y; w[4 * s + 3] = x.x;
    }
    float* wdst = W + row * d + i1;
    float* ehi = E_hi + row * ldE + o;
    float* elo = E_lo + row * ldE + o;
    uint8_t* mrow = mask + (row * d + i1) / 4;
    const int n_prune = 4 - n_keep;
#pragma unroll 1
    for (int m = 0; m < 4; ++m) {  // groups 8m..8m+7; this lane's group 8m+ql sits in slot 0
        float e_own[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        uint32_t bits_own = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int q0 = 4 * (8 * m + j);
            // the group's 1/U_qq and in-group U entries, loaded by every lane ahead of the branch
            const float4 rq = *reinterpret_cast<const float4*>(rinv + q0);
            const float4 ua = *reinterpret_cast<const float4*>(u1 + q0 * kUp + q0);
            const float4 ub = *reinterpret_cast<const float4*>(u1 + (q0 + 1) * kUp + q0);
            const float4 uc = *reinterpret_cast<const float4*>(u1 + (q0 + 2) * kUp + q0);
            uint32_t bits = 0;
            float xp[3] = {0.0f, 0.0f, 0.0f};  // errors of the pruned columns, in column order
            if (ql == j) {
                const float rv[4] = {rq.x, rq.y, rq.z, rq.w};
                const float ug[3][4] = {{ua.x, ua.y, ua.z, ua.w}, {ub.x, ub.y, ub.z, ub.w}, {uc.x, uc.y, uc.z, uc.w}};
                float wg[4] = {w[0], w[1], w[2], w[3]};
                bits = obs_keep_bits(wg, rv, n_keep);
                int p = 0;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const bool pruned = !((bits >> k) & 1u);
                    const float x = pruned ? wg[k] * rv[k] : 0.0f;
#pragma unroll
                    for (int kk = k + 1; kk < 4; ++kk) wg[kk] = pruned ? fmaf(-x, ug[k][kk], wg[kk]) : wg[kk];
                    wg[k] = pruned ? 0.0f : wg[k];
                    e_own[k] = x;
                    xp[0] = pruned && p == 0 ? x : xp[0];
                    xp[1] = pruned && p == 1 ? x : xp[1];
                    xp[2] = pruned && p == 2 ? x : xp[2];
                    p += pruned ? 1 : 0;
                }
                w[0] = wg[0]; w[1] = wg[1]; w[2] = wg[2]; w[3] = wg[3];
                bits_own = bits;
            }
            bits = __shfl_sync(kFull, bits, oct | j);
            xp[0] = __shfl_sync(kFull, xp[0], oct | j);
            if (n_prune > 1) xp[1] = __shfl_sync(kFull, xp[1], oct | j);
            if (n_prune > 2) xp[2] = __shfl_sync(kFull, xp[2], oct | j);
            // pruned column indices inside the group, in order (exactly n_prune
            // of them unless a score is NaN, which a failed pivot reports anyway)
            uint32_t rest = ~bits & 0xFu;
            const int np = min(n_prune, __popc(rest));
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                if (p >= np) break;
                const int k = __ffs(rest) - 1;
                rest &= rest - 1;
                const float x = xp[p];
                const float* ur = u1 + (q0 + k) * kUp + 4 * ql;
                if (ql > j) {  // slot 0 lies after the group
                    const float4 uu = *reinterpret_cast<const float4*>(ur + 32 * m);
                    w[0] = fmaf(-x, uu.x, w[0]); w[1] = fmaf(-x, uu.y, w[1]);
                    w[2] = fmaf(-x, uu.z, w[2]); w[3] = fmaf(-x, uu.w, w[3]);
                }
#pragma unroll
                for (int s = 1; s < 4; ++s) {
                    if (m + s < 4) {
                        const float4 uu = *reinterpret_cast<const float4*>(ur + 32 * (m + s));
                        w[4 * s] = fmaf(-x, uu.x, w[4 * s]);
                        w[4 * s + 1] = fmaf(-x, uu.y, w[4 * s + 1]);
                        w[4 * s + 2] = fmaf(-x, uu.z, w[4 * s + 2]);
                        w[4 * s + 3] = fmaf(-x, uu.w, w[4 * s + 3]);
                    }
                }
            }
        }
        // slot 0 is final: natural columns 32m+4ql..+3, errors reversed, the mask byte
        *reinterpret_cast<float4*>(wdst + 32 * m + 4 * ql) = make_float4(w[0], w[1], w[2], w[3]);
        float hv[4], lv[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float v = e_own[3 - t];
            hv[t] = tf32_round(v);
            lv[t] = v - hv[t];
        }
        *reinterpret_cast<float4*>(ehi + 124 - 32 * m - 4 * ql) = make_float4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<float4*>(elo + 124 - 32 * m - 4 * ql) = make_float4(lv[0], lv[1], lv[2], lv[3]);
        mrow[8 * m + ql] = static_cast<uint8_t>(bits_own);
#pragma unroll
        for (int k = 0; k < 12; ++k) w[k] = w[k + 4];
        w[12] = w[13] = w[14] = w[15] = 0.0f;
    }
}

// Wr[:, c] = W[:, d-1-c] for the sweep (one float4 per thread step).
__global__ void reverse_columns_kernel(const float* __restrict__ W, float* __restrict__ Wr, int r, int d) {
    pdl_wait();
    const size_t q = static_cast<size_t>(d / 4), total = static_cast<size_t>(r) * q;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t row = e / q, c4 = e % q;
        const float4 x = reinterpret_cast<const float4*>(W + row * d)[q - 1 - c4];
        reinterpret_cast<float4*>(Wr + row * d)[c4] = make_float4(x.w, x.z, x.y, x.x);
    }
}

constexpr int kMaxDepth = 16;
constexpr int kLookAhead = 1024;  // split the Schur update of nodes whose A22 is at least this wide

struct Work {
    float *A, *A_hi, *A_lo, *V_hi, *V_lo, *VT_hi, *VT_lo;
    float *T_hi[kMaxDepth], *T_lo[kMaxDepth];  // the inverse step's temporary, one per recursion depth
    int d;
    int* bad;
    cudaStream_t side;  // stream of the triangular-inverse steps
    cudaEvent_t ev;     // "this node's factor is complete", re-recorded per node
    cudaStream_t ahead;              // stream of the look-ahead Schur updates
    cudaEvent_t evl;                 // "this node's L21 is complete"
    cudaEvent_t ev21[kMaxDepth], ev22[kMaxDepth];  // look-ahead updates done, per recursion depth
    cudaEvent_t evv[kMaxDepth];  // a node's V21 (and its V^T split) complete on w.side, per depth
};

// Regions of a node's matrix that its parent's look-ahead update is still
// writing on the look-ahead stream: rows n1.. x cols ..n1 (ev21) and rows
// n1.. x cols n1.. (ev22), n1 = half_blocks(n); null when already complete.
struct Pending {
    cudaEvent_t ev21 = nullptr, ev22 = nullptr;
};

int gemm(const float* ah, const float* al, long long lda, const float* bh, const float* bl, long long ldb, int M, int N,
         int K, umma::GemmOut o, cudaStream_t st) {
    return umma::gemm_nt(umma::kTF32x3, {ah, al, lda}, {bh, bl, ldb}, M, N, K, o, st);
}

long long half_blocks(int n) { return static_cast<long long>(n / kB / 2) * kB; }

// Solves X L^T = B in place for B = A[r0 : r0+m, c0 : c0+n] (and its split),
// L = the lower factor in A[c0 : c0+n, c0 : c0+n].  Recursive on L: only the
// 128 x 128 diagonal blocks are inverted (their inverses sit in V), the rest is
// GEMM updates, which keeps the solve as stable as a triangular solve.
int trsm(Work& w, long long r0, int m, long long c0, int n, cudaStream_t st) {
    const long long d = w.d;
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    int rc;
    if (n == kB) {  // B <- B V_cc^T, in place; only the split is read later (solved blocks
                    // are operands from then on, never a Cin)
        umma::GemmOut o{};
        o.C_hi = at(w.A_hi, r0, c0); o.C_lo = at(w.A_lo, r0, c0); o.ld_split = d;
        o.alpha = 1.0f; o.beta = 0.0f;
        return gemm(at(w.A_hi, r0, c0), at(w.A_lo, r0, c0), d, at(w.V_hi, c0, c0), at(w.V_lo, c0, c0), d, m, kB, kB,
                    o, st);
    }
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    if ((rc = trsm(w, r0, m, c0, n1, st))) return rc;
    {  // B2 -= B1 L21^T
        umma::GemmOut o{};
        o.C = at(w.A, r0, c0 + n1); o.ldc = d;
        o.Cin = at(w.A, r0, c0 + n1); o.ldcin = d;
        o.C_hi = at(w.A_hi, r0, c0 + n1); o.C_lo = at(w.A_lo, r0, c0 + n1); o.ld_split = d;
        o.alpha = -1.0f; o.beta = 1.0f;
        if ((rc = gemm(at(w.A_hi, r0, c0), at(w.A_lo, r0, c0), d, at(w.A_hi, c0 + n1, c0), at(w.A_lo, c0 + n1, c0),
                       d, m, n2, n1, o, st)))
            return rc;
    }
    return trsm(w, r0, m, c0 + n1, n2, st);
}

int trtri_t(Work& w, int off, int n, int depth, cudaStream_t st);
int trtri_v(Work& w, int off, int n, int depth, cudaStream_t st);

// Schur update A[r0.., c0..] -= L[r0.., lc..] L[c0.., lc..]^T over an (m x nn)
// region with inner size k, with split; lower_only for diagonal regions.
int schur(Work& w, long long r0, long long c0, int m, int nn, long long lc, int k, int lower, cudaStream_t st) {
    const long long d = w.d;
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    umma::GemmOut o{};
    o.C = at(w.A, r0, c0); o.ldc = d;
    o.Cin = at(w.A, r0, c0); o.ldcin = d;
    o.C_hi = at(w.A_hi, r0, c0); o.C_lo = at(w.A_lo, r0, c0); o.ld_split = d;
    o.alpha = -1.0f; o.beta = 1.0f; o.lower_only = lower;
    return gemm(at(w.A_hi, r0, lc), at(w.A_lo, r0, lc), d, at(w.A_hi, c0, lc), at(w.A_lo, c0, lc), d, m, nn, k, o, st);
}

int wait_on(cudaStream_t st, cudaEvent_t ev) {
    if (!ev) return TB_OK;
    const cudaError_t e = cudaStreamWaitEvent(st, ev, 0);
    pdl_fence(st);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "tb_obs_sparsegpt stream wait");
}
int record_on(cudaEvent_t ev, cudaStream_t st) {
    const cudaError_t e = cudaEventRecord(ev, st);
    return e == cudaSuccess ? TB_OK : cuda_fail(e, "tb_obs_sparsegpt event record");
}

// Recursive Cholesky of A[off : off+n] (lower, in place, with split); the
// 128 x 128 diagonal blocks also get their inverses in V / VT.
//  * Inverse steps: once a node's factor is enqueued on st, its inverse step
//    goes to w.side behind an event, beside the rest of the factorisation,
//    whose chain of small dependent launches leaves most SMs idle.  Inverse
//    steps only touch V's off-diagonal blocks and T, which the factor side
//    never reads, and on w.side they keep the recursion's order.
//  * Look-ahead: of the Schur update A22 -= L21 L21^T only the top-left
//    triangle (what the child factors first) runs on st; the lower-left block
//    and the lower-right triangle go to w.ahead, and the child waits for them
//    just before its own solve and update touch those regions.
int chol(Work& w, int off, int n, cudaStream_t st, int depth, Pending pend) {
    if (n == kB) {
        const cudaError_t e = launch_pdl(base_chol_inv_kernel, dim3(1), dim3(kBaseThreads), kBaseSmem, st,
                                         static_cast<const float*>(w.A), w.V_hi, w.V_lo, w.VT_hi, w.VT_lo, w.d, off,
                                         w.bad);
        return e == cudaSuccess ? check_launch("base_chol_inv_kernel") : cuda_fail(e, "base_chol_inv_kernel launch");
    }
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    const long long o1 = off + n1;
    int rc = chol(w, off, n1, st, depth + 1, Pending{});
    if (!rc) rc = wait_on(st, pend.ev21);                 // A21 fully updated by the parent
    if (!rc) rc = trsm(w, o1, n2, off, n1, st);          // L21 = A21 L11^-T
    if (!rc) rc = record_on(w.ev, st);                    // L21 and V11 exist: T on the side stream
    if (!rc) rc = wait_on(w.side, w.ev);
    if (!rc) rc = trtri_t(w, off, n, depth, w.side);
    if (!rc) rc = wait_on(st, pend.ev22);                 // A22 fully updated by the parent
    if (rc) return rc;
    Pending child{};
    if (n2 >= kLookAhead && depth < kMaxDepth) {
        const int h1 = static_cast<int>(half_blocks(n2)), h2 = n2 - h1;
        if ((rc = record_on(w.evl, st))) return rc;
        if ((rc = wait_on(w.ahead, w.evl))) return rc;
        if ((rc = schur(w, o1 + h1, o1, h2, h1, off, n1, 0, w.ahead))) return rc;        // lower-left block
        if ((rc = record_on(w.ev21[depth], w.ahead))) return rc;
        if ((rc = schur(w, o1 + h1, o1 + h1, h2, h2, off, n1, 1, w.ahead))) return rc;   // lower-right triangle
        if ((rc = record_on(w.ev22[depth], w.ahead))) return rc;
        if ((rc = schur(w, o1, o1, h1, h1, off, n1, 1, st))) return rc;                 // top-left triangle
        child.ev21 = w.ev21[depth];
        child.ev22 = w.ev22[depth];
    } else if ((rc = schur(w, o1, o1, n2, n2, off, n1, 1, st))) {
        return rc;
    }
    if ((rc = chol(w, off + n1, n2, st, depth + 1, child))) return rc;
    if ((rc = record_on(w.ev, st))) return rc;
    if ((rc = wait_on(w.side, w.ev))) return rc;
    if ((rc = trtri_v(w, off, n, depth, w.side))) return rc;
    return record_on(w.evv[depth], w.side);
}

// Node steps of the triangular inverse V = L^-1 for the node [off, off+n):
// V21 = -V22 (L21 V11), with V^T kept alongside.  trtri_t forms
// T^T = V11^T L21^T as soon as L21 and V11 exist (long before the node's
// lower half is factored); trtri_v then forms V21 = -V22 T once V22 exists.
// T lives in a buffer of the node's recursion depth: between the two steps
// only deeper nodes run theirs.  Both products take a triangular left operand,
// so each output tile row runs only over the K tiles inside the triangle.
int trtri_t(Work& w, int off, int n, int depth, cudaStream_t st) {
    const long long d = w.d;
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    const long long o1 = off + n1;
    umma::GemmOut o{};
    o.C_hi = w.T_hi[depth]; o.C_lo = w.T_lo[depth]; o.ld_split = n2;
    o.alpha = 1.0f; o.beta = 0.0f;
    o.tri_a = 1;  // V11^T upper
    return gemm(at(w.VT_hi, off, off), at(w.VT_lo, off, off), d, at(w.A_hi, o1, off), at(w.A_lo, o1, off), d, n1, n2,
                n1, o, st);
}

int trtri_v(Work& w, int off, int n, int depth, cudaStream_t st) {
    const long long d = w.d;
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    const long long o1 = off + n1;
    umma::GemmOut o{};
    o.C_hi = at(w.V_hi, o1, off); o.C_lo = at(w.V_lo, o1, off); o.ld_split = d;
    o.Ct_hi = at(w.VT_hi, off, o1); o.Ct_lo = at(w.VT_lo, off, o1); o.ldct = d;
    o.alpha = -1.0f; o.beta = 0.0f;
    o.tri_a = 2;  // V22 lower
    return gemm(at(w.V_hi, o1, o1), at(w.V_lo, o1, o1), d, w.T_hi[depth], w.T_lo[depth], n2, n2, n1, n2, o, st);
}

// Largest n1 x n2 of the inverse steps at each recursion depth (T's size).
void trtri_sizes(int n, int depth, size_t* need) {
    if (n == kB || depth >= kMaxDepth) return;
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    need[depth] = std::max(need[depth], static_cast<size_t>(n1) * n2);
    trtri_sizes(n1, depth + 1, need);
    trtri_sizes(n2, depth + 1, need);
}

struct Sweep {
    float* W;                        // the caller's weights (final values, natural order)
    float* Wr;                       // working copy, columns reversed
    int r, d, n_keep;
    const float *V_hi, *V_lo, *VT_hi, *VT_lo;  // split of L^-1 (reversed Hessian) and of its transpose
    uint8_t* mask;
    float *E_hi, *E_lo;              // r x d errors, columns reversed, pitch d
    cudaStream_t ahead;              // look-ahead updates
    cudaEvent_t evl;                 // "the high part's errors are complete"
    const cudaEvent_t* ev;           // [kMaxDepth] look-ahead update done, per depth
    const cudaEvent_t* evv;          // [kMaxDepth] a node's V21 complete, per depth
    bool* evv_waited;                // [kMaxDepth] st already waited on evv[depth]
};

// Column sweep in reversed coordinates.  With P the reversal, U = P V P, so
// natural column q is reversed column d-1-q and the lazy update of later
// columns, W[:, c] -= sum_{k < c} E[:, k] U[k][c], reads in reversed order
//   Wr[:, c'] -= sum_{k' > c'} Er[:, k'] V[k'][c'],
// a product whose right operand is V^T's block, rows c', columns k', as
// stored.  The recursion is the factorisation's own: node [o, o+n) sweeps its
// high part [o1, o+n) first (the earlier natural columns), then updates its low
// part with Wr[:, o : o1] -= Er[:, o1 : o+n] (V^T[o : o1, o1 : o+n])^T, whose
// right operand is exactly this node's V21 -- the last inverse step of the
// node, which can therefore still be running while the high part is swept.
// W[:, k0..] reversed: Wr[:, c0 : c0+nc] -= Er[:, k0 : k0+k] V^T[c0 : c0+nc, k0 : k0+k]^T.
int sweep_update(const Sweep& s, int k0, int k, int c0, int nc, cudaStream_t st) {
    const long long d = s.d;
    umma::GemmOut o{};
    o.C = s.Wr + c0; o.ldc = d;
    o.Cin = s.Wr + c0; o.ldcin = d;
    o.alpha = -1.0f; o.beta = 1.0f;
    return umma::gemm_nt(umma::kTF32x3, {s.E_hi + k0, s.E_lo + k0, d},
                         {s.VT_hi + c0 * d + k0, s.VT_lo + c0 * d + k0, d}, s.r, nc, k, o, st);
}

// pend: the parent's look-ahead update of this node's low part (reversed
// columns o .. o + half_blocks(n)) is still running on s.ahead; null when complete.
int sweep(const Sweep& s, int o, int n, cudaStream_t st, int depth, cudaEvent_t pend) {
    if (n == kB) {
        const cudaError_t e = launch_pdl(inblock_kernel, dim3((s.r + kIbRows - 1) / kIbRows), dim3(kIbThreads), kIbSmem,
                                         st, s.W, static_cast<const float*>(s.Wr), s.r, s.d, s.d - o - kB, s.V_hi,
                                         s.V_lo, s.n_keep, s.mask, s.E_hi, s.E_lo, static_cast<long long>(s.d));
        return e == cudaSuccess ? check_launch("inblock_kernel") : cuda_fail(e, "inblock_kernel launch");
    }
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1, o1 = o + n1;
    int rc = sweep(s, o1, n2, st, depth + 1, nullptr);
    if (!rc) rc = wait_on(st, pend);          // the low part has all earlier errors applied
    // This node's V21 exists.  evv[depth] holds the record of the last node of
    // this depth in the factorisation's post-order, the rightmost one, which is
    // also the first node of this depth that the sweep (high parts first)
    // reaches; every other node of the depth recorded earlier on the same
    // stream, so one wait per depth covers them all.
    if (!rc && !s.evv_waited[depth]) {
        rc = wait_on(st, s.evv[depth]);
        s.evv_waited[depth] = true;
    }
    if (rc) return rc;
    if (n1 >= kLookAhead && depth < kMaxDepth) {
        // Look-ahead: the part of the low half that the child sweeps first (its
        // high part) is updated on st, the rest on s.ahead (ordered after the
        // parent's piece there), and the child waits for it before its own
        // update of it.
        const int h = static_cast<int>(half_blocks(n1));
        if ((rc = record_on(s.evl, st))) return rc;
        if ((rc = wait_on(s.ahead, s.evl))) return rc;
        if ((rc = sweep_update(s, o1, n2, o, h, s.ahead))) return rc;
        if ((rc = record_on(s.ev[depth], s.ahead))) return rc;
        if ((rc = sweep_update(s, o1, n2, o + h, n1 - h, st))) return rc;
        return sweep(s, o, n1, st, depth + 1, s.ev[depth]);
    }
    if ((rc = sweep_update(s, o1, n2, o, n1, st))) return rc;
    return sweep(s, o, n1, st, depth + 1, nullptr);
}

}  // namespace

namespace {

// Per-device workspace kept between calls (grow-only): the d x d matrices of a
// 14336-wide layer take ~9 GB, and re-mapping that much per call costs more
// than the factorisation.
struct Workspace {
    int dev = -1;
    float* ptr = nullptr;
    size_t floats = 0;
    cudaStream_t side = nullptr, ahead = nullptr, chain = nullptr;
    cudaEvent_t ev = nullptr, join = nullptr, evl = nullptr, join_ahead = nullptr, fork = nullptr, done = nullptr;
    cudaEvent_t wcopy = nullptr;
    cudaEvent_t ev21[kMaxDepth] = {}, ev22[kMaxDepth] = {}, evv[kMaxDepth] = {};
    cudaEvent_t phase[4] = {};  // timing events on the chain stream: start, H ready, factored, swept
};
std::mutex g_ws_mu;
std::vector<Workspace> g_ws;
// Chain-stream phase times of this host thread's last successful call.
thread_local float g_obs_phase_ms[4] = {0, 0, 0, 0};

// Per-device workspace of at least `floats` floats, with the side stream and
// events of the inverse steps (created once per device).
int workspace(size_t floats, Workspace* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_ws_mu);
    Workspace* w = nullptr;
    for (auto& x : g_ws)
        if (x.dev == dev) w = &x;
    if (!w) {
        Workspace x;
        x.dev = dev;
        // The chain of dependent steps runs on a high-priority stream; the
        // inverse steps and look-ahead updates beside it on low-priority ones,
        // so freed SMs go to the chain first.
        int least = 0, greatest = 0;
        e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&x.chain, cudaStreamNonBlocking, greatest);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&x.side, cudaStreamNonBlocking, least);
        if (e == cudaSuccess) e = cudaStreamCreateWithPriority(&x.ahead, cudaStreamNonBlocking, least);
        cudaEvent_t* evs[] = {&x.ev, &x.join, &x.evl, &x.join_ahead, &x.fork, &x.done, &x.wcopy};
        for (cudaEvent_t* p : evs)
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(p, cudaEventDisableTiming);
        for (auto& p : x.phase)
            if (e == cudaSuccess) e = cudaEventCreate(&p);
        for (int k = 0; k < kMaxDepth && e == cudaSuccess; ++k) {
            e = cudaEventCreateWithFlags(&x.ev21[k], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&x.ev22[k], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&x.evv[k], cudaEventDisableTiming);
        }
        if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt stream/event setup");
        g_ws.push_back(x);
        w = &g_ws.back();
    }
    if (w->floats < floats) {
        if (w->ptr) {
            cudaDeviceSynchronize();
            cudaFree(w->ptr);
        }
        w->ptr = nullptr;
        w->floats = 0;
        e = cudaMalloc(reinterpret_cast<void**>(&w->ptr), floats * sizeof(float));
        if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt workspace");
        w->floats = floats;
    }
    *out = *w;
    return TB_OK;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_obs_hessian(const void* xt, int d, int n, float* H, void* stream) {
    if (n <= 0) return fail(TB_ERR_SHAPE, "tb_obs_hessian: n must be positive");
    return tb_obs_hessian_scaled(xt, d, n, 1.0f / static_cast<float>(n), H, stream);
}

extern "C" int tb_obs_hessian_scaled(const void* xt, int d, int n, float scale, float* H, void* stream) {
    if (d <= 0 || n <= 0 || d % kB || n % 64) return fail(TB_ERR_SHAPE, "tb_obs_hessian: d %% 128 and n %% 64 must be 0");
    if (!xt || !H) return fail(TB_ERR_ARG, "tb_obs_hessian: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    pdl_fence(static_cast<cudaStream_t>(stream));  // the caller may have queued a cross-stream wait
    umma::GemmOut o{};
    o.C = H; o.ldc = d;
    o.alpha = scale;
    o.beta = 0.0f;
    o.lower_only = 1;
    return umma::gemm_nt(umma::kBF16, {xt, nullptr, n}, {xt, nullptr, n}, d, d, n, o, static_cast<cudaStream_t>(stream));
}

extern "C" int tb_obs_sparsegpt(float* W, int r, int d, const float* H, float damp_frac, int n_keep, int m,
                                uint8_t* mask, float* ut_out, void* stream) {
    if (r <= 0 || d <= 0 || r % kB || d % kB) return fail(TB_ERR_SHAPE, "tb_obs_sparsegpt: r and d must be multiples of 128");
    if (d > (1 << 20)) return fail(TB_ERR_SHAPE, "tb_obs_sparsegpt: d above 2^20 (recursion depth)");
    if (m != 4 || n_keep <= 0 || n_keep >= m) return fail(TB_ERR_UNSUPPORTED, "tb_obs_sparsegpt: N:4 patterns only (N in 1..3)");
    if (!W || !H || !mask) return fail(TB_ERR_ARG, "tb_obs_sparsegpt: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    const auto user = static_cast<cudaStream_t>(stream);
    const size_t dd = static_cast<size_t>(d) * d;
    const size_t rd = static_cast<size_t>(r) * d;
    // Workspace: 7 d x d FP32 matrices (A with its split, the splits of V and V^T), the
    // inverse steps' temporaries T (one per recursion depth, with split;
    // about d^2/3 in all), the error matrix E (r x d, with split), the
    // column-reversed copy of W (r x d) and two scalars.
    size_t tneed[kMaxDepth] = {};
    trtri_sizes(d, 0, tneed);
    size_t tsum = 0;
    for (size_t x : tneed) tsum += (x + 63) / 64 * 64;  // keep each buffer 256-byte aligned
    Workspace wsp;
    const size_t ws_floats = 7 * dd + 2 * tsum + 3 * rd + 64;
    if ((rc = workspace(ws_floats, &wsp))) return rc;
    float* ws = wsp.ptr;
    cudaError_t e = cudaSuccess;
    // everything below runs on the internal chain stream, forked from and
    // joined back into the caller's stream
    const cudaStream_t st = wsp.chain;
    e = cudaEventRecord(wsp.fork, user);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, wsp.fork, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(wsp.ahead, wsp.fork, 0);
    if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt stream fork");
    pdl_fence(st);
    pdl_fence(wsp.ahead);
    pdl_fence(wsp.side);  // its first launch follows the previous call's last one
    cudaEventRecord(wsp.phase[0], st);
    Work w{};
    w.d = d;
    w.side = wsp.side;
    w.ev = wsp.ev;
    w.ahead = wsp.ahead;
    w.evl = wsp.evl;
    for (int k = 0; k < kMaxDepth; ++k) {
        w.ev21[k] = wsp.ev21[k];
        w.ev22[k] = wsp.ev22[k];
        w.evv[k] = wsp.evv[k];
    }
    w.A = ws; w.A_hi = ws + dd; w.A_lo = ws + 2 * dd;
    w.V_hi = ws + 3 * dd; w.V_lo = ws + 4 * dd;
    w.VT_hi = ws + 5 * dd; w.VT_lo = ws + 6 * dd;
    float* tp = ws + 7 * dd;
    for (int k = 0; k < kMaxDepth; ++k) {
        const size_t sz = (tneed[k] + 63) / 64 * 64;
        w.T_hi[k] = tp;
        w.T_lo[k] = tp + sz;
        tp += 2 * sz;
    }
    float* E_hi = tp;
    float* E_lo = E_hi + rd;
    float* Wr = E_lo + rd;
    double* dsum = reinterpret_cast<double*>(Wr + rd);
    w.bad = reinterpret_cast<int*>(dsum + 1);
    e = cudaFuncSetAttribute(base_chol_inv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kBaseSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(inblock_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kIbSmem));
    if (e == cudaSuccess) e = cudaMemsetAsync(w.bad, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt setup");
    e = launch_pdl(diag_sum_kernel, dim3(1), dim3(1024), 0, st, H, d, dsum);
    if (e == cudaSuccess)
        e = launch_pdl(reverse_damp_kernel, dim3(d / 32, d / 32), dim3(32, 8), 0, st, H, d,
                       static_cast<const double*>(dsum), damp_frac, w.A, w.A_hi, w.A_lo);
    rc = e == cudaSuccess ? check_launch("hessian prep") : cuda_fail(e, "hessian prep launch");
    if (!rc && d > kB) {  // on the side stream, ahead of every inverse step there
        e = launch_pdl(zero_adjacent_kernel, dim3(16, d / kB - 1), dim3(256), 0, w.side, w.V_hi, w.V_lo,
                       w.VT_hi, w.VT_lo, d);
        rc = e == cudaSuccess ? check_launch("zero_adjacent_kernel") : cuda_fail(e, "zero_adjacent_kernel launch");
    }
    if (!rc) {  // the sweep's reversed copy of W, on the look-ahead stream while the factorisation starts
        e = launch_pdl(reverse_columns_kernel, dim3(148 * 8), dim3(256), 0, w.ahead, static_cast<const float*>(W), Wr,
                       r, d);
        if (e == cudaSuccess) e = cudaEventRecord(wsp.wcopy, w.ahead);
        rc = e == cudaSuccess ? check_launch("reverse_columns_kernel") : cuda_fail(e, "reverse_columns launch");
    }
    if (!rc) cudaEventRecord(wsp.phase[1], st);
    if (!rc) rc = chol(w, 0, d, st, 0, Pending{});
    if (!rc) cudaEventRecord(wsp.phase[2], st);
    // The sweep starts as soon as the last 128-block is factored: it waits for
    // each node's last inverse step only where it reads that node's V21.
    if (!rc) rc = wait_on(st, wsp.wcopy);
    bool evv_waited[kMaxDepth] = {};
    if (!rc)
        rc = sweep(Sweep{W, Wr, r, d, n_keep, w.V_hi, w.V_lo, w.VT_hi, w.VT_lo, mask, E_hi, E_lo, w.ahead, w.evl, w.ev21,
                         w.evv,
                         evv_waited},
                   0, d, st, 0, nullptr);
    if (!rc) cudaEventRecord(wsp.phase[3], st);
    // join: the inverse steps (side) and look-ahead updates (ahead) finish
    // before anything reads V or the next call reuses the workspace (also on errors)
    e = cudaEventRecord(wsp.join, w.side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, wsp.join, 0);
    if (e == cudaSuccess) e = cudaEventRecord(wsp.join_ahead, w.ahead);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, wsp.join_ahead, 0);
    if (e != cudaSuccess && !rc) rc = cuda_fail(e, "tb_obs_sparsegpt stream join");
    pdl_fence(st);
    int bad = 0;
    if (!rc && ut_out) {
        e = launch_pdl(reverse_transpose_kernel, dim3(d / 32, d / 32), dim3(32, 8), 0, st,
                       static_cast<const float*>(w.V_hi), static_cast<const float*>(w.V_lo), d, ut_out);
        rc = e == cudaSuccess ? check_launch("reverse_transpose_kernel") : cuda_fail(e, "reverse_transpose launch");
    }
    // join the chain stream back into the caller's stream (also on errors)
    e = cudaEventRecord(wsp.done, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(user, wsp.done, 0);
    if (e != cudaSuccess && !rc) rc = cuda_fail(e, "tb_obs_sparsegpt stream join");
    if (!rc) {
        e = cudaMemcpyAsync(&bad, w.bad, sizeof(int), cudaMemcpyDeviceToHost, user);
        if (e == cudaSuccess) e = cudaStreamSynchronize(user);
        if (e != cudaSuccess) rc = cuda_fail(e, "tb_obs_sparsegpt sync");
    }
    if (!rc) {
        const int ge = umma::gemm_take_error(user);
        if (ge) rc = fail(TB_ERR_TIMEOUT, "a tcgen05 GEMM pipeline wait expired");
    }
    if (!rc && bad == 2) rc = fail(TB_ERR_TIMEOUT, "a wait inside the 128-block factorisation expired");
    if (!rc && bad == 1) rc = fail(TB_ERR_CONFIG, "H + lambda I is not positive definite in FP32 (a Cholesky pivot <= 0)");
    if (!rc) {  // the call synchronised: the chain stream's phase events are complete
        float* t = g_obs_phase_ms;
        cudaEventElapsedTime(&t[0], wsp.phase[0], wsp.phase[1]);
        cudaEventElapsedTime(&t[1], wsp.phase[1], wsp.phase[2]);
        cudaEventElapsedTime(&t[2], wsp.phase[2], wsp.phase[3]);
        cudaEventElapsedTime(&t[3], wsp.phase[0], wsp.phase[3]);
    }
    return rc;
}

extern "C" int tb_obs_sparsegpt_phase_times(float* ms_out, int n) {
    if (!ms_out || n < 1) return fail(TB_ERR_ARG, "tb_obs_sparsegpt_phase_times: null or empty output");
    for (int i = 0; i < n && i < 4; ++i) ms_out[i] = g_obs_phase_ms[i];
    return TB_OK;
}

// Exact OBS pruning of one weight matrix against calibration activations, in
// the column-block ("SparseGPT") formulation: BASELINE configuration 4, for
// which the reference has no implementation (docs/EHAP.md:248-250).  It keeps
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
#include "tb_runtime.h"
#include "tb_umma.cuh"

namespace tb {

int tb_split_tf32_2d(const float* x, float* hi, float* lo, int rows, int cols, long long ld, cudaStream_t st);

namespace {

constexpr int kB = 128;  // diagonal / column block
constexpr int kU1Ld = kB + 4;

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// diag sum of the lower-tile H (one block reduction, deterministic order per block).
__global__ void diag_sum_kernel(const float* __restrict__ H, int d, double* __restrict__ out) {
    __shared__ double part[1024];
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

// A = P (H + lambda I) P on the lower triangle (H valid on lower tiles), plus
// its tf32 hi/lo split; upper triangle zero.
__global__ void reverse_damp_kernel(const float* __restrict__ H, int d, const double* __restrict__ diag_sum, float frac,
                                    float* __restrict__ A, float* __restrict__ A_hi, float* __restrict__ A_lo) {
    const float lambda = static_cast<float>(frac * (*diag_sum / d));
    const size_t total = static_cast<size_t>(d) * d;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int i = static_cast<int>(e / d), j = static_cast<int>(e % d);
        float v = 0.0f;
        if (j <= i) {
            const int a = d - 1 - j, b = d - 1 - i;  // H[a][b] with a >= b: lower
            v = H[static_cast<size_t>(a) * d + b];
            if (i == j) v += lambda;
        }
        A[e] = v;
        const float h = tf32_round(v);
        A_hi[e] = h;
        A_lo[e] = v - h;
    }
}

// Cholesky and inverse of one 128 x 128 diagonal block held in shared memory.
// A block (lower) -> L (written back, lower); V = L^-1 (lower) to V with its
// split, and V^T (upper) to VT with its split.  Sets *bad if a pivot is not
// positive.
__global__ void __launch_bounds__(1024) base_chol_inv_kernel(float* __restrict__ A, float* __restrict__ V,
                                                             float* __restrict__ V_hi, float* __restrict__ V_lo,
                                                             float* __restrict__ VT, float* __restrict__ VT_hi,
                                                             float* __restrict__ VT_lo, int ld, int off,
                                                             int* __restrict__ bad) {
    extern __shared__ float sm[];
    float* sA = sm;                    // 128 x 129
    float* sV = sm + kB * (kB + 1);    // 128 x 129
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const size_t base = static_cast<size_t>(off) * ld + off;
    for (int e = t; e < kB * kB; e += blockDim.x) {
        const int i = e / kB, j = e % kB;
        sA[i * (kB + 1) + j] = (j <= i) ? A[base + static_cast<size_t>(i) * ld + j] : 0.0f;
        sV[i * (kB + 1) + j] = 0.0f;
    }
    __syncthreads();
    for (int j = 0; j < kB; ++j) {
        if (t == 0) {
            const float dj = sA[j * (kB + 1) + j];
            if (!(dj > 0.0f)) atomicExch(bad, 1);
            sA[j * (kB + 1) + j] = dj > 0.0f ? __fsqrt_rn(dj) : 1.0f;
        }
        __syncthreads();
        const float piv = sA[j * (kB + 1) + j];
        for (int i = j + 1 + t; i < kB; i += blockDim.x) sA[i * (kB + 1) + j] = __fdiv_rn(sA[i * (kB + 1) + j], piv);
        __syncthreads();
        for (int i = j + 1 + warp; i < kB; i += 32) {
            const float lij = sA[i * (kB + 1) + j];
            for (int k = j + 1 + lane; k <= i; k += 32)
                sA[i * (kB + 1) + k] = __fsub_rn(sA[i * (kB + 1) + k], __fmul_rn(lij, sA[k * (kB + 1) + j]));
        }
        __syncthreads();
    }
    // V = L^-1 by forward substitution, one column per thread.
    if (t < kB) {
        const int c = t;
        sV[c * (kB + 1) + c] = __fdiv_rn(1.0f, sA[c * (kB + 1) + c]);
        for (int i = c + 1; i < kB; ++i) {
            float s = 0.0f;
            for (int k = c; k < i; ++k) s = __fadd_rn(s, __fmul_rn(sA[i * (kB + 1) + k], sV[k * (kB + 1) + c]));
            sV[i * (kB + 1) + c] = __fdiv_rn(-s, sA[i * (kB + 1) + i]);
        }
    }
    __syncthreads();
    for (int e = t; e < kB * kB; e += blockDim.x) {
        const int i = e / kB, j = e % kB;
        const size_t g = base + static_cast<size_t>(i) * ld + j;
        if (j <= i) {
            A[g] = sA[i * (kB + 1) + j];
            const float v = sV[i * (kB + 1) + j];
            const float h = tf32_round(v);
            V[g] = v;
            V_hi[g] = h;
            V_lo[g] = v - h;
        }
        if (j >= i) {  // VT[i][j] = V[j][i]
            const float v = sV[j * (kB + 1) + i];
            const float h = tf32_round(v);
            VT[g] = v;
            VT_hi[g] = h;
            VT_lo[g] = v - h;
        }
    }
}

// Ut = (P V P)^T on the lower triangle: Ut[i][j] = V[d-1-j][d-1-i], with split.
__global__ void reverse_transpose_kernel(const float* __restrict__ V, int d, float* __restrict__ Ut,
                                         float* __restrict__ Ut_hi, float* __restrict__ Ut_lo) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;  // output tile (rows by.., cols bx..)
    // source rows d-1-(bx+..), cols d-1-(by+..)
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int sr = d - 1 - (bx + k), sc = d - 1 - (by + threadIdx.x);
        tile[k][threadIdx.x] = V[static_cast<size_t>(sr) * d + sc];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int i = by + k, j = bx + threadIdx.x;
        const float v = (j <= i) ? tile[threadIdx.x][k] : 0.0f;
        const size_t g = static_cast<size_t>(i) * d + j;
        const float h = tf32_round(v);
        Ut[g] = v;
        Ut_hi[g] = h;
        Ut_lo[g] = v - h;
    }
}

// In-block OBS sweep of columns [i1, i1+128) for every row: one warp per row,
// lane l holding columns 4l..4l+3 of the block.  M must be 4 here (the lane's
// four columns are one group); N:4 with N in {1, 2, 3}.
__global__ void __launch_bounds__(256) inblock_kernel(float* __restrict__ W, int r, int d, int i1,
                                                      const float* __restrict__ Ut, int n_keep,
                                                      uint8_t* __restrict__ mask, float* __restrict__ E_hi,
                                                      float* __restrict__ E_lo) {
    extern __shared__ float u1_raw[];
    float (*U1)[kU1Ld] = reinterpret_cast<float (*)[kU1Ld]>(u1_raw);  // U1[q][j] = U[i1+q][i1+j] = Ut[i1+j][i1+q]
    for (int e = threadIdx.x; e < kB * kB; e += blockDim.x) {
        const int q = e % kB, j = e / kB;
        U1[q][j] = (j >= q) ? Ut[static_cast<size_t>(i1 + j) * d + i1 + q] : 0.0f;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + warp;
    if (row >= r) return;
    float* wr = W + static_cast<size_t>(row) * d + i1;
    float w[4];
    {
        const float4 x = reinterpret_cast<const float4*>(wr)[lane];
        w[0] = x.x; w[1] = x.y; w[2] = x.z; w[3] = x.w;
    }
    float err[4] = {0, 0, 0, 0};
    uint32_t keep_bits = 0;
    for (int g = 0; g < kB / 4; ++g) {
        if (lane == g) {
            // saliency w^2 / U_qq^2 for the group; prune the 4 - n_keep smallest, lowest index first
            float s[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float u = U1[4 * g + k][4 * g + k];
                s[k] = __fdiv_rn(__fmul_rn(w[k], w[k]), __fmul_rn(u, u));
            }
            uint32_t bits = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                int rank = 0;
#pragma unroll
                for (int o = 0; o < 4; ++o) rank += (s[o] < s[k] || (o < k && s[o] == s[k])) ? 1 : 0;
                if (rank >= 4 - n_keep) bits |= 1u << k;
            }
            keep_bits = bits;
        }
        const uint32_t bits = __shfl_sync(0xFFFFFFFFu, keep_bits, g);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int q = 4 * g + k;
            float e = 0.0f;
            if (lane == g) {
                const float kept = ((bits >> k) & 1u) ? w[k] : 0.0f;
                e = __fdiv_rn(__fsub_rn(w[k], kept), U1[q][q]);
                err[k] = e;
            }
            e = __shfl_sync(0xFFFFFFFFu, e, g);
            // w_j -= e * U[q][j] for j >= q (columns of later lanes, and this lane's k' >= k)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const int j = 4 * lane + kk;
                if (j >= q) w[kk] = __fsub_rn(w[kk], __fmul_rn(e, U1[q][j]));
            }
            if (lane == g) w[k] = ((bits >> k) & 1u) ? w[k] : 0.0f;
        }
    }
    // w now holds the kept (updated) values of this lane's group; pruned ones are 0
    reinterpret_cast<float4*>(wr)[lane] = make_float4(w[0], w[1], w[2], w[3]);
    mask[(static_cast<size_t>(row) * d + i1) / 4 + lane] = static_cast<uint8_t>(keep_bits);
    float4 h, l;
    h.x = tf32_round(err[0]); l.x = err[0] - h.x;
    h.y = tf32_round(err[1]); l.y = err[1] - h.y;
    h.z = tf32_round(err[2]); l.z = err[2] - h.z;
    h.w = tf32_round(err[3]); l.w = err[3] - h.w;
    reinterpret_cast<float4*>(E_hi + static_cast<size_t>(row) * kB)[lane] = h;
    reinterpret_cast<float4*>(E_lo + static_cast<size_t>(row) * kB)[lane] = l;
}

struct Work {
    float *A, *A_hi, *A_lo, *V, *V_hi, *V_lo, *VT, *VT_hi, *VT_lo, *T_hi, *T_lo;
    int d;
    int* bad;
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
    if (n == kB) {  // B <- B V_cc^T, in place (one 128-column output tile per row block)
        umma::GemmOut o{};
        o.C = at(w.A, r0, c0); o.ldc = d;
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

// Recursive Cholesky of A[off : off+n] (lower, in place, with split); the
// 128 x 128 diagonal blocks also get their inverses in V / VT.
int chol(Work& w, int off, int n, cudaStream_t st, size_t base_smem) {
    const long long d = w.d;
    if (n == kB) {
        base_chol_inv_kernel<<<1, 1024, base_smem, st>>>(w.A, w.V, w.V_hi, w.V_lo, w.VT, w.VT_hi, w.VT_lo, w.d, off,
                                                         w.bad);
        return check_launch("base_chol_inv_kernel");
    }
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    int rc = chol(w, off, n1, st, base_smem);
    if (rc) return rc;
    const long long o1 = off + n1;
    if ((rc = trsm(w, o1, n2, off, n1, st))) return rc;  // L21 = A21 L11^-T
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    {  // A22 -= L21 L21^T on the lower tiles, with split
        umma::GemmOut o{};
        o.C = at(w.A, o1, o1); o.ldc = d;
        o.Cin = at(w.A, o1, o1); o.ldcin = d;
        o.C_hi = at(w.A_hi, o1, o1); o.C_lo = at(w.A_lo, o1, o1); o.ld_split = d;
        o.alpha = -1.0f; o.beta = 1.0f; o.lower_only = 1;
        if ((rc = gemm(at(w.A_hi, o1, off), at(w.A_lo, o1, off), d, at(w.A_hi, o1, off), at(w.A_lo, o1, off), d, n2,
                       n2, n1, o, st)))
            return rc;
    }
    return chol(w, off + n1, n2, st, base_smem);
}

// Recursive inverse V = L^-1 of the factor in A (diagonal 128-blocks already
// inverted by the base kernel): V21 = -V22 (L21 V11), with V^T kept alongside.
int trtri(Work& w, int off, int n, cudaStream_t st) {
    if (n == kB) return TB_OK;
    const long long d = w.d;
    auto at = [&](float* p, long long r, long long c) { return p + r * d + c; };
    const int n1 = static_cast<int>(half_blocks(n)), n2 = n - n1;
    const long long o1 = off + n1;
    int rc = trtri(w, off, n1, st);
    if (!rc) rc = trtri(w, off + n1, n2, st);
    if (rc) return rc;
    {  // T^T = V11^T L21^T  (n1 x n2), split only
        umma::GemmOut o{};
        o.C_hi = w.T_hi; o.C_lo = w.T_lo; o.ld_split = n2;
        o.alpha = 1.0f; o.beta = 0.0f;
        if ((rc = gemm(at(w.VT_hi, off, off), at(w.VT_lo, off, off), d, at(w.A_hi, o1, off), at(w.A_lo, o1, off), d,
                       n1, n2, n1, o, st)))
            return rc;
    }
    {  // V21 = -V22 T, with split, and V21^T into VT12
        umma::GemmOut o{};
        o.C = at(w.V, o1, off); o.ldc = d;
        o.C_hi = at(w.V_hi, o1, off); o.C_lo = at(w.V_lo, o1, off); o.ld_split = d;
        o.Ct = at(w.VT, off, o1); o.ldct = d;
        o.alpha = -1.0f; o.beta = 0.0f;
        if ((rc = gemm(at(w.V_hi, o1, o1), at(w.V_lo, o1, o1), d, w.T_hi, w.T_lo, n2, n2, n1, n2, o, st))) return rc;
    }
    return tb_split_tf32_2d(at(w.VT, off, o1), at(w.VT_hi, off, o1), at(w.VT_lo, off, o1), n1, n2, d, st);
}

}  // namespace

// Strided 2-D tf32 split (rows x cols block with leading dimension ld).
__global__ void split2d_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo, int rows,
                               int cols, long long ld) {
    const size_t total = static_cast<size_t>(rows) * cols;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const size_t g = (e / cols) * ld + e % cols;
        const float v = x[g];
        const float h = tf32_round(v);
        hi[g] = h;
        lo[g] = v - h;
    }
}

int tb_split_tf32_2d(const float* x, float* hi, float* lo, int rows, int cols, long long ld, cudaStream_t st) {
    const size_t total = static_cast<size_t>(rows) * cols;
    const unsigned grid = static_cast<unsigned>(std::min<size_t>((total + 255) / 256, 148u * 16u));
    split2d_kernel<<<grid, 256, 0, st>>>(x, hi, lo, rows, cols, ld);
    return check_launch("split2d_kernel");
}

namespace {

// Per-device workspace kept between calls (grow-only): the d x d matrices of a
// 14336-wide layer take ~9 GB, and re-mapping that much per call costs more
// than the factorisation.
struct Workspace {
    int dev = -1;
    float* ptr = nullptr;
    size_t floats = 0;
};
std::mutex g_ws_mu;
std::vector<Workspace> g_ws;

int workspace(size_t floats, float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_ws_mu);
    for (auto& w : g_ws)
        if (w.dev == dev) {
            if (w.floats < floats) {
                cudaDeviceSynchronize();
                cudaFree(w.ptr);
                w.ptr = nullptr;
                w.floats = 0;
                e = cudaMalloc(reinterpret_cast<void**>(&w.ptr), floats * sizeof(float));
                if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt workspace");
                w.floats = floats;
            }
            *out = w.ptr;
            return TB_OK;
        }
    Workspace w;
    w.dev = dev;
    e = cudaMalloc(reinterpret_cast<void**>(&w.ptr), floats * sizeof(float));
    if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt workspace");
    w.floats = floats;
    g_ws.push_back(w);
    *out = w.ptr;
    return TB_OK;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" int tb_obs_hessian(const void* xt, int d, int n, float* H, void* stream) {
    if (d <= 0 || n <= 0 || d % kB || n % 64) return fail(TB_ERR_SHAPE, "tb_obs_hessian: d %% 128 and n %% 64 must be 0");
    if (!xt || !H) return fail(TB_ERR_ARG, "tb_obs_hessian: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    umma::GemmOut o{};
    o.C = H; o.ldc = d;
    o.alpha = 1.0f / static_cast<float>(n);
    o.beta = 0.0f;
    o.lower_only = 1;
    return umma::gemm_nt(umma::kBF16, {xt, nullptr, n}, {xt, nullptr, n}, d, d, n, o, static_cast<cudaStream_t>(stream));
}

extern "C" int tb_obs_sparsegpt(float* W, int r, int d, const float* H, float damp_frac, int n_keep, int m,
                                uint8_t* mask, float* ut_out, void* stream) {
    if (r <= 0 || d <= 0 || r % kB || d % kB) return fail(TB_ERR_SHAPE, "tb_obs_sparsegpt: r and d must be multiples of 128");
    if (m != 4 || n_keep <= 0 || n_keep >= m) return fail(TB_ERR_UNSUPPORTED, "tb_obs_sparsegpt: N:4 patterns only (N in 1..3)");
    if (!W || !H || !mask) return fail(TB_ERR_ARG, "tb_obs_sparsegpt: null pointer");
    int rc = require_device(nullptr);
    if (rc) return rc;
    auto st = static_cast<cudaStream_t>(stream);
    const size_t dd = static_cast<size_t>(d) * d;
    // Workspace: 11 d x d FP32 matrices, the error panel split and two scalars.
    float* ws = nullptr;
    const size_t ws_floats = 11 * dd + 2 * static_cast<size_t>(r) * kB + 64;
    if ((rc = workspace(ws_floats, &ws))) return rc;
    cudaError_t e = cudaSuccess;
    Work w{};
    w.d = d;
    w.A = ws; w.A_hi = ws + dd; w.A_lo = ws + 2 * dd;
    w.V = ws + 3 * dd; w.V_hi = ws + 4 * dd; w.V_lo = ws + 5 * dd;
    w.VT = ws + 6 * dd; w.VT_hi = ws + 7 * dd; w.VT_lo = ws + 8 * dd;
    w.T_hi = ws + 9 * dd; w.T_lo = ws + 10 * dd;
    float* E_hi = ws + 11 * dd;
    float* E_lo = E_hi + static_cast<size_t>(r) * kB;
    double* dsum = reinterpret_cast<double*>(E_lo + static_cast<size_t>(r) * kB);
    w.bad = reinterpret_cast<int*>(dsum + 1);
    const size_t base_smem = 2 * kB * (kB + 1) * sizeof(float);
    const size_t u1_smem = kB * kU1Ld * sizeof(float);
    e = cudaFuncSetAttribute(base_chol_inv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(base_smem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(inblock_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(u1_smem));
    if (e == cudaSuccess) e = cudaMemsetAsync(w.V, 0, 6 * dd * sizeof(float), st);  // V and VT (+ splits) triangles
    if (e == cudaSuccess) e = cudaMemsetAsync(w.bad, 0, sizeof(int), st);
    if (e != cudaSuccess) return cuda_fail(e, "tb_obs_sparsegpt setup");
    diag_sum_kernel<<<1, 1024, 0, st>>>(H, d, dsum);
    reverse_damp_kernel<<<148 * 16, 256, 0, st>>>(H, d, dsum, damp_frac, w.A, w.A_hi, w.A_lo);
    rc = check_launch("hessian prep");
    if (!rc) rc = chol(w, 0, d, st, base_smem);
    if (!rc) rc = trtri(w, 0, d, st);
    // Ut (lower) = (P V P)^T into A's buffers (A is no longer needed).
    float *Ut = w.A, *Ut_hi = w.A_hi, *Ut_lo = w.A_lo;
    if (!rc) {
        reverse_transpose_kernel<<<dim3(d / 32, d / 32), dim3(32, 8), 0, st>>>(w.V, d, Ut, Ut_hi, Ut_lo);
        rc = check_launch("reverse_transpose_kernel");
    }
    for (int i1 = 0; !rc && i1 < d; i1 += kB) {
        inblock_kernel<<<r / 8, 256, u1_smem, st>>>(W, r, d, i1, Ut, n_keep, mask, E_hi, E_lo);
        if ((rc = check_launch("inblock_kernel"))) break;
        const int i2 = i1 + kB;
        if (i2 < d) {  // W[:, i2:] -= E U[i1:i2, i2:] = E (Ut[i2:, i1:i2])^T
            umma::GemmOut o{};
            o.C = W + i2; o.ldc = d;
            o.Cin = W + i2; o.ldcin = d;
            o.alpha = -1.0f; o.beta = 1.0f;
            rc = umma::gemm_nt(umma::kTF32x3, {E_hi, E_lo, kB},
                               {Ut_hi + static_cast<size_t>(i2) * d + i1, Ut_lo + static_cast<size_t>(i2) * d + i1, d},
                               r, d - i2, kB, o, st);
        }
    }
    int bad = 0;
    if (!rc && ut_out) {
        e = cudaMemcpyAsync(ut_out, Ut, dd * sizeof(float), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) rc = cuda_fail(e, "tb_obs_sparsegpt Ut copy");
    }
    if (!rc) {
        e = cudaMemcpyAsync(&bad, w.bad, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "tb_obs_sparsegpt sync");
    }
    if (!rc) {
        const int ge = umma::gemm_take_error(st);
        if (ge) rc = fail(TB_ERR_TIMEOUT, "a tcgen05 GEMM pipeline wait expired");
    }
    if (!rc && bad) rc = fail(TB_ERR_CONFIG, "H + lambda I is not positive definite in FP32 (a Cholesky pivot <= 0)");
    return rc;
}

// tcgen05 (5th-generation tensor core) GEMM for sm_100a, NT form:
//   C[M, N] = alpha * A[M, K] * B[N, K]^T + beta * Cin[M, N]
// A and B row-major with K contiguous (both operands "K-major").
//
// One CTA per 128 x 128 output tile, 192 threads:
//   warp 4 lane 0  issues TMA loads (cp.async.bulk.tensor.2d, 128-byte swizzle)
//                  of 128-row x 128-byte K-slices into a STAGES-deep ring;
//   warp 5 lane 0  issues tcgen05.mma into one of two 128 x 128 FP32
//                  accumulators in tensor memory (TMEM, 2 x 128 columns),
//                  switching buffer every 4 K-slices, and commits each stage
//                  back to the producer through an mbarrier;
//   warps 0-3      read each finished buffer with tcgen05.ld (warp w owns TMEM
//                  lanes 32w..32w+31 = output rows), add it into FP32 registers
//                  with round-to-nearest (the tensor core's own accumulation
//                  truncates), and apply the epilogue through shared memory
//                  (the drained operand ring), one coalesced row at a time.
// Kinds:
//   kTF32x3  FP32-accurate product from TF32 tensor cores: every operand is
//            given as hi = tf32(x) and lo = x - hi, and the tile accumulates
//            hi*hi + hi*lo + lo*hi (the lo*lo term is below FP32 rounding).
//   kBF16    BF16 x BF16 with FP32 accumulation (exact products).
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// and leaves after a bounded drain (no trap, no endless spin).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace tb {
namespace umma {

enum Kind { kTF32x3 = 0, kBF16 = 1 };

struct GemmOut {
    float* C;            // output, row-major, ldc
    long long ldc;
    const float* Cin;    // beta * Cin added (may alias C); ignored when beta == 0
    long long ldcin;
    float* C_hi;         // optional tf32 hi/lo split of the output (same ld as C_split)
    float* C_lo;
    long long ld_split;
    float* Ct;           // optional transposed copy of the output, ldct
    long long ldct;
    float* Ct_hi;        // optional tf32 hi/lo split of the transposed copy (same ldct)
    float* Ct_lo;
    float alpha, beta;
    int lower_only;      // compute only tiles with tile_row >= tile_col
    int tri_a;           // A is square and triangular (M == K): 1 = upper, so output tile row
                         // t runs over K tiles t.. only; 2 = lower, K tiles ..t only; 0 = dense.
                         // Products on CTA pairs (M % 256 == 0, K >= 512) run a pair of row
                         // tiles over the union of their ranges, so the 128-block next to
                         // the triangle's diagonal blocks (below for upper, right for lower)
                         // must be zero.
};

// Operand view for the host wrapper: row-major [rows, K] with leading dimension ld (elements).
struct Operand {
    const void* hi;      // FP32 hi part (kTF32x3) or BF16 data (kBF16)
    const void* lo;      // FP32 lo part (kTF32x3), unused for kBF16
    long long ld;
};

// Launches the NT GEMM on `stream`.  M, N multiples of 128; K a multiple of 32
// (kTF32x3) or 64 (kBF16); operand bases 16-byte aligned, ld * elem % 16 == 0.
int gemm_nt(Kind kind, const Operand& A, const Operand& B, int M, int N, int K, const GemmOut& out,
            cudaStream_t stream);

// Error code recorded by the last gemm_nt launches on this device since the
// previous call (0 = none; 1 = a pipeline wait expired); resets it.
int gemm_take_error(cudaStream_t stream);

}  // namespace umma
}  // namespace tb

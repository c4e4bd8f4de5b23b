/* tb_kernels.h - C ABI of the B200 (sm_100a) pruning kernels.
 *
 * Drop-in replacement for the reference's kernel boundary:
 *   include/tensorbit/core/kernels.hpp:24-124   (7 C++ launch_* declarations)
 *   src/kernels.cu:338-435                      (their CUDA launchers)
 *   src/kernels_stubs.cpp:13-63                 (their CPU-build no-op stubs)
 * plus the host-side loops of the pruners that the reference never moved to a
 * device (include/tensorbit/core/ehap.hpp, coring.hpp), so that one call can do
 * the whole per-tensor score -> N:M mask -> pack pass.
 *
 * Conventions (all entry points):
 *   - extern "C", plain pointers and sizes; no C++ or torch types.
 *   - Every function returns an int status: TB_OK (0) or a negative TB_ERR_*.
 *     Nothing aborts the process (the reference aborts via CUDA_CHECK,
 *     common.hpp:38-49); the text of the last error is in tb_last_error().
 *   - `stream` is a cudaStream_t passed as void*; NULL means the legacy default
 *     stream.  Launches are asynchronous; results are ready after the stream
 *     synchronises.  Size/argument checks happen on the host before launch.
 *   - Device pointers are owned by the caller unless stated otherwise.
 *   - Floating-point results reproduce the reference's CPU expression trees
 *     bit for bit (IEEE round-to-nearest, no fused multiply-add); masks
 *     reproduce the reference CPU path's selection, ties included.
 *   - Without a CUDA device every compute call returns TB_ERR_NO_DEVICE; there
 *     is no CPU fallback.
 */
#ifndef TB_KERNELS_H
#define TB_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_ABI_VERSION 1

/* ---- status codes ------------------------------------------------------ */
enum {
    TB_OK              = 0,
    TB_ERR_SHAPE       = -1, /* sizes disagree or numel % M != 0 (EHAPError/CORINGError::kShapeMismatch) */
    TB_ERR_ZERO_SIZE   = -2, /* empty tensor (kZeroSizeTensor)                                        */
    TB_ERR_CONFIG      = -3, /* bad N:M (CORINGError::kInvalidNMConfig) or sparsity (EHAPError::kInvalidConfig) */
    TB_ERR_CUDA        = -4, /* CUDA runtime error; see tb_last_error()                               */
    TB_ERR_TIMEOUT     = -5, /* a bounded device-side wait gave up                                    */
    TB_ERR_UNSUPPORTED = -6, /* combination not implemented (e.g. M > 8: masks are one byte per group) */
    TB_ERR_ARG         = -7, /* null pointer, bad enum value, misaligned pointer                      */
    TB_ERR_NO_DEVICE   = -8, /* no CUDA device visible                                                */
    TB_ERR_CAPACITY    = -9  /* request exceeds a fixed capacity of the entry point                   */
};

/* ---- enumerations (values equal the reference's enum values) ----------- */
enum { TB_F32 = 0, TB_F16 = 1, TB_BF16 = 2 };                 /* TBHeader::precision codes, serialization.hpp:48 */
enum { TB_IMP_OBD = 0, TB_IMP_OBS = 1, TB_IMP_NORMALIZED = 2 }; /* ImportanceMode, ehap.hpp:49-53 */
enum { TB_MASK_TOPN = 0, TB_MASK_OPTIMAL = 1, TB_MASK_ITERATIVE = 2 }; /* MaskStrategy, coring.hpp:37-41 */
enum { TB_REDIST_NONE = 0, TB_REDIST_PROPORTIONAL = 1, TB_REDIST_UNIFORM = 2 }; /* RedistMode, coring.hpp:43-47 */

/* ---- library / device plumbing ----------------------------------------- */
int         tb_abi_version(void);
const char* tb_last_error(void);               /* thread-local text of the last failure */
int         tb_device_count(int* count);
int         tb_set_device(int device);
int         tb_malloc(void** ptr, size_t bytes);  /* device memory for TensorDense (tensor.hpp:97-104) */
int         tb_free(void* ptr);
/* Page-locked host memory (usable from every device), for host buffers that
 * feed tb_memcpy_h2d / tb_score_mask_pack_host at full PCIe speed. */
int         tb_host_alloc(void** ptr, size_t bytes);
int         tb_host_free(void* ptr);
int         tb_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
int         tb_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
int         tb_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
int         tb_memset(void* dst, int value, size_t bytes, void* stream);
int         tb_stream_sync(void* stream);
/* Peer memory between the processes (or devices) of one node, for the
 * sample-split pass below.  No reference counterpart: the reference prunes in
 * one process and names multi-GPU collectives as future work
 * (docs/CLOUD.md:155-169).  tb_ipc_handle exports a tb_malloc allocation as
 * TB_IPC_HANDLE_BYTES opaque bytes; another process passes those bytes to
 * tb_ipc_open and gets a device pointer to the same memory, readable by its
 * kernels over NVLink, until tb_ipc_close.  Within one process,
 * tb_enable_peer_access lets the current device read peer_device's memory
 * (returns TB_OK when already enabled or when peer_device is the current one). */
#define TB_IPC_HANDLE_BYTES 64
int         tb_ipc_handle(const void* dev_ptr, void* handle_out);
int         tb_ipc_open(const void* handle, void** dev_ptr_out);
int         tb_ipc_close(void* dev_ptr);
int         tb_enable_peer_access(int peer_device);
/* Builds the per-device tie tables needed by TB_MASK_TOPN / TB_MASK_ITERATIVE
 * for this (n, m) on the current device.  Calls that need them build them on
 * first use; call this first if the stream will later be captured. */
int         tb_prepare_nm(int n, int m);

/* ---- legacy launchers: kernels.hpp:24-124, same arguments -------------- */
/* F[i] = sum_b g[b*N+i]^2 (kernels.hpp:24-28; not called by the reference pruners). */
int tb_fisher_diagonal(const float* gradients, float* fisher_diag, size_t B, size_t N, void* stream);
/* F[i] = F[i] + (alpha*g[i])*g[i] (kernels.hpp:38-42).  Composed with
 * tb_fisher_beta_decay this is bit-identical to the reference's host EMA step
 * F = beta*F + (alpha*(1-beta))*g*g (ehap.hpp:194-197). */
int tb_fisher_accumulate(float* fisher_diag, const float* gradients, size_t N, float alpha, void* stream);
/* F[i] = beta*F[i] (kernels.hpp:51-54). */
int tb_fisher_beta_decay(float* fisher_diag, float beta, size_t N, void* stream);
/* OBD importance s = w*w*(F+damping), or w*w when F is NULL (kernels.hpp:65-70). */
int tb_ehap_importance(const float* weights, const float* fisher_diag, float* importance, size_t N,
                       float damping, void* stream);
/* 2:4 top-N mask, one byte per group (kernels.hpp:85-88). */
int tb_nm_mask_2_4(const float* importance, uint8_t* mask_out, size_t N, void* stream);
/* n:m top-N mask, one byte per group (kernels.hpp:101-106); m <= 8. */
int tb_nm_mask_generic(const float* importance, uint8_t* mask_out, size_t N_elements, int group_n,
                       int group_m, void* stream);
/* Zero w[i] where bit (i % m) of mask[i / m] is clear (kernels.hpp:120-124). */
int tb_apply_mask(float* weights, const uint8_t* mask, size_t N, int group_m, void* stream);

/* ---- stage entry points (the pruners' loops, on the device) ------------ */
/* load_safetensor's element widening (src/main.cpp:204-250): BF16 exactly, F16
 * as the reference decodes it (exponent 0 keeps the fraction in an FP32 with
 * exponent 0), F32 copied. */
int tb_decode_to_f32(const void* in, int dtype, float* out, size_t N, void* stream);
/* One EHAPPruner::accumulate_fisher call (ehap.hpp:148-201) over N gradients of
 * dtype g_dtype: first_step != 0 gives F = (alpha*g)*g, otherwise
 * F = beta*F + ((alpha*(1-beta))*g)*g with the reference's float rounding. */
int tb_fisher_ema_step(float* fisher, const void* gradients, int g_dtype, size_t N, float alpha,
                       float beta, int first_step, void* stream);
/* Sample-split Fisher: F (+)= sum_s weights[s] * g_s^2 over S samples of dtype
 * g_dtype ([S][g_stride], g_stride 0 = N); weights is a host array.  With the
 * EMA weights c_0 = alpha beta^(S-1), c_t = alpha (1-beta) beta^(S-1-t) this is
 * the accumulate_fisher recurrence (ehap.hpp:190-197) regrouped, so ranks holding
 * disjoint samples can sum their partials with one all-reduce.  Agrees with the
 * serial recurrence to FP32 rounding (different association), not bit for bit.
 * accumulate == 0 overwrites F. */
int tb_fisher_weighted_sum(float* fisher, const void* gradients, int g_dtype, size_t S, size_t g_stride,
                           size_t N, const float* weights, int accumulate, void* stream);
/* EHAPPruner::compute_importance (ehap.hpp:206-285) for all three modes; F may be
 * NULL (no Fisher state: s = w*w).  Weights of dtype w_dtype are widened as the
 * reference's safetensors loader does (src/main.cpp:213-245). */
int tb_importance(const void* weights, int w_dtype, const float* fisher, float* importance,
                  size_t N, float damping, int mode, void* stream);
/* CORINGPruner::generate_nm_mask (coring.hpp:90-165): strategy TB_MASK_*,
 * `rounds` swap-refine rounds, optional per-group |score| sort (permute_weights).
 * Writes N/m bytes. */
int tb_nm_mask(const float* importance, uint8_t* mask_out, size_t N, int n, int m, int strategy,
               int rounds, int permute, void* stream);
/* CORINGPruner::redistribute (coring.hpp:228-294) of the weights as they are now. */
int tb_redistribute(float* weights, const uint8_t* mask, const float* importance, size_t N, int m,
                    int mode, void* stream);

/* EHAPPruner::select_pruning_mask (ehap.hpp:290-329): keep = (size_t)(sparsity *
 * (float)N) (at least 1); the threshold is the (N-keep)-th smallest score and
 * every score >= it is kept.  Writes 1 byte per element to mask_out (may be
 * NULL), the threshold and the number of pruned elements to host memory, and
 * synchronises the stream.  keep >= N keeps everything (threshold 0, pruned 0).
 * Scratch: about 16 KB of device memory, stream-ordered from a pool the
 * library keeps per device (its memory is retained between calls). */
int tb_threshold_select(const float* scores, size_t N, float sparsity, uint8_t* mask_out,
                        float* threshold_out, uint64_t* pruned_out, void* stream);
/* EHAPPruner::apply_mask (ehap.hpp:334-362): zero weights[i] where mask[i] == 0
 * (1 byte per element); the number zeroed goes to *pruned_out (host, may be
 * NULL; when given the call synchronises the stream). */
int tb_ehap_apply_mask(float* weights, const uint8_t* mask, size_t N, uint64_t* pruned_out, void* stream);
/* apply_fisher_normalization (ehap.hpp:720-731): F /= ||F||_2 with the
 * reference's serial float sum (one device thread; off by default). */
int tb_fisher_normalize(float* fisher, size_t N, void* stream);
/* EHAPPruner::compensate_weights (ehap.hpp:367-403): mode 0 none, 1 bias (serial
 * sum of pruned weights added to the last weight), 2 redistribution over groups
 * of 8 in proportion to the kept scores. */
int tb_compensate(float* weights, const uint8_t* mask, const float* importance, size_t N, int mode,
                  void* stream);

/* EHAPPruner::prune_block_obs (ehap.hpp:502-704): blockwise OBS with
 * H = diag(F + damping) + U U^T over contiguous blocks of `block` weights.
 * U holds K gradient snapshots (hist: host array of K device pointers, oldest
 * first, K <= 16) weighted exp(-(K-1-k)/2), or sqrt(off_diag_alpha) * w when
 * K == 0.  Per-block prune targets follow the reference's exp(-4 rel)
 * allocation; each block is pruned greedily by w_i^2 / [H^-1]_ii with OBS
 * updates and rank-1 deflation.  Weights are updated in place; the number
 * pruned goes to *pruned_out (host) and the call synchronises the stream.
 * Scratch (the per-block importances, targets and launch order, ~12 bytes per
 * block) is stream-ordered from the library's per-device pool (memory
 * retained between calls, so later calls allocate nothing from the driver);
 * the launch setup per (block, snapshots) is queried once per device.
 * block <= 224 (one thread per row; a block's downdate columns, up to
 * block - 1 of them, live in shared memory). */
int tb_block_obs(float* weights, const float* fisher, const float* const* hist, int K, size_t N,
                 size_t block, float sparsity, float damping, float off_diag_alpha, uint64_t* pruned_out,
                 void* stream);
/* Diagnostics, no reference counterpart: the phase times (milliseconds) of
 * this host thread's last tb_block_obs call.  ms_out[0] = block importance on
 * the device and its copy to the host (CUDA events), [1] = host target
 * allocation and launch planning (host clock; the stream is idle meanwhile),
 * [2] = target upload and the greedy kernels (CUDA events), [3] = the whole
 * call (host clock).  Writes min(n, 4) values. */
int tb_block_obs_phase_times(float* ms_out, int n);

/* ---- stage 3 building blocks: tcgen05 tensor-core GEMM (sm_100a) --------- */
/* Splits x into hi = tf32(x) (round to nearest) and lo = x - hi, the operand
 * form of the FP32-accurate TF32 GEMM below. */
int tb_split_tf32(const float* x, float* hi, float* lo, size_t n, void* stream);
/* C[M,N] = alpha * A[M,K] * B[N,K]^T + beta * Cin, A and B row-major FP32 given
 * as hi/lo pairs (tb_split_tf32); products hi*hi + hi*lo + lo*hi on TF32 tensor
 * cores, accumulated in tensor memory in groups of 128 K and summed in FP32
 * registers (round to nearest).  M, N multiples of 128, K of 32; 16-byte
 * aligned operands with ld*4 % 16 == 0.  lower_only writes only the 128x128
 * tiles on or below the diagonal.  M % 256 == 0 and K >= 512 run on CTA pairs
 * (tcgen05 cta_group::2, 256x256 tiles where N % 256 == 0), the rest on
 * single CTAs (128x128 tiles). */
int tb_gemm_nt_tf32x3(const float* a_hi, const float* a_lo, long long lda, const float* b_hi,
                      const float* b_lo, long long ldb, int M, int N, int K, float alpha, float beta,
                      const float* c_in, long long ldcin, float* c, long long ldc, int lower_only,
                      void* stream);
/* Same with BF16 operands (K a multiple of 64), FP32 accumulation. */
int tb_gemm_nt_bf16(const void* a, long long lda, const void* b, long long ldb, int M, int N, int K,
                    float alpha, float beta, const float* c_in, long long ldcin, float* c, long long ldc,
                    int lower_only, void* stream);
/* TB_ERR_TIMEOUT if a bounded pipeline wait inside a GEMM launched since the
 * last call expired (the kernel then skipped its output); synchronises. */
int tb_gemm_status(void* stream);

/* ---- stage 3: column-block exact OBS against calibration activations ----- */
/* No counterpart in the reference (docs/EHAP.md:248-250 lists activation
 * Hessians as missing); the OBS saliency and update follow ehap.hpp:683-691.
 * H = X^T X / n from X^T given as BF16 [d][n] (row-major, d % 128 == 0,
 * n % 64 == 0); only the 128x128 tiles on or below the diagonal are written. */
int tb_obs_hessian(const void* xt_bf16, int d, int n, float* H, void* stream);
/* H = scale * X^T X over the n tokens given (same layout and tiles as
 * tb_obs_hessian).  With calibration tokens split across ranks, each rank
 * passes its own tokens and scale = 1 / (total tokens); the ranks' results
 * summed (one all-reduce) give the Hessian of all tokens.  No reference
 * counterpart: the reference has no activation Hessian. */
int tb_obs_hessian_scaled(const void* xt_bf16, int d, int n, float scale, float* H, void* stream);
/* Prunes W [r][d] (FP32, in place; r, d multiples of 128) to N:4 against H
 * (lower tiles valid, e.g. from tb_obs_hessian): lambda = damp_frac *
 * mean(diag H) is added to the diagonal, U = chol_upper((H + lambda I)^-1) is
 * formed on tensor cores (3xTF32 tcgen05 GEMMs), and columns are swept in
 * blocks of 128: per group of 4 the 4 - n_keep smallest w^2 / U_qq^2 are
 * pruned and each pruned column's error updates the later columns of its row
 * (inside the block directly, beyond it through tcgen05 GEMMs over the errors
 * of whole column ranges).  Rows are independent, so a row range of W may be
 * pruned on its own (each rank of a row split passes its rows).  mask gets
 * r*d/4 bytes (bit k = keep column 4g+k, the .tb convention).  ut_out (d x d,
 * may be NULL) receives U^T.  A workspace of 7.5 d^2 + 3 r d floats is
 * allocated on first use and kept per device for later calls (grow-only;
 * ~6.9 GB at d = 14336, r = 4096), so calls on one device must not overlap;
 * two internal streams per device carry the parts of the factorisation and
 * the sweep that run beside the caller's stream.  Synchronises the stream.
 * TB_ERR_CONFIG if H + lambda I is not positive definite in FP32;
 * TB_ERR_TIMEOUT if an internal bounded wait expired. */
int tb_obs_sparsegpt(float* W, int r, int d, const float* H, float damp_frac, int n_keep, int m,
                     uint8_t* mask, float* ut_out, void* stream);
/* Diagnostics, no reference counterpart: phase times (milliseconds, CUDA
 * events on the internal chain stream) of this host thread's last successful
 * tb_obs_sparsegpt call: [0] damping and the reversed copy of H, [1] the
 * factorisation (its chain of dependent steps), [2] the column sweep up to
 * its last in-block step, [3] all three.  Writes min(n, 4) values. */
int tb_obs_sparsegpt_phase_times(float* ms_out, int n);

/* ---- fused score -> mask -> pack pass ------------------------------------ */
/* One pass over a tensor: Fisher EMA over S gradient samples, importance,
 * CORING N:M mask, apply, redistribution, and emission of the .tb weight and
 * mask sections.  Equivalent to the reference sequence
 *   accumulate_fisher x S -> compute_importance -> CORINGPruner::prune
 *   -> generate_nm_mask                       (src/main.cpp:375,397-409)
 * without the EHAP global pre-prune. */
typedef struct tb_prune_args {
    uint32_t struct_size;      /* sizeof(tb_prune_args) */
    /* inputs (device pointers) */
    const void*  weights;      /* [N] of w_dtype                                         */
    int32_t      w_dtype;
    int32_t      g_dtype;
    const void*  grads;        /* [S, g_stride] of g_dtype, sample-major; NULL iff S == 0 */
    uint64_t     S;            /* gradient samples                                       */
    uint64_t     N;            /* elements                                               */
    uint64_t     g_stride;     /* elements between samples; 0 means N                    */
    const float* fisher_in;    /* [N] Fisher state after fisher_steps_in steps, or NULL   */
    uint64_t     fisher_steps_in;
    /* EHAPConfig subset (ehap.hpp:70-93) */
    float        alpha;        /* accumulate_fisher's alpha (tb-prune passes 0.01)        */
    float        beta;         /* ema_decay                                              */
    float        damping;      /* lambda                                                 */
    int32_t      importance_mode;
    int32_t      use_fisher;   /* use_diagonal_fisher                                    */
    /* CORINGConfig subset (coring.hpp:49-69) */
    int32_t      nm_n, nm_m;
    int32_t      mask_strategy;
    int32_t      iterative_rounds;
    int32_t      redist_mode;
    int32_t      permute;
    /* outputs (device pointers) */
    float*       w_out;        /* [N] FP32 pruned weights = .tb weight section           */
    uint8_t*     mask_out;     /* [N/m] packed groups     = .tb mask section             */
    float*       fisher_out;   /* [N] or NULL                                            */
    float*       scores_out;   /* [N] or NULL                                            */
    unsigned long long* near_ties; /* device counter incremented per near-tie group, or NULL */
} tb_prune_args;

int tb_score_mask_pack(const tb_prune_args* args, void* stream);

/* tb-prune's per-tensor sequence (src/main.cpp:372-409) in three device
 * passes: EHAPPruner::accumulate_fisher x S + compute_importance
 * (ehap.hpp:148-285), the one-shot global select and apply (ehap.hpp:290-362,
 * 425-439: keep = (size_t)(sparsity * (float)N), at least 1; every score >= the
 * (N-keep)-th smallest kept, the rest zeroed), compute_importance again on the
 * pruned weights, and CORINGPruner::prune + generate_nm_mask (coring.hpp:
 * 90-313) with the .tb sections written - bit-identical to running those
 * calls one after another (compensation none, Fisher normalisation off, as
 * tb-prune configures them).  Pass 1 writes F (fisher_out, required when a
 * Fisher state exists) and the scores (scores_out, required); the radix select
 * ranks those scores; pass 2 recomputes each score, applies the threshold and
 * runs CORING on the recomputed importance, writing w_out, mask_out and
 * scores_out (now the importance CORING ranked).  *threshold_out (0 when
 * everything is kept), *ehap_pruned_out (weights the threshold zeroed) and
 * *coring_pruned_out (the analytic (N/M)*(M-N) of coring.hpp:192,222) are
 * host values, any may be NULL; synchronises the stream when threshold_out or
 * ehap_pruned_out is given.  Scratch: about
 * 16 KB, stream-ordered from the library's per-device pool.  Sparsity outside (0, 1) -> TB_ERR_CONFIG before any
 * N:M check, as the reference's EHAP stage fails first. */
int tb_prune_one_shot_nm(const tb_prune_args* args, float sparsity, float* threshold_out,
                         uint64_t* ehap_pruned_out, uint64_t* coring_pruned_out, void* stream);

/* tb_prune_one_shot_nm without the host wait: the threshold and the EHAP count
 * are copied, in stream order, to threshold_dst / ehap_pruned_dst (device
 * memory or pinned host memory, either may be NULL) and are valid once the
 * stream reaches that point, so a caller can queue many tensors and read their
 * counts after one synchronisation.  *coring_pruned_out is a host value as
 * above.  Outputs, errors and scratch as tb_prune_one_shot_nm. */
int tb_prune_one_shot_nm_async(const tb_prune_args* args, float sparsity, float* threshold_dst,
                               uint64_t* ehap_pruned_dst, uint64_t* coring_pruned_out, void* stream);

/* Sample split, producer side: this rank's partial Fisher
 *   F_part[i] = sum over its S samples of weights[s] * g_s[i]^2
 * (from +0, samples in order: the arithmetic of tb_fisher_weighted_sum, bit
 * for bit) for all N elements, each element stored to the rank that owns it:
 * ranks r = 0..n_ranks-1 own [starts[r], starts[r+1]) (host array of
 * n_ranks + 1 offsets from 0 to N, inner ones multiples of 8) and element
 * starts[r] lands at dest[r][0] (host array of device pointers: a peer's
 * buffer mapped with tb_ipc_open, or this device's own).  The pass visits the
 * elements starting with owner start_owner's range (cyclically): ranks that
 * start at different owners (e.g. rank + 1) spread their remote stores over
 * the peers instead of all writing to one peer at a time.  The stores to other
 * GPUs travel over NVLink inside the pass, so the exchange of an all-reduce
 * becomes writes of (P-1)/P of the partial, and each owner then reads the P
 * partials of its range from its own memory (tb_score_mask_pack_peer with
 * local pointers).  No counterpart in the reference (one process, no
 * collectives; docs/CLOUD.md:155-169).  S <= 128 per call (TB_ERR_CAPACITY). */
int tb_fisher_partial_scatter(const void* gradients, int g_dtype, size_t S, size_t g_stride, size_t N,
                              const float* weights, int n_ranks, const uint64_t* starts, float* const* dest,
                              int start_owner, void* stream);

/* Sample-split pass: the reduction of the ranks' partial Fisher sums fused
 * into the score -> mask -> pack pass (a reduce-scatter over peer memory).
 * When the S calibration gradients of a tensor are split across P ranks, each
 * rank forms its partial F_r = sum over its samples of c_t g_t^2
 * (tb_fisher_weighted_sum with the EMA weights, accumulate_fisher's
 * recurrence of ehap.hpp:190-197 regrouped) for all elements; then every rank
 * calls this on its own group range, reading the P partials of that range
 * directly (its own and the peers', mapped with tb_ipc_open or peer access):
 *   F[i] = ((partials[0][i] + partials[1][i]) + ...) + partials[P-1][i]
 * (FP32 adds in index order, the same on every rank), then importance, mask,
 * apply, redistribution and the .tb sections exactly as tb_score_mask_pack
 * with that Fisher state.  args: as for tb_score_mask_pack with S == 0 and
 * fisher_in == NULL; fisher_steps_in > 0 (the samples the partials cover).
 * partials: host array of n_partials (1..8) device pointers, each already
 * offset to this launch's first element.  The partials must be complete
 * before the launch (e.g. a stream-ordered collective or event between the
 * producers and this call) and must not be overwritten until every rank's
 * call has finished.  Not bit-identical to the serial recurrence (different
 * association); masks can differ only where scores nearly tie. */
int tb_score_mask_pack_peer(const tb_prune_args* args, const float* const* partials, int n_partials,
                            void* stream);

/* Same pass with every pointer in args a HOST pointer (pinned memory is
 * fastest).  The library stages chunks through device buffers it allocates
 * (kept per device and grown on demand), overlapping host->device copies, the
 * kernel and device->host copies on several internal streams, and returns when
 * the outputs are in host memory.  Safe to call from several host threads:
 * calls on one device are serialised by a per-device lock held for the whole
 * call (a second caller waits), calls on different devices run in parallel. */
int tb_score_mask_pack_host(const tb_prune_args* args);

/* tb_score_mask_pack_host for callers that cannot allocate device memory.
 * No counterpart in the reference (its pruners run on host memory only).
 * Who needs it: a process whose GPU memory is already reserved by another
 * allocator - a framework's caching pool, or a server that fixes its memory
 * budget at start-up - where a cudaMalloc from this library would fail or
 * fragment that pool.  This entry point calls no cudaMalloc / cudaFree: it
 * stages chunks through a static 16 MiB device array that every GPU loading
 * the library holds until the process exits.  Results are identical to
 * tb_score_mask_pack_host.
 *   - Limit: one chunk of 16*M elements with all S samples must fit in the
 *     16 MiB array; larger requests return TB_ERR_CAPACITY with the sizes.
 *   - Top-N / iterative masks need the (N, M) tie table already on the
 *     device (tb_prepare_nm once, where allocation is allowed); otherwise
 *     TB_ERR_UNSUPPORTED.  TB_MASK_OPTIMAL needs no table.
 *   - The first call on a device resolves the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - Runs on the legacy default stream and returns when the outputs are in
 *     host memory.  All calls share the one array (it keeps the last call's
 *     contents; the tie counter is cleared per call): calls that overlap on
 *     the GPU, e.g. from two host threads, race and must be serialised. */
int tb_score_mask_pack_host_noalloc(const tb_prune_args* args);

#ifdef __cplusplus
}
#endif
#endif /* TB_KERNELS_H */

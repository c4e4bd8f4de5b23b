/* CPU restatement ("port" oracle) of the reference pruning path.
 *
 * TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py load this library, and only to check or time
 * against it; the shipped library never links it.
 *
 * Status codes follow the reference's error enums so a test can compare them
 * with oracle/_ref directly: 0 = ok; 100 + EHAPError / CORINGError for the
 * first failing call of a sequence (kShapeMismatch=1, kZeroSizeTensor=2,
 * kInvalidConfig/kInvalidNMConfig=3, kCudaNotAvailable=4). */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int port_fisher(const float* grads, size_t S, size_t N, float alpha, float beta, int use_fisher,
                float* F_out);
int port_importance(const float* grads, size_t S, const float* w, size_t N, float alpha,
                    float beta, float damping, int mode, int use_fisher, int normalize,
                    float* s_out);
int port_nm_mask(const float* s, size_t N, int n, int m, int strategy, int rounds, int permute,
                 int hw_layout, uint8_t* mask_out);
int port_nm_mask_status(size_t N_scores, size_t N_mask, int n, int m);
int port_coring_prune(const float* s, float* w_inout, size_t N, int n, int m, int strategy,
                      int rounds, int redist, int permute, int hw_layout, uint8_t* mask_out,
                      size_t* pruned_out);
int port_apply_redistribute(float* w_inout, const uint8_t* mask, const float* s, size_t N, int n,
                            int m, int redist, int do_apply, size_t* pruned_out);
int port_select_mask(const float* s, size_t N, float sparsity, uint8_t* mask_out,
                     size_t* pruned_out);
int port_pipeline(float* w_inout, const float* grads, size_t S, size_t N, float alpha, float beta,
                  float damping, int imp_mode, int use_fisher, int normalize, int ehap_strategy,
                  float sparsity, int prune_rounds, const float* hist, size_t K, int n, int m,
                  int mask_strategy, int rounds, int redist, int permute, float* F_out,
                  float* s_out, uint8_t* mask_out, size_t* ehap_pruned, size_t* coring_pruned);
void port_tb_header(uint8_t out[4096], uint32_t n, uint32_t m, uint64_t num_weights,
                    uint64_t num_mask_bytes, uint32_t elem_size);
void port_decode_half(const uint16_t* in, size_t n, int is_bf16, float* out);
void port_mock_tensor(size_t N, float* w_out, float* g_out);
size_t port_near_ties(const float* s, size_t N, int n, int m);
void port_compensate(float* w, const uint8_t* mask, const float* s, size_t N, int mode);
int port_block_obs(float* w_inout, const float* grads, size_t S, const float* hist, size_t K, size_t N,
                   size_t block, float sparsity, float damping, float off_alpha, float fisher_alpha,
                   int use_fisher, size_t hist_size, size_t* pruned_out);
void port_topn_group(const float* vals, int n, int m, uint8_t* mask_out);

#ifdef __cplusplus
}
#endif

/* libb200lmhead.so -- the grouped MoE GEMM of the expert cache's consumer for B200 (sm_100a):
 * MXFP4 expert weights (e2m1 codes, one E8M0 exponent per 32 K-values) times per-token FP8
 * activations, over the blocks moe_align_block_size / r4d_lru_fused lay out (16 rows per
 * block, one expert per block). The reference's MoE layer runs it twice per projection, once
 * over the resident (hot) experts and once over the others (cold), into one output
 * (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff L584-606).
 *
 * Packed layouts (B200 formats; codes and scales are the checkpoint's):
 *   wq   uint8 [E][N/16][K/32][32 lanes][8 B]  the codes in mma.sync A-fragment order (byte
 *        4 h + r of lane 4 g + t: row g + 8 (r & 1), k = 16 h + 2 t + 8 (r >> 1) low nibble,
 *        k + 1 high nibble)
 *   ws   uint8 [E][N/16][16][K/32]            E8M0 exponents (the checkpoint's [E, N, K/32])
 *   wref uint8 [E][N]                         per-row maximum exponent (the reference's
 *                                             argument; accepted, not read)
 */
#ifndef B200_MOE_GEMM_H
#define B200_MOE_GEMM_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces the closed r4d_gemm_moe_mxfp4a8_nt_b16 (ABI as the reference binds it,
 * r4d_mxfp4_moe.py.lru.diff L454-500; argument order of tests/k1/moe_ref_harness.py:55-56,
 * 221-225): for every block b < *num_post_pad / 16 with e = expert_ids[b] >= 0 and every row
 * i = sorted_ids[16 b + r] < mtk,
 *   c[i, n] = bf16(topk_weights[i] * x_scale[i / top_k] * sum_k qx[i / top_k, k] * W_e[n, k])
 * with W_e[n, k] = e2m1 * 2^(e8m0 - 127); topk_weights may be 0 (none). qx e4m3 [tokens, K],
 * x_scale fp32 [tokens], c bf16 [mtk, N]; rows not named are not written. em = capacity of
 * sorted_ids (>= 16), K % 32 == 0, N % 16 == 0. wv / sk / npw (gfx1201 launch knobs) are
 * accepted and ignored. Returns nothing, like the reference; the last call's status is
 * r4d_gemm_moe_mxfp4a8_nt_b16_last_error(): 0, -1 em < 16 / mtk < 0 / top_k < 1,
 * -2 N % 16, -3 K % 32 or K too deep for shared memory, -10 misaligned qx / wq / ws, else a
 * CUDA error. Allocates nothing; the device count of live blocks makes it graph capturable. */
void r4d_gemm_moe_mxfp4a8_nt_b16(long qx, long x_scale, long wq, long ws, long wref, long c,
                                 long sorted_ids, long expert_ids, long num_post_pad, long topk_weights,
                                 int em, int mtk, int top_k, int K, int N, int wv, int sk, int npw,
                                 long stream);
int r4d_gemm_moe_mxfp4a8_nt_b16_last_error(void);
int r4d_gemm_moe_mxfp4a8_nt_b16_block(void);  /* 16 rows per block */
int r4d_gemm_moe_mxfp4a8_nt_b16_group(void);  /* 32 K-values per E8M0 exponent */

/* The projection's two calls (r4d_mxfp4_moe.py.lru.diff _gemm_split, L584-606) in ONE launch:
 * the hot call over the resident slots' copies wq_hot with r4d_lru_fused's by-slot blocks
 * (sorted_hot / eids_hot / npad_hot, capacity em_hot) and the cold call over the full tensors
 * wq_cold with its by-expert blocks, into the same c. Same result as the two calls; saves the
 * second launch and balances both calls' units over the SMs together. Returns 0, or the codes
 * of r4d_gemm_moe_mxfp4a8_nt_b16_last_error (-10 also for a misaligned wq_cold). New. */
int b200_moe_gemm_hot_cold(const void* qx, const float* x_scale, const void* wq_hot, const void* wq_cold,
                           void* c, const int* sorted_hot, const int* eids_hot, const int* npad_hot,
                           int em_hot, const int* sorted_cold, const int* eids_cold, const int* npad_cold,
                           int em_cold, const float* topk_weights, int mtk, int top_k, int K, int N,
                           cudaStream_t stream);

/* Dynamic shared memory one launch uses at reduction depth K, or -1 if K is not supported.
 * New (no counterpart in the reference). */
int b200_moe_gemm_smem_bytes(int K);

/* Device error word of the grouped GEMM (1 = a bounded pipeline wait ran out); reset != 0
 * clears it. Synchronous. New. */
int b200_moe_gemm_error(int reset);

#ifdef __cplusplus
}
#endif

#endif /* B200_MOE_GEMM_H */

/* libb200lmhead.so -- the tail of the MoE block for B200 (sm_100a): the shared expert's gate,
 * y = sigmoid(gate) * out, and the routed experts' sum over top_k (moe_sum). Same conventions as b200_lmhead.h: plain pointers and sizes, an int status
 * (0 = ok, negative = argument error, positive = cudaError_t), caller-owned outputs, no
 * allocation. dtype 0 = bf16, 1 = f16, 2 = f32; every tensor of one call shares it.
 */
#ifndef B200_MOE_TAIL_H
#define B200_MOE_TAIL_H

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces the Triton _sigmoid_gate_mul_kernel behind sigmoid_gate_mul
 * (kernels/fused_gate_mul.py:19-38, 56-73). gate [rows, 1] contiguous; out [rows, cols] with
 * unit column stride and row stride stride_out; y [rows, cols] contiguous (a fresh buffer: out
 * may be an all-reduce output, fused_gate_mul.py:59-62). Bit-identical to
 * `F.sigmoid(gate) * out`. -1: negative sizes or stride_out < cols; -2: bad dtype. */
int b200_sigmoid_gate_mul(void* y, const void* out, const void* gate, int rows, int cols,
                          long long stride_out, int dtype, cudaStream_t stream);

/* Replaces the Triton _gemv_sigmoid_gate_mul_kernel behind gemv_sigmoid_gate_mul
 * (fused_gate_mul.py:91-121, 150-166): y = sigmoid(x @ w.T) * out with the [1, K]
 * shared_expert_gate weight folded in. x [rows, K] (row stride stride_x), w [1, K]
 * contiguous, out [rows, N] (row stride stride_out), y [rows, N] contiguous. The dot is
 * accumulated in fp32 and rounded to dtype before the sigmoid, as F.linear's output is; its
 * summation order is this kernel's (the gate scalar may differ from a library GEMM's in the
 * last bit, fused_gate_mul.py:84-88). One CTA per row: for decode-sized rows (the caller's
 * max_rows, fused_gate_mul.py:124-147). -1: rows outside [1, 65535], K or N < 1, or a row
 * stride below its row length; -2: bad dtype. */
int b200_gemv_sigmoid_gate_mul(void* y, const void* out, const void* x, const void* w, int rows,
                               int K, int N, long long stride_x, long long stride_out, int dtype,
                               cudaStream_t stream);

/* Replaces vLLM's ops.moe_sum(input, output) as the MoE block calls it
 * (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff L638, L696):
 * out[t, :] = sum_k in[t, k, :]. in [tokens, topk, H] contiguous; out [tokens, H] with row
 * stride stride_out. top_k in {2, 3, 4}: the running sum is rounded to dtype after every add
 * (vLLM's kernel keeps it in the storage type); any other top_k: torch.sum's CUDA order, four
 * fp32 accumulators over k = i mod 4 combined as ((a0 + a1) + a2) + a3, one rounding.
 * -1: tokens or H < 0, topk outside [1, 32], stride_out < H; -2: bad dtype. */
int b200_moe_sum(const void* in, void* out, int tokens, int topk, int H, long long stride_out,
                 int dtype, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_MOE_TAIL_H */

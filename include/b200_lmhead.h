/* libb200lmhead.so -- fused SiLU*mul FP8 quant, per-token group FP8 quant, and the FP8 / W4
 * lm_head GEMVs of the decode hot path, for B200 (sm_100a).
 *
 * Plain pointers and sizes, no torch types; every entry returns an int status (0 = ok,
 * negative = argument error, positive = cudaError_t) except r4d_gemm_w4a16_nt_m64, whose
 * reference ABI returns void. Nothing allocates; outputs and scratch are caller-owned.
 *
 * Packed weight layouts (B200 formats; their codes, scales and zeros are the reference's):
 *   FP8 wq  e4m3 [N/16 strips][K/128][16 rows][128 B]; 16-byte chunk c of strip row r is
 *           stored at chunk c ^ (r & 7). ws fp32 [N/128, K/128] row-major (unchanged).
 *   W4  wq  u32 [N_pad/16][K/128][2][8 g][4 t][4 words]; word w of lane (g, t) holds the
 *           offset-binary codes of k = 128*kb + 32*w + 8*t + j in nibble (j & 1)*4 + (j >> 1)
 *           of row 16*strip + 8*half + g.
 *       wsz int32 [N_pad/16, K/128, 16]: f16 scale | f16(-(1024 + zero)) << 16 (unchanged).
 */
#ifndef B200_LMHEAD_H
#define B200_LMHEAD_H

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Fused silu_and_mul + FP8 quant (replaces the Triton _silu_mul_quant_kernel behind
 * silu_mul_quant, kernels/fused_silu_mul_quant.py:26-101). x = [rows, 2*d] (gate | up) with
 * row stride stride_x elements, dtype 0 = bf16, 1 = f16. q e4m3 [rows, d]; group 0: scale fp32
 * [rows] = max(amax/448, 1/(448*512)) with q = e4m3(clamp(a / scale)); group 128: scale
 * [rows, d/128] = max(amax_g, 1e-10) * (1/448). act (nullable) [rows, d] in x's dtype.
 * Returns -1 for d > 8192 or negative sizes, -2 bad dtype, -3 unaligned group-128 call. */
int b200_silu_mul_quant(const void* x, int rows, int d, long long stride_x, int dtype, void* q,
                        float* scale, void* act, int group, cudaStream_t stream);

/* per_token_group_quant_fp8(x, group) (vLLM; called at kernels/fp8_target_lmhead.py:73):
 * s = max(amax, 1e-10) * (1/448), q = e4m3(clamp(x / s)); q [M, K], s [M, K/group]. */
int b200_per_token_group_quant_fp8(const void* x, int M, int K, long long stride_x, int dtype,
                                   int group, void* q, float* s, cudaStream_t stream);

/* scaled_fp8_quant(x, use_per_token_if_dynamic=True) (vLLM), the MoE hidden-state quant behind
 * fp8_quant_shared (patches/model_executor/kernels/linear/mxfp4/r4dhip.py.diff L19-34):
 * amax = min(max |x_row|, *scale_ub if given), scale = max(amax/448, 1/(448*512)),
 * q = e4m3(clamp(x / scale)). x [rows, K] with row stride stride_x; q [rows, K] contiguous;
 * scale fp32 [rows]. -1 negative sizes or stride_x < K; -2 bad dtype. */
int b200_per_token_quant_fp8(const void* x, int rows, int K, long long stride_x, int dtype,
                             const float* scale_ub, void* q, float* scale, cudaStream_t stream);

/* Bytes of the caller-owned scratch the fused lm_head entries use (activation tiles and rows,
 * per-CTA row statistics, partial accumulators). It needs no initialisation; calls that share
 * it must not overlap on the GPU. */
long long b200_lmhead_workspace_bytes(void);

/* Device error word (1 = a bounded pipeline wait timed out, 2 = a peer's statistics did not
 * arrive at the combine); reset != 0 clears it. Synchronous. While it is set, every head call's
 * row statistics come out poisoned (max and logsumexp NaN, argmax -1). */
int b200_lmhead_error(int reset);

/* Fused FP8 target lm_head (replaces gemm_fp8_block = per_token_group_quant_fp8 +
 * fp8hip_block_scaled_mm, kernels/fp8_target_lmhead.py:70-74, and adds the row statistics).
 * x bf16 [M, K]; wq / ws packed as above over N rows (N % 128 == 0, K % 128 == 0); y bf16
 * [M, ldy] (nullable); row_max fp32 [M], row_arg int64 [M] = first argmax + vocab_offset,
 * row_lse fp32 [M] (each nullable; any of them needs the workspace); qx_out e4m3 [M, K] and
 * xs_out fp32 [M, K/128] (nullable) receive the quantized activation.
 * Returns -1 M < 0, -2 N % 128, -3 K % 128, -8 shape exceeds shared memory, -9 workspace
 * missing / too small, -10 misaligned pointer. */
int b200_fp8_lmhead(const void* x, int M, int K, const void* wq, const float* ws, int N,
                    long long vocab_offset, void* y, long long ldy, float* row_max, long long* row_arg,
                    float* row_lse, void* qx_out, float* xs_out, void* workspace,
                    long long workspace_bytes, cudaStream_t stream);

/* b200_fp8_lmhead on this rank's vocabulary shard (vocab_offset = its first row) with the
 * peer-memory combine of b200_p2p_combine_row_stats fused into its last kernel: row_max /
 * row_arg / row_lse receive the GLOBAL (max, first argmax, logsumexp) over every rank's shard
 * (the reference's all-gather + argmax over ranks, patches/models/qwen4_exp/amd/mtp.py.diff
 * L194-227, in one launch set). peers / rank / world / counters / M_cap as for
 * b200_p2p_combine_row_stats (M <= M_cap; the same buffer and counters may serve both).
 * Extra code: -14 bad combine arguments. New (no single counterpart in the reference). */
int b200_fp8_lmhead_combined(const void* x, int M, int K, const void* wq, const float* ws, int N,
                             long long vocab_offset, void* y, long long ldy, float* row_max, long long* row_arg,
                             float* row_lse, void* qx_out, float* xs_out, void* workspace,
                             long long workspace_bytes, void* const* peers, int rank, int world,
                             unsigned long long* counters, int M_cap, cudaStream_t stream);

/* b200_fp8_lmhead without the workspace argument: the scratch is a device array inside the
 * library (about 23.4 MB per device), for callers that cannot allocate device memory. No
 * counterpart in the reference. Extra codes: -9 K > 16384, -13 device index >= 64. The first
 * call per device looks the array up; one array serves all streams of a device, so calls must
 * not overlap on the GPU. */
int b200_fp8_lmhead_static_scratch(const void* x, int M, int K, const void* wq, const float* ws,
                                   int N, long long vocab_offset, void* y, long long ldy,
                                   float* row_max, long long* row_arg, float* row_lse, void* qx_out,
                                   float* xs_out, cudaStream_t stream);

/* Vocabulary-sharded combine (new; the reference gathers full logits instead): pack this
 * rank's (max, argmax, logsumexp) as [M][3] float64, all-gather them (NCCL), then combine the
 * `world` blocks (rank-major, shards in vocabulary order) into the global max, first argmax
 * and logsumexp. Returns 0, -1 bad sizes, else the launch's cudaError_t. */
int b200_pack_row_stats(const float* row_max, const long long* row_arg, const float* row_lse, int M,
                        double* out, cudaStream_t stream);
int b200_combine_row_stats(const double* gathered, int world, int M, float* row_max, long long* row_arg,
                           float* row_lse, cudaStream_t stream);

/* The same combine as ONE kernel over NVLink peer memory (no NCCL call): each rank stores its
 * rows, as 8-byte words carrying 32 data bits and the call's 32-bit tag, into every rank's
 * peer-addressable buffer (b200_p2p_combine_bytes each; e.g. torch symmetric memory), reads
 * every rank's rows from its own buffer until their tags are this call's (bounded, 1 s; timeout
 * sets error word 2) and combines. `peers` is a device array of the world buffer pointers as
 * this GPU addresses them (world <= 64); `counters` a device uint64 array [M_cap] of per-token
 * call counters starting at 0; buffers zeroed before the first call; all ranks make the same
 * calls with the same M (a call with M == 0 does nothing). Returns 0, -1 bad sizes, else the
 * launch's cudaError_t. */
long long b200_p2p_combine_bytes(int world, int M_cap);
int b200_p2p_combine_row_stats(const float* row_max, const long long* row_arg, const float* row_lse, int M,
                               int M_cap, void* const* peers, int rank, int world,
                               unsigned long long* counters, float* out_max, long long* out_arg,
                               float* out_lse, cudaStream_t stream);

/* The closed fp8hip GEMM's ABI (tests/k3/test_fp8sk.py:13-34): pre-quantized e4m3 qx [M, K]
 * and fp32 xs [M, K/128], packed w / ws, bf16 y [M, N]. */
int fp8hip_gemm_w8a8_launch(void* qx, void* w, void* xs, void* ws, void* y, int M, int N, int K,
                            void* stream);

/* hcq_gemm_fp8blk_nt_m16 (kernels/experimental/fp8skinny/hcq_fp8skinny.hip:168-199): the same
 * operands for M <= 16 with the reference's precondition codes on its launch knobs:
 * -1 M outside 1..16, -2 N % 128, -3 K % 128, -4 (K/128) % SK, -5 WV*SK*32 > 1024,
 * -6 NPW not in {1,2,4}, -7 (WV*NPW*SK*256 + 16*K/128)*4 > 64 KB. */
int hcq_gemm_fp8blk_nt_m16(void* a, void* as, void* w, void* ws, void* c, int M, int K, int N,
                           int WV, int SK, int NPW, void* stream);
int hcq_gemm_fp8blk_nt_m16_max_m(void);

/* Read-only bandwidth control (hcq_stream_probe, hcq_fp8skinny.hip:206-224): streams `bytes`
 * (multiple of 16) from w over `wgs` CTAs; -1 bytes % 16, -2 wgs < 1. */
int hcq_stream_probe(void* w, long long bytes, int wgs, void* out, void* stream);

/* Fused W4 draft lm_head (the math of r4d_gemm_w4a16_nt_m64 behind gemm_w4a16,
 * kernels/draft_w4_lmhead.py:351-403, plus the row statistics the MTP head reduces,
 * patches/models/qwen4_exp/amd/mtp.py.diff L194-227). x [M, K] (x_dtype 0 = bf16, rounded to
 * f16 in the kernel; 1 = f16); wq / wsz packed as above over N_pad rows; rows >= n_valid are
 * padding (written to y, excluded from the statistics). Same outputs and codes as
 * b200_fp8_lmhead plus -11 bad dtype. */
int b200_w4_lmhead(const void* x, int x_dtype, int M, int K, const void* wq, const void* wsz,
                   int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                   float* row_max, long long* row_arg, float* row_lse, void* workspace,
                   long long workspace_bytes, cudaStream_t stream);

/* b200_w4_lmhead for the symmetric int4 format with bf16 group scales (the draft head's
 * configuration in this project's benchmark; the reference itself packs f16 scale + zero):
 * `wscale` bf16 [N_pad/16, K/128, 16], a code q in 0..15 means (q - 8) * scale. Same codes. */
int b200_w4_lmhead_sym(const void* x, int x_dtype, int M, int K, const void* wq, const void* wscale,
                       int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                       float* row_max, long long* row_arg, float* row_lse, void* workspace,
                       long long workspace_bytes, cudaStream_t stream);

/* The W4 draft head on this rank's vocabulary shard with the combine fused in, as
 * b200_fp8_lmhead_combined: sym 0 = b200_w4_lmhead's format, 1 = b200_w4_lmhead_sym's. The
 * row outputs are the GLOBAL statistics: the sharded form of MTP.get_top_tokens /
 * _w4_local_logits (patches/models/qwen4_exp/amd/mtp.py.diff L141-172, L194-227). Same codes
 * as b200_w4_lmhead plus -14. */
int b200_w4_lmhead_combined(int sym, const void* x, int x_dtype, int M, int K, const void* wq, const void* wsz,
                            int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                            float* row_max, long long* row_arg, float* row_lse, void* workspace,
                            long long workspace_bytes, void* const* peers, int rank, int world,
                            unsigned long long* counters, int M_cap, cudaStream_t stream);

/* r4d_gemm_w4a16_nt_m64 (ABI bound at kernels/draft_w4_lmhead.py:118-127): f16 a [M, K],
 * M <= 64, packed wq / wsz, bf16 c [M, N] with N = N_pad. WV/SK/MB/NPW/NT are the gfx1201
 * launch knobs, accepted and ignored. Returns void like the reference; the status of the
 * last call is r4d_gemm_w4a16_nt_m64_last_error(). */
void r4d_gemm_w4a16_nt_m64(long a, long wq, long wsz, long c, int M, int K, int N, int WV, int SK,
                           int MB, int NPW, int NT, long stream);
int r4d_gemm_w4a16_nt_m64_last_error(void);
int r4d_gemm_w4a16_nt_m64_max_m(void);  /* 64  (R4D_GEMM_W4_MAX_M) */
int r4d_gemm_w4a16_nt_m64_group(void);  /* 128 (the quantization group along K) */

#ifdef __cplusplus
}
#endif

#endif /* B200_LMHEAD_H */

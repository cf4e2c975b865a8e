/* librlu.so -- device-side LRU expert-slot cache for B200 (sm_100a).
 *
 * Drop-in for the C ABI of davetha/r9700-lru-expert-cache kernels/lru/r4d_lru.hip:577-631:
 * same symbol names, argument order, meaning and return codes, with cudaStream_t in place of
 * hipStream_t. Bound from Python with ctypes exactly as the reference's MoE patch does
 * (patches/.../r4d_mxfp4_moe.py.lru.diff L179-206).
 *
 * Ownership: the caller owns every buffer. No call allocates, synchronises with the host or
 * branches on host state, so all three are CUDA-graph capturable; only buffer contents change
 * between replays. Calls on one stream run in order. Errors are returned, never thrown.
 */
#ifndef R4D_LRU_H
#define R4D_LRU_H

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* One cache update for one MoE layer (replaces r4d_lru_manage, r4d_lru.hip:579-589).
 *   topk_ids    int32 [mk]     routed expert ids; ids outside [0, E) are ignored
 *   table       int32 [E]      expert -> slot or -1        (mutated)
 *   map_cold    int32 [E]      expert -> expert if not resident, else -1   (mutated)
 *   slot_expert int32 [S]      slot -> expert or -1        (mutated)
 *   slot_stamp  int64 [S]      slot -> step last routed    (mutated)
 *   routed      uint8 [E]      scratch: 1 for experts routed this step (written)
 *   step        int64 [1]      incremented once per call
 *   miss        int32 [max_inserts, 2]  (expert, slot) pairs; expert written for the first
 *                               nins misses, slot for the first n_miss of them
 *   n_miss      int32 [1]      victims installed this call
 * More than max_distinct distinct experts: read-through (only step / n_miss / routed change).
 * Returns 0, or -1 when E <= 0, S <= 0, S > 1024, max_inserts outside [0, 1024] (or, a B200
 * limit, E > 65536), else the launch's cudaError_t. */
int r4d_lru_manage(const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts,
                   int* table, int* map_cold, int* slot_expert, long long* slot_stamp,
                   unsigned char* routed, long long* step, int* miss, int* n_miss,
                   cudaStream_t stream);

/* The same update followed by both moe_align_block_size(topk, bs, E, map,
 * ignore_invalid_experts=True) outputs computed from the rewritten table -- the resident side
 * bucketed by slot, the fallback side by expert id (replaces r4d_lru_fused,
 * r4d_lru.hip:596-610). Every element of the six outputs is written on every call:
 * sorted_* int32 [L] (sentinel mk), eids_* int32 [NB] (-1 unused), npad_* int32 [1].
 * L and NB must be what vLLM allocates: L = mk < E ? min(mk*bs, mk + E*(bs-1))
 * : mk + E*(bs-1); NB = ceil(L / bs). Tokens inside a bucket are in ascending index order.
 * Returns -1 when E <= 0, E > 1024, S <= 0, S > 1024, bs/L/NB <= 0, mk < 0 or max_inserts
 * outside [0, 1024]. */
int r4d_lru_fused(const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts,
                  int* table, int* map_cold, int* slot_expert, long long* slot_stamp,
                  unsigned char* routed, long long* step, int* miss, int* n_miss, int bs, int L,
                  int NB, int* sorted_hot, int* eids_hot, int* npad_hot, int* sorted_cold,
                  int* eids_cold, int* npad_cold, cudaStream_t stream);

/* For each of the first n_miss (expert e, slot s) pairs, copy bytes [e*b_i, (e+1)*b_i) of
 * source i to bytes [s*b_i, (s+1)*b_i) of destination i, for the six buffers (replaces
 * r4d_lru_gather, r4d_lru.hip:612-629). Sources may be mapped pinned host memory (UVA).
 * grid = (chunks, lanes) CTAs of 256 threads. Returns -1 when a size is not a positive
 * multiple of 16 or chunks / lanes <= 0. */
int r4d_lru_gather(void* d0, const void* s0, long b0, void* d1, const void* s1, long b1, void* d2,
                   const void* s2, long b2, void* d3, const void* s3, long b3, void* d4,
                   const void* s4, long b4, void* d5, const void* s5, long b5, const int* miss,
                   const int* n_miss, int chunks, int lanes, cudaStream_t stream);

/* Device address of a pinned host buffer (cudaHostGetDevicePointer); the reference's test
 * makes the same call through hipHostGetDevicePointer (tests/lru/test_lru.py:42-50). */
int r4d_lru_host_device_pointer(void* host, void** dev);

#ifdef __cplusplus
}
#endif

#endif /* R4D_LRU_H */

// moe_sum: out[t, :] = sum_k in[t, k, :] over the top_k routed-expert rows of each token, the
// last step of the MoE block after the grouped down-projection
// (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff L638, L696:
// `ops.moe_sum(ic3.view(M, top_k, H), output)`), for sm_100a.
//
// Rounding follows vLLM's op: for top_k in {2, 3, 4} its kernel keeps the running sum in the
// storage dtype (each `x += in[k]` is an fp32 add rounded back to the dtype; ROUND_EACH). For
// any other top_k it is torch.sum over the top_k axis, whose CUDA reduction (ATen
// native/cuda/Reduce.cuh, thread_reduce_impl with vt0 = 4) gives each output thread four fp32
// accumulators: a_i sums the rows k = i, i + 4, i + 8, ... in order, and the result is
// ((a0 + a1) + a2) + a3, rounded once. For this layout (the top_k axis is not the fastest
// moving one) and top_k <= 32 no thread splits the top_k axis, so that order is the whole sum.
//
// B200 mapping: HBM-bound (top_k * 2 bytes read + 2 written per output element). One thread
// per 16-byte chunk of a token's output row: it issues its top_k 16-byte loads at once (the
// rows of one token are H * 2 bytes apart, so every load of a warp is a coalesced 512-byte
// segment), sums in registers and writes one 16-byte store.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace {

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }

constexpr int MS_THREADS = 256;
constexpr int MS_MAX_TOPK = 32;

// One work item = E consecutive elements of one token's output row (E = 16 / sizeof(T) when
// VEC, else 1). TOPK_C > 0: top_k known at compile time (fully unrolled loads).
template <typename T, bool VEC, bool ROUND_EACH, int TOPK_C>
__global__ void __launch_bounds__(MS_THREADS)
    moe_sum_kernel(const T* __restrict__ in, T* __restrict__ out, int tokens, int topk_rt, int H,
                   long long stride_out) {
  constexpr int E = VEC ? 16 / (int)sizeof(T) : 1;
  const int topk = TOPK_C > 0 ? TOPK_C : topk_rt;
  const unsigned per_row = (unsigned)(H / E);
  const unsigned long long total = (unsigned long long)tokens * per_row;
  const unsigned long long i = (unsigned long long)blockIdx.x * MS_THREADS + threadIdx.x;
  if (i >= total) return;
  const unsigned long long t = i / per_row;
  const unsigned c = (unsigned)(i - t * per_row);
  const T* src = in + (t * topk) * (unsigned long long)H + (unsigned long long)c * E;
  // ROUND_EACH: one running sum (acc[0]); otherwise four interleaved accumulators
  float acc[4][E];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[a][e] = 0.f;
  // row k goes to accumulator k & 3; every call below has a compile-time accumulator index
  auto add = [&](int a, const T* p) {
    if (ROUND_EACH) a = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      acc[a][e] += to_f(p[e]);
      if (ROUND_EACH) acc[a][e] = to_f(from_f<T>(acc[a][e]));
    }
  };
  if constexpr (VEC && TOPK_C > 0) {
    uint4 v[TOPK_C];
#pragma unroll
    for (int k = 0; k < TOPK_C; ++k) v[k] = __ldg(reinterpret_cast<const uint4*>(src + (long long)k * H));
#pragma unroll
    for (int k = 0; k < TOPK_C; ++k) add(k & 3, reinterpret_cast<const T*>(&v[k]));
  } else {
    for (int k0 = 0; k0 < topk; k0 += 4) {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int k = k0 + a;
        if (k < topk) {
          if constexpr (VEC) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + (long long)k * H));
            add(a, reinterpret_cast<const T*>(&v));
          } else {
            add(a, src + (long long)k * H);
          }
        }
      }
    }
  }
  union {
    uint4 raw;
    T v[E];
  } o;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float r = ROUND_EACH ? acc[0][e] : ((acc[0][e] + acc[1][e]) + acc[2][e]) + acc[3][e];
    o.v[e] = from_f<T>(r);
  }
  if constexpr (VEC) {
    *reinterpret_cast<uint4*>(out + t * (unsigned long long)stride_out + (unsigned long long)c * E) = o.raw;
  } else {
    out[t * (unsigned long long)stride_out + c] = o.v[0];
  }
}

template <typename T, bool VEC>
void launch_vec(const T* in, T* out, int tokens, int topk, int H, long long so, unsigned blocks,
                cudaStream_t st) {
  switch (topk) {
    case 2: moe_sum_kernel<T, VEC, true, 2><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    case 3: moe_sum_kernel<T, VEC, true, 3><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    case 4: moe_sum_kernel<T, VEC, true, 4><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    case 6: moe_sum_kernel<T, VEC, false, 6><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    case 8: moe_sum_kernel<T, VEC, false, 8><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    case 10: moe_sum_kernel<T, VEC, false, 10><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
    default: moe_sum_kernel<T, VEC, false, 0><<<blocks, MS_THREADS, 0, st>>>(in, out, tokens, topk, H, so); break;
  }
}

template <typename T>
int launch(const void* in, void* out, int tokens, int topk, int H, long long stride_out,
           cudaStream_t st) {
  constexpr int E = 16 / (int)sizeof(T);
  const T* ip = static_cast<const T*>(in);
  T* op = static_cast<T*>(out);
  const bool vec = H % E == 0 && stride_out % E == 0 &&
                   (reinterpret_cast<uintptr_t>(in) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  const long long items = (long long)tokens * (vec ? H / E : H);
  const long long blocks = (items + MS_THREADS - 1) / MS_THREADS;
  if (blocks > 0x7fffffffLL) return -1;
  if (vec) {
    launch_vec<T, true>(ip, op, tokens, topk, H, stride_out, (unsigned)blocks, st);
  } else if (topk >= 2 && topk <= 4) {
    moe_sum_kernel<T, false, true, 0><<<(unsigned)blocks, MS_THREADS, 0, st>>>(ip, op, tokens, topk, H, stride_out);
  } else {
    moe_sum_kernel<T, false, false, 0><<<(unsigned)blocks, MS_THREADS, 0, st>>>(ip, op, tokens, topk, H, stride_out);
  }
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// out[t, :] = sum over k of in[t, k, :]: in [tokens, topk, H] contiguous, out [tokens, H] with
// unit column stride and row stride stride_out; dtype 0 = bf16, 1 = f16, 2 = f32. Mirrors
// vLLM's ops.moe_sum(input, output) as called at r4d_mxfp4_moe.py.lru.diff L638 / L696.
// Returns 0, -1 for bad sizes (tokens or H < 0, topk outside [1, 32], stride_out < H), -2
// for a bad dtype, else a CUDA error code.
int b200_moe_sum(const void* in, void* out, int tokens, int topk, int H, long long stride_out,
                 int dtype, cudaStream_t stream) {
  if (tokens < 0 || H < 0 || topk < 1 || topk > MS_MAX_TOPK || (tokens > 1 && stride_out < H)) return -1;
  if (dtype < 0 || dtype > 2) return -2;
  if (tokens == 0 || H == 0) return 0;
  if (dtype == 0) return launch<__nv_bfloat16>(in, out, tokens, topk, H, stride_out, stream);
  if (dtype == 1) return launch<__half>(in, out, tokens, topk, H, stride_out, stream);
  return launch<float>(in, out, tokens, topk, H, stride_out, stream);
}

}  // extern "C"

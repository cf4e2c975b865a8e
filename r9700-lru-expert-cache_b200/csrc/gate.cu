// Shared-expert gate of the MoE block, y = sigmoid(gate) * out, for sm_100a.
//
// sigmoid_gate_mul: drop-in for _sigmoid_gate_mul_kernel (kernels/fused_gate_mul.py:19-38).
//   Rounds as aten's `F.sigmoid(g) * out` does, so the result is bit-identical to that stock
//   path: s = T(1 / (1 + exp(-float(g)))) (sigmoid in fp32, stored in the gate's dtype), then
//   y = T(float(s) * float(out)) (the multiply's fp32 opmath, rounded on store). Built without
//   fast math, so expf and `/` are the accurate / IEEE forms aten's kernels use.
// gemv_sigmoid_gate_mul: drop-in for _gemv_sigmoid_gate_mul_kernel (fused_gate_mul.py:91-121).
//   The [1, K] shared_expert_gate GEMV folded in: g = T(sum_k x[k] * w[k]) (fp32 accumulation,
//   rounded as F.linear's output is), then the same sigmoid and multiply. The fp32 summation
//   order is this kernel's, so g may differ from a library GEMM's in its last bit
//   (fused_gate_mul.py:84-88); everything after the dot rounds exactly as the stock path.
//
// B200 mapping. Both are HBM-bound byte streams (2 bytes read + 2 written per element of
// `out`); no tensor cores. Mode 1 is a flat grid over 16-byte chunks of `out`: rows of any
// count share CTAs, each thread keeps U chunks in flight (U = 4 once the grid fills the 148
// SMs, 1 below that so small decode batches spread over as many SMs as they can). Mode 2 runs
// one CTA per row (decode-sized row counts only): the row's first `out` chunks are loaded
// before the dot so that the HBM round trip for `out` overlaps the x.w reduction.
#include <cuda_runtime.h>
#include <limits.h>
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

// aten's sigmoid for a value stored as T: fp32 opmath, rounded to T, widened back (exact).
template <typename T>
__device__ __forceinline__ float gate_scale(float g) {
  return to_f(from_f<T>(1.0f / (1.0f + expf(-g))));
}

// 16-byte chunk of T: E elements.
template <typename T>
struct Chunk {
  static constexpr int E = 16 / sizeof(T);
  union {
    uint4 raw;
    T v[E];
  };
};

template <typename T>
__device__ __forceinline__ uint4 scale_chunk(uint4 raw, float s) {
  Chunk<T> c;
  c.raw = raw;
#pragma unroll
  for (int i = 0; i < Chunk<T>::E; ++i) c.v[i] = from_f<T>(s * to_f(c.v[i]));
  return c.raw;
}

constexpr int GM_THREADS = 256;

// Mode 1. VEC: rows 16-byte aligned and cols % E == 0, one work item = one 16-byte chunk;
// otherwise one work item = one element. I is the index type (uint32 when the item count
// allows it, which keeps the row division short).
template <typename T, bool VEC, int U, typename I>
__global__ void __launch_bounds__(GM_THREADS)
    sigmoid_gate_mul_kernel(T* __restrict__ y, const T* __restrict__ out,
                            const T* __restrict__ gate, int rows, int cols, long long stride_out) {
  constexpr int E = VEC ? Chunk<T>::E : 1;
  const I per_row = (I)(cols / E);
  const I total = (I)rows * per_row;
  const I stride = (I)gridDim.x * GM_THREADS;
  for (I base = (I)blockIdx.x * GM_THREADS + threadIdx.x; base < total; base += stride * U) {
    uint4 v[U];
    T e[U];
    float g[U];
    I r[U], c[U];
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const I i = base + (I)k * stride;
      if (i < total) {
        r[k] = i / per_row;
        c[k] = i - r[k] * per_row;
        const T* src = out + (long long)r[k] * stride_out + (long long)c[k] * E;
        if constexpr (VEC) v[k] = __ldg(reinterpret_cast<const uint4*>(src));
        else e[k] = src[0];
        g[k] = to_f(gate[r[k]]);
      }
    }
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const I i = base + (I)k * stride;
      if (i < total) {
        const float s = gate_scale<T>(g[k]);
        T* dst = y + (long long)r[k] * cols + (long long)c[k] * E;
        if constexpr (VEC) *reinterpret_cast<uint4*>(dst) = scale_chunk<T>(v[k], s);
        else dst[0] = from_f<T>(s * to_f(e[k]));
      }
    }
  }
}

// Mode 2: one CTA per row. VEC: K % E == N % E == 0 and every row 16-byte aligned.
template <typename T, bool VEC>
__global__ void __launch_bounds__(512)
    gemv_sigmoid_gate_mul_kernel(T* __restrict__ y, const T* __restrict__ out,
                                 const T* __restrict__ x, const T* __restrict__ w, int K, int N,
                                 long long stride_x, long long stride_out) {
  constexpr int E = VEC ? Chunk<T>::E : 1;
  __shared__ float s_red[16];
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const int nt = blockDim.x;
  const T* xr = x + (long long)row * stride_x;
  const T* orow = out + (long long)row * stride_out;
  T* yr = y + (long long)row * N;
  const int kc = K / E, nc = N / E;

  // this thread's first chunk of `out`, in flight during the dot
  uint4 o0;
  T oe0 = from_f<T>(0.f);
  if (tid < nc) {
    if constexpr (VEC) o0 = __ldg(reinterpret_cast<const uint4*>(orow) + tid);
    else oe0 = orow[tid];
  }

  float acc = 0.f;
  for (int c = tid; c < kc; c += nt) {
    if constexpr (VEC) {
      Chunk<T> a, b;
      a.raw = __ldg(reinterpret_cast<const uint4*>(xr) + c);
      b.raw = __ldg(reinterpret_cast<const uint4*>(w) + c);
#pragma unroll
      for (int i = 0; i < E; ++i) acc = fmaf(to_f(a.v[i]), to_f(b.v[i]), acc);
    } else {
      acc = fmaf(to_f(xr[c]), to_f(w[c]), acc);
    }
  }
  acc = b200::warp_sum(acc);
  if ((tid & 31) == 0) s_red[tid >> 5] = acc;
  __syncthreads();
  float dot = 0.f;
  for (int i = 0; i < (nt >> 5); ++i) dot += s_red[i];        // same order in every thread

  // F.linear's output is stored in T before the sigmoid sees it
  const float s = gate_scale<T>(to_f(from_f<T>(dot)));
  if (tid < nc) {
    if constexpr (VEC) reinterpret_cast<uint4*>(yr)[tid] = scale_chunk<T>(o0, s);
    else yr[tid] = from_f<T>(s * to_f(oe0));
  }
  for (int c = tid + nt; c < nc; c += nt) {
    if constexpr (VEC) {
      reinterpret_cast<uint4*>(yr)[c] = scale_chunk<T>(__ldg(reinterpret_cast<const uint4*>(orow) + c), s);
    } else {
      yr[c] = from_f<T>(s * to_f(orow[c]));
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int num_sms() {
  static int sms[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 64 && sms[dev] == 0) cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
  return dev < 64 && sms[dev] > 0 ? sms[dev] : 148;
}

template <typename T, bool VEC, int U>
void launch_gm_u(T* y, const T* out, const T* gate, int rows, int cols, long long stride_out,
                 long long total, cudaStream_t st) {
  long long blocks = (total + (long long)GM_THREADS * U - 1) / ((long long)GM_THREADS * U);
  if (blocks > 65535) blocks = 65535;
  if (total + (long long)GM_THREADS * 65535 * U <= (long long)UINT_MAX)
    sigmoid_gate_mul_kernel<T, VEC, U, uint32_t><<<(unsigned)blocks, GM_THREADS, 0, st>>>(
        y, out, gate, rows, cols, stride_out);
  else
    sigmoid_gate_mul_kernel<T, VEC, U, unsigned long long><<<(unsigned)blocks, GM_THREADS, 0, st>>>(
        y, out, gate, rows, cols, stride_out);
}

template <typename T>
int launch_gm(void* y, const void* out, const void* gate, int rows, int cols, long long stride_out,
              cudaStream_t st) {
  constexpr int E = Chunk<T>::E;
  T* yp = static_cast<T*>(y);
  const T* op = static_cast<const T*>(out);
  const T* gp = static_cast<const T*>(gate);
  const bool vec = cols % E == 0 && stride_out % E == 0 && aligned16(out) && aligned16(y);
  if (vec) {
    const long long total = (long long)rows * (cols / E);
    // U = 4 only once the U = 4 grid still covers every SM
    if (total >= (long long)GM_THREADS * 4 * num_sms())
      launch_gm_u<T, true, 4>(yp, op, gp, rows, cols, stride_out, total, st);
    else
      launch_gm_u<T, true, 1>(yp, op, gp, rows, cols, stride_out, total, st);
  } else {
    launch_gm_u<T, false, 1>(yp, op, gp, rows, cols, stride_out, (long long)rows * cols, st);
  }
  return (int)cudaGetLastError();
}

template <typename T>
int launch_gemv(void* y, const void* out, const void* x, const void* w, int rows, int K, int N,
                long long stride_x, long long stride_out, cudaStream_t st) {
  constexpr int E = Chunk<T>::E;
  const bool vec = K % E == 0 && N % E == 0 && stride_x % E == 0 && stride_out % E == 0 &&
                   aligned16(x) && aligned16(w) && aligned16(out) && aligned16(y);
  const int items = vec ? (K > N ? K : N) / E : (K > N ? K : N);
  int nt = (items + 31) / 32 * 32;
  nt = nt < 64 ? 64 : (nt > 512 ? 512 : nt);
  if (vec)
    gemv_sigmoid_gate_mul_kernel<T, true><<<rows, nt, 0, st>>>(
        static_cast<T*>(y), static_cast<const T*>(out), static_cast<const T*>(x),
        static_cast<const T*>(w), K, N, stride_x, stride_out);
  else
    gemv_sigmoid_gate_mul_kernel<T, false><<<rows, nt, 0, st>>>(
        static_cast<T*>(y), static_cast<const T*>(out), static_cast<const T*>(x),
        static_cast<const T*>(w), K, N, stride_x, stride_out);
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// y[r, :] = sigmoid(gate[r]) * out[r, :] for a [rows, 1] gate (contiguous) and a [rows, cols]
// `out` with unit column stride and row stride `stride_out` elements; y is [rows, cols]
// contiguous. dtype 0 = bf16, 1 = f16, 2 = f32 (gate, out and y share it). Bit-identical to
// `F.sigmoid(gate) * out`. Mirrors sigmoid_gate_mul (kernels/fused_gate_mul.py:56-73).
// Returns 0, -1 for negative sizes or stride_out < cols, -2 for a bad dtype, else a CUDA
// error code.
int b200_sigmoid_gate_mul(void* y, const void* out, const void* gate, int rows, int cols,
                          long long stride_out, int dtype, cudaStream_t stream) {
  if (rows < 0 || cols < 0 || (rows > 1 && stride_out < cols)) return -1;
  if (dtype < 0 || dtype > 2) return -2;
  if (rows == 0 || cols == 0) return 0;
  if (dtype == 0) return launch_gm<__nv_bfloat16>(y, out, gate, rows, cols, stride_out, stream);
  if (dtype == 1) return launch_gm<__half>(y, out, gate, rows, cols, stride_out, stream);
  return launch_gm<float>(y, out, gate, rows, cols, stride_out, stream);
}

// y[r, :] = sigmoid(T(x[r, :] . w)) * out[r, :]: the [1, K] gate GEMV folded into the gate
// multiply. x [rows, K] (row stride stride_x), w [1, K] contiguous, out [rows, N] (row stride
// stride_out), y [rows, N] contiguous; all of one dtype (0 = bf16, 1 = f16, 2 = f32). One CTA
// per row, for decode-sized row counts (the caller's max_rows bound, fused_gate_mul.py:124-147).
// Mirrors gemv_sigmoid_gate_mul (fused_gate_mul.py:150-166). Returns 0, -1 for bad sizes
// (rows outside [1, 65535], K or N < 1, a row stride below its row length), -2 for a bad
// dtype, else a CUDA error code.
int b200_gemv_sigmoid_gate_mul(void* y, const void* out, const void* x, const void* w, int rows,
                               int K, int N, long long stride_x, long long stride_out, int dtype,
                               cudaStream_t stream) {
  if (rows < 1 || rows > 65535 || K < 1 || N < 1) return -1;
  if ((rows > 1 && (stride_x < K || stride_out < N))) return -1;
  if (dtype < 0 || dtype > 2) return -2;
  if (dtype == 0)
    return launch_gemv<__nv_bfloat16>(y, out, x, w, rows, K, N, stride_x, stride_out, stream);
  if (dtype == 1) return launch_gemv<__half>(y, out, x, w, rows, K, N, stride_x, stride_out, stream);
  return launch_gemv<float>(y, out, x, w, rows, K, N, stride_x, stride_out, stream);
}

}  // extern "C"

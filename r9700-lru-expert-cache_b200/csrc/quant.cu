// Fused SiLU*mul -> FP8-e4m3 activation quant and per-token group-128 FP8 quant (sm_100a).
//
// silu_mul_quant: drop-in for _silu_mul_quant_kernel (kernels/fused_silu_mul_quant.py:26-57).
//   Per row of x = [gate | up] (each d wide): s = bf16(g / (1 + exp(-g))), a = bf16(s * u)
//   (the storage-dtype rounding of vLLM's act_and_mul_kernel), amax = max |a|,
//   scale = max(amax / 448, 1 / (448 * 512)), q = e4m3(clamp(a / scale, +-448)) -- a true
//   IEEE division, not a reciprocal multiply (fused_silu_mul_quant.py:9-14). Built without
//   fast math so `/` and expf are the IEEE / accurate forms. The clamp is the reference's
//   maximum(-448, minimum(v, 448)) (fused_silu_mul_quant.py:56), whose fmin-first order sends
//   a NaN to +448; the row amax ignores NaNs as fmax does.
//   The group variant (group = 128) replaces the per-row scale with one per 128 columns,
//   following per_token_group_quant_fp8: scale = max(amax, 1e-10) * fp32(1/448).
//
// B200 mapping: one warp per row (4 rows per 128-thread CTA), 16-byte loads of 8 elements
// when the row is 16-byte aligned, warp-shuffle amax. Rows up to 1024 wide keep the
// activation in registers between the amax and the quantization (one pass); wider or
// unaligned rows recompute it in a second pass, bit-identical by construction, so any d up
// to the reference's 8192 bound runs.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace {

constexpr float kFp8Max = 448.0f;
constexpr float kMinScale = 1.0f / (448.0f * 512.0f);   // vllm min_scaling_factor<fp8>
constexpr float kGroupEps = 1e-10f;
constexpr int ROWS_PER_CTA = 4;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

// a = T(T(silu(g)) * u), returned widened to float (exact).
template <typename T>
__device__ __forceinline__ float silu_mul_elem(T g, T u, T* a_out) {
  const float gf = to_f(g);
  const float s = to_f(from_f<T>(gf / (1.0f + expf(-gf))));
  const T a = from_f<T>(s * to_f(u));
  *a_out = a;
  return to_f(a);
}

// Load 8 consecutive elements of T at p (16-byte aligned when VEC).
template <typename T, bool VEC>
__device__ __forceinline__ void load8(const T* p, int n_valid, T (&v)[8]) {
  if (VEC) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    const T* rv = reinterpret_cast<const T*>(&r);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = rv[i];
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = (i < n_valid) ? p[i] : from_f<T>(0.f);
  }
}

// GROUP == 0: per-row scale. GROUP == 128: per-128-column scales (requires VEC, d % 128 == 0).
template <typename T, bool VEC, int GROUP>
__global__ void __launch_bounds__(32 * ROWS_PER_CTA)
    silu_mul_quant_kernel(const T* __restrict__ x, long long stride_x, int rows, int d,
                          uint8_t* __restrict__ q, float* __restrict__ scale, T* __restrict__ act) {
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const T* xg = x + (long long)row * stride_x;
  const T* xu = xg + d;
  const int nchunk = (d + 7) / 8;

  if constexpr (GROUP == 0) {
    // pass 1: amax of the stored activation (and the optional bf16 activation itself)
    float amax = 0.f;
    for (int c = lane; c < nchunk; c += 32) {
      const int nv = min(8, d - 8 * c);
      T g[8], u[8], a[8];
      load8<T, VEC>(xg + 8 * c, nv, g);
      load8<T, VEC>(xu + 8 * c, nv, u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float af = silu_mul_elem<T>(g[i], u[i], &a[i]);
        if (i < nv) amax = fmaxf(amax, fabsf(af));
      }
      if (act != nullptr) {
        T* ap = act + (long long)row * d + 8 * c;
        if (VEC) {
          *reinterpret_cast<uint4*>(ap) = *reinterpret_cast<const uint4*>(a);
        } else {
          for (int i = 0; i < nv; ++i) ap[i] = a[i];
        }
      }
    }
    amax = b200::warp_max(amax);
    const float sc = fmaxf(amax / kFp8Max, kMinScale);
    if (lane == 0) scale[row] = sc;
    // pass 2: recompute (bit-identical) and quantize with a true division
    for (int c = lane; c < nchunk; c += 32) {
      const int nv = min(8, d - 8 * c);
      T g[8], u[8], a[8];
      load8<T, VEC>(xg + 8 * c, nv, g);
      load8<T, VEC>(xu + 8 * c, nv, u);
      uint8_t b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float af = silu_mul_elem<T>(g[i], u[i], &a[i]);
        b[i] = b200::f32_to_e4m3(fmaxf(fminf(af / sc, kFp8Max), -kFp8Max));
      }
      uint8_t* qp = q + (long long)row * d + 8 * c;
      if (VEC) {
        *reinterpret_cast<uint2*>(qp) = *reinterpret_cast<const uint2*>(b);
      } else {
        for (int i = 0; i < nv; ++i) qp[i] = b[i];
      }
    }
  } else {
    // group-128: 16 chunks per group; chunk c = lane + 32*j, lanes 0-15 / 16-31 own one group
    const int ngroups = d / (GROUP > 0 ? GROUP : 1);
    for (int base = 0; base < nchunk; base += 32) {
      // all 32 lanes iterate together (the group shuffle needs them); a lane past the row
      // end works on the first chunk of this pass and stores nothing. nchunk % 16 == 0, so
      // a half-warp is either wholly live or wholly idle.
      const bool live = base + lane < nchunk;
      const int c = live ? base + lane : base;
      T g[8], u[8], a[8];
      load8<T, true>(xg + 8 * c, 8, g);
      load8<T, true>(xu + 8 * c, 8, u);
      float af[8];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        af[i] = silu_mul_elem<T>(g[i], u[i], &a[i]);
        amax = fmaxf(amax, fabsf(af[i]));
      }
      if (act != nullptr && live)
        *reinterpret_cast<uint4*>(act + (long long)row * d + 8 * c) = *reinterpret_cast<const uint4*>(a);
      // reduce over the 16 lanes of this group (d % 128 == 0: a group never straddles)
#pragma unroll
      for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      if (!live) continue;
      const float sc = fmaxf(amax, kGroupEps) * (1.0f / kFp8Max);
      const int grp = c / 16;
      if ((lane & 15) == 0) scale[(long long)row * ngroups + grp] = sc;
      uint8_t b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) b[i] = b200::f32_to_e4m3(fmaxf(fminf(af[i] / sc, kFp8Max), -kFp8Max));
      *reinterpret_cast<uint2*>(q + (long long)row * d + 8 * c) = *reinterpret_cast<const uint2*>(b);
    }
  }
}

// Per-row scale, rows of at most 32 * 8 * RC elements (16-byte aligned): one pass. Each lane
// keeps its RC chunks of the activation in registers between the amax and the quantization,
// so every element costs one expf and two divisions instead of twice that; the values are
// those of silu_mul_quant_kernel bit for bit (same expressions, same order).
template <typename T, int RC>
__global__ void __launch_bounds__(32 * ROWS_PER_CTA)
    silu_mul_quant_reg_kernel(const T* __restrict__ x, long long stride_x, int rows, int d,
                              uint8_t* __restrict__ q, float* __restrict__ scale, T* __restrict__ act) {
  const int row = blockIdx.x * ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const T* xg = x + (long long)row * stride_x;
  const T* xu = xg + d;
  const int nchunk = d / 8;
  float af[RC][8];
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < RC; ++j) {
    const int c = lane + 32 * j;
    if (c < nchunk) {
      T g[8], u[8], a[8];
      load8<T, true>(xg + 8 * c, 8, g);
      load8<T, true>(xu + 8 * c, 8, u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        af[j][i] = silu_mul_elem<T>(g[i], u[i], &a[i]);
        amax = fmaxf(amax, fabsf(af[j][i]));
      }
      if (act != nullptr)
        *reinterpret_cast<uint4*>(act + (long long)row * d + 8 * c) = *reinterpret_cast<const uint4*>(a);
    }
  }
  amax = b200::warp_max(amax);
  const float sc = fmaxf(amax / kFp8Max, kMinScale);
  if (lane == 0) scale[row] = sc;
#pragma unroll
  for (int j = 0; j < RC; ++j) {
    const int c = lane + 32 * j;
    if (c < nchunk) {
      uint8_t b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) b[i] = b200::f32_to_e4m3(fmaxf(fminf(af[j][i] / sc, kFp8Max), -kFp8Max));
      *reinterpret_cast<uint2*>(q + (long long)row * d + 8 * c) = *reinterpret_cast<const uint2*>(b);
    }
  }
}

// Per-token dynamic FP8 quant of a [rows, K] activation (vLLM scaled_fp8_quant with
// use_per_token_if_dynamic=True): amax = max |x| over the row, clipped to *scale_ub when
// given, scale = max(amax / 448, 1 / (448 * 512)), q = e4m3(clamp(x / scale, +-448)) with a
// true division.
//
// WPR warps per row, 256-thread CTAs (256 / (32 * WPR) rows each). RC > 0: the row (16-byte
// aligned, K % 8 == 0, at most 256 * WPR * RC elements) stays in registers as raw 16-byte
// chunks between the amax and the quantization, so HBM is read once; chunk c of the row goes
// to thread c % (32 * WPR) of its row group. RC is kept <= 4 so the kernel runs at full
// occupancy and the warps of an SM overlap their loads with one another's arithmetic. RC == 0:
// two passes over the row (the second served by L1 / L2), for wide or unaligned rows. The
// row amax of several warps meets in shared memory.
constexpr int TQ_THREADS = 256;

template <typename T, int WPR, int RC, bool VEC>
__global__ void __launch_bounds__(TQ_THREADS)
    token_quant_kernel(const T* __restrict__ x, long long stride_x, int rows, int K,
                       const float* __restrict__ scale_ub, uint8_t* __restrict__ q,
                       float* __restrict__ scale) {
  constexpr int RPC = TQ_THREADS / (32 * WPR);              // rows per CTA
  constexpr int TPR = 32 * WPR;                              // threads per row
  __shared__ float s_amax[TQ_THREADS / 32];
  const int warp = threadIdx.x >> 5;
  const int rit = threadIdx.x % TPR;                         // thread index within the row
  const int row = blockIdx.x * RPC + threadIdx.x / TPR;
  const bool live = row < rows;                              // every thread reaches the barrier
  const T* xr = x + (long long)(live ? row : 0) * stride_x;
  uint8_t* qr = q + (long long)(live ? row : 0) * K;
  const int nchunk = (K + 7) / 8;
  float amax = 0.f;
  uint4 keep[RC > 0 ? RC : 1];
  if constexpr (RC > 0) {
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      const int c = rit + TPR * j;
      if (live && c < nchunk) keep[j] = __ldg(reinterpret_cast<const uint4*>(xr) + c);
    }
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      if (live && rit + TPR * j < nchunk) {
        const T* v = reinterpret_cast<const T*>(&keep[j]);
#pragma unroll
        for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(to_f(v[i])));
      }
    }
  } else if (live) {
    for (int c = rit; c < nchunk; c += TPR) {
      T v[8];
      load8<T, VEC>(xr + 8 * c, min(8, K - 8 * c), v);
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(to_f(v[i])));
    }
  }
  amax = b200::warp_max(amax);
  if constexpr (WPR > 1) {
    if ((threadIdx.x & 31) == 0) s_amax[warp] = amax;
    __syncthreads();
    const int w0 = (warp / WPR) * WPR;
#pragma unroll
    for (int w = 0; w < WPR; ++w) amax = fmaxf(amax, s_amax[w0 + w]);
  }
  if (!live) return;
  if (scale_ub != nullptr) amax = fminf(amax, *scale_ub);
  const float sc = fmaxf(amax / kFp8Max, kMinScale);
  if (rit == 0) scale[row] = sc;
  if constexpr (RC > 0) {
#pragma unroll
    for (int j = 0; j < RC; ++j) {
      const int c = rit + TPR * j;
      if (c < nchunk) {
        const T* v = reinterpret_cast<const T*>(&keep[j]);
        uint8_t b[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) b[i] = b200::f32_to_e4m3(fmaxf(fminf(to_f(v[i]) / sc, kFp8Max), -kFp8Max));
        *reinterpret_cast<uint2*>(qr + 8 * c) = *reinterpret_cast<const uint2*>(b);
      }
    }
  } else {
    for (int c = rit; c < nchunk; c += TPR) {
      const int nv = min(8, K - 8 * c);
      T v[8];
      load8<T, VEC>(xr + 8 * c, nv, v);
      uint8_t b[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) b[i] = b200::f32_to_e4m3(fmaxf(fminf(to_f(v[i]) / sc, kFp8Max), -kFp8Max));
      if (VEC) {
        *reinterpret_cast<uint2*>(qr + 8 * c) = *reinterpret_cast<const uint2*>(b);
      } else {
        for (int i = 0; i < nv; ++i) qr[8 * c + i] = b[i];
      }
    }
  }
}

template <typename T, int WPR>
void launch_tq_wpr(const T* xp, long long stride_x, int rows, int K, const float* ub, uint8_t* qp,
                   float* scale, int rc, cudaStream_t stream) {
  constexpr int RPC = TQ_THREADS / (32 * WPR);
  const dim3 grid((rows + RPC - 1) / RPC), block(TQ_THREADS);
  if (rc == 1)
    token_quant_kernel<T, WPR, 1, true><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
  else if (rc == 2)
    token_quant_kernel<T, WPR, 2, true><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
  else if (rc == 3)
    token_quant_kernel<T, WPR, 3, true><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
  else
    token_quant_kernel<T, WPR, 4, true><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
}

template <typename T>
int launch_token_quant(const void* x, long long stride_x, int rows, int K, const float* ub,
                       void* q, float* scale, cudaStream_t stream) {
  const bool vec = (K % 8 == 0) && (stride_x % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(q) & 7) == 0);
  const T* xp = static_cast<const T*>(x);
  uint8_t* qp = static_cast<uint8_t*>(q);
  const int nchunk = K / 8;
  if (vec && nchunk <= 32 * 8 * 4) {
    // the fewest warps per row that keep RC <= 4, then more while the grid has fewer CTAs
    // than SMs (decode-sized row counts spread over more of the chip)
    int wpr = 1;
    while (wpr < 8 && nchunk > 32 * wpr * 4) wpr *= 2;
    while (wpr < 8 && (long long)rows * wpr * 32 < (long long)TQ_THREADS * 148) wpr *= 2;
    const int rc = (nchunk + 32 * wpr - 1) / (32 * wpr);
    switch (wpr) {
      case 1: launch_tq_wpr<T, 1>(xp, stride_x, rows, K, ub, qp, scale, rc, stream); break;
      case 2: launch_tq_wpr<T, 2>(xp, stride_x, rows, K, ub, qp, scale, rc, stream); break;
      case 4: launch_tq_wpr<T, 4>(xp, stride_x, rows, K, ub, qp, scale, rc, stream); break;
      default: launch_tq_wpr<T, 8>(xp, stride_x, rows, K, ub, qp, scale, rc, stream); break;
    }
  } else {
    const dim3 grid(rows), block(TQ_THREADS);               // one row per CTA, two passes
    if (vec)
      token_quant_kernel<T, 8, 0, true><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
    else
      token_quant_kernel<T, 8, 0, false><<<grid, block, 0, stream>>>(xp, stride_x, rows, K, ub, qp, scale);
  }
  return (int)cudaGetLastError();
}

// Per-token group quant of a [M, K] activation: half a warp per 128-wide group.
template <typename T>
__global__ void __launch_bounds__(256)
    group_quant_kernel(const T* __restrict__ x, long long stride_x, int M, int K, int group,
                       uint8_t* __restrict__ q, float* __restrict__ s) {
  const int ng = K / group;
  const int cpg = group / 8;                      // chunks of 8 per group (16 for 128)
  const long long nchunks = (long long)M * K / 8;
  for (long long c = (long long)blockIdx.x * blockDim.x + threadIdx.x;; c += (long long)gridDim.x * blockDim.x) {
    // every lane of a warp iterates together so the group shuffle is well defined
    const long long cbase = c - (threadIdx.x & 31);
    if (cbase >= nchunks) break;
    const bool live = c < nchunks;
    const long long cc = live ? c : cbase;
    const int m = (int)(cc / (K / 8));
    const int kc = (int)(cc % (K / 8));
    T v[8];
    load8<T, true>(x + (long long)m * stride_x + 8 * kc, 8, v);
    float f[8];
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      f[i] = to_f(v[i]);
      amax = fmaxf(amax, fabsf(f[i]));
    }
    for (int o = cpg >> 1; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (!live) continue;
    const float sc = fmaxf(amax, kGroupEps) * (1.0f / kFp8Max);
    if (kc % cpg == 0) s[(long long)m * ng + kc / cpg] = sc;
    uint8_t b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b[i] = b200::f32_to_e4m3(fmaxf(fminf(f[i] / sc, kFp8Max), -kFp8Max));
    *reinterpret_cast<uint2*>(q + (long long)m * K + 8 * kc) = *reinterpret_cast<const uint2*>(b);
  }
}

template <typename T>
int launch_silu(const void* x, long long stride_x, int rows, int d, void* q, float* scale,
                void* act, int group, cudaStream_t stream) {
  const bool vec = (d % 8 == 0) && (stride_x % 8 == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(q) & 7) == 0) &&
                   (act == nullptr || (reinterpret_cast<uintptr_t>(act) & 15) == 0);
  const dim3 grid((rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA), block(32 * ROWS_PER_CTA);
  const T* xp = static_cast<const T*>(x);
  uint8_t* qp = static_cast<uint8_t*>(q);
  T* ap = static_cast<T*>(act);
  if (group == 0) {
    const int nchunk = d / 8;
    if (vec && nchunk <= 32)
      silu_mul_quant_reg_kernel<T, 1><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
    else if (vec && nchunk <= 64)
      silu_mul_quant_reg_kernel<T, 2><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
    else if (vec && nchunk <= 128)
      silu_mul_quant_reg_kernel<T, 4><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
    else if (vec)
      silu_mul_quant_kernel<T, true, 0><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
    else
      silu_mul_quant_kernel<T, false, 0><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
  } else {
    if (!vec || d % 128) return -3;
    silu_mul_quant_kernel<T, true, 128><<<grid, block, 0, stream>>>(xp, stride_x, rows, d, qp, scale, ap);
  }
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// Fused silu_and_mul + FP8 quant of x = [rows, 2*d] (gate | up), row stride `stride_x`
// elements; dtype 0 = bf16, 1 = f16. q: e4m3 [rows, d]; scale: fp32 [rows] (group == 0) or
// [rows, d/128] (group == 128); act: optional [rows, d] activation in x's dtype (nullable).
// Mirrors silu_mul_quant (kernels/fused_silu_mul_quant.py:75-101). Returns 0, -1 for a
// shape the reference's supported() refuses (d > 8192 / d < 0), -2 for a bad dtype, -3 for
// an unaligned group-128 call, else a CUDA error code.
int b200_silu_mul_quant(const void* x, int rows, int d, long long stride_x, int dtype, void* q,
                        float* scale, void* act, int group, cudaStream_t stream) {
  if (rows < 0 || d < 0 || d > 8192) return -1;
  if (group != 0 && group != 128) return -3;
  if (rows == 0 || d == 0) return 0;
  if (dtype == 0) return launch_silu<__nv_bfloat16>(x, stride_x, rows, d, q, scale, act, group, stream);
  if (dtype == 1) return launch_silu<__half>(x, stride_x, rows, d, q, scale, act, group, stream);
  return -2;
}

// scaled_fp8_quant(x, use_per_token_if_dynamic=True) of a [rows, K] activation with row
// stride `stride_x` (the MoE hidden-state quant behind fp8_quant_shared,
// patches/model_executor/kernels/linear/mxfp4/r4dhip.py.diff L19-34): q e4m3 [rows, K]
// contiguous, scale fp32 [rows]; scale_ub: optional device fp32 scalar that caps the row
// amax (nullable). dtype 0 = bf16, 1 = f16. Returns 0, -1 for negative sizes or
// stride_x < K, -2 for a bad dtype, else a CUDA error code.
int b200_per_token_quant_fp8(const void* x, int rows, int K, long long stride_x, int dtype,
                             const float* scale_ub, void* q, float* scale, cudaStream_t stream) {
  if (rows < 0 || K < 0 || (rows > 1 && stride_x < K)) return -1;
  if (dtype != 0 && dtype != 1) return -2;
  if (rows == 0) return 0;
  if (dtype == 0) return launch_token_quant<__nv_bfloat16>(x, stride_x, rows, K, scale_ub, q, scale, stream);
  return launch_token_quant<__half>(x, stride_x, rows, K, scale_ub, q, scale, stream);
}

// per_token_group_quant_fp8(x, group) (called at kernels/fp8_target_lmhead.py:73) for a
// [M, K] activation with row stride `stride_x`: q e4m3 [M, K] contiguous, s fp32 [M, K/group]
// row-major. group in {32, 64, 128}; K % group == 0; 16-byte aligned rows.
int b200_per_token_group_quant_fp8(const void* x, int M, int K, long long stride_x, int dtype,
                                   int group, void* q, float* s, cudaStream_t stream) {
  if (M < 0 || K < 0) return -1;
  if (group != 32 && group != 64 && group != 128) return -3;
  if (K % group || stride_x % 8 || (reinterpret_cast<uintptr_t>(x) & 15)) return -3;
  if (M == 0 || K == 0) return 0;
  const long long nchunks = (long long)M * K / 8;
  const long long nblk = (nchunks + 255) / 256;
  const int grid = (int)(nblk < 4096 ? nblk : 4096);
  if (dtype == 0)
    group_quant_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(x), stride_x, M, K, group, static_cast<uint8_t*>(q), s);
  else if (dtype == 1)
    group_quant_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half*>(x), stride_x,
                                                         M, K, group, static_cast<uint8_t*>(q), s);
  else
    return -2;
  return (int)cudaGetLastError();
}

}  // extern "C"

// Shared device helpers for the B200 (sm_100a) decode hot-path kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#define B200_DEVINL __device__ __forceinline__

namespace b200 {

B200_DEVINL unsigned lane_id() { return threadIdx.x & 31u; }

B200_DEVINL unsigned lanemask_lt() {
  unsigned m;
  asm volatile("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

B200_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- warp / block reductions ------------------------------------------------------------

template <typename T>
B200_DEVINL T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

B200_DEVINL float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Inclusive warp scan of an int.
B200_DEVINL int warp_inclusive_scan(int v) {
  const int l = (int)lane_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (l >= o) v += n;
  }
  return v;
}

// ---- mbarrier (shared::cta) --------------------------------------------------------------

B200_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

B200_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

B200_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

B200_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

B200_DEVINL bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

B200_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. try_wait suspends the thread in hardware until the phase
// completes or a short system time limit passes, so a waiting warp costs no issue slots and
// wakes as soon as the phase flips. Returns false once `deadline_ns` (globaltimer) has passed;
// the caller then records an error and leaves instead of waiting forever.
B200_DEVINL bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint64_t deadline_ns) {
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 15u) == 0 && globaltimer_ns() > deadline_ns) return false;
  }
  return true;
}

// Stage tags of a ring whose slots several consumer warps share: the producer stores (release)
// the index of the stage it is about to issue into a slot; a consumer that sees its stage's
// index there (acquire) knows the slot's previous round has been consumed, so its parity wait
// on the slot's barrier can only end on this stage's own phase.
B200_DEVINL void tag_publish(int* tag, int q) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(tag)), "r"(q) : "memory");
}

B200_DEVINL bool tag_wait_bounded(const int* tag, int q, uint64_t deadline_ns) {
  for (uint32_t n = 0;; ++n) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(tag)) : "memory");
    if (v == q) return true;
    if ((n & 63u) == 63u && globaltimer_ns() > deadline_ns) return false;
  }
}

// 1-D bulk copy global -> shared, completion counted on `bar` (transaction bytes).
// Both addresses 16-byte aligned and `bytes` a multiple of 16.
B200_DEVINL void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 evict-first hint for data streamed once (lm_head weights).
B200_DEVINL void bulk_g2s_stream(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1], %2, [%3], %4;" ::"r"(smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

B200_DEVINL uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- shared-memory vector loads ------------------------------------------------------------

B200_DEVINL uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// ---- warp-level tensor-core MMAs (legacy mma.sync, used for the M <= 16 GEMVs) -------------

// D(16x8 f32) += A(16x32 e4m3, row) * B(32x8 e4m3, col)
// (Not volatile: pure register math, so the compiler may overlap it with the next loads.)
B200_DEVINL void mma_e4m3_16832(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D(16x8 f32) += A(16x16 f16, row) * B(16x8 f16, col)
B200_DEVINL void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                               uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- conversions -----------------------------------------------------------------------------

// fp32 -> e4m3 (round to nearest even, saturating to +-448), one byte.
B200_DEVINL uint8_t f32_to_e4m3(float v) {
  return (uint8_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

B200_DEVINL uint32_t pack4_e4m3(float a, float b, float c, float d) {
  return (uint32_t)f32_to_e4m3(a) | ((uint32_t)f32_to_e4m3(b) << 8) |
         ((uint32_t)f32_to_e4m3(c) << 16) | ((uint32_t)f32_to_e4m3(d) << 24);
}

// Online (max, first-argmax, sum of exp) state for one logit row. The exponentials use the
// __expf intrinsic: every argument is <= 0 (a logit minus a running max), where its relative
// error stays near 1e-6, far inside what the log-sum-exp needs, at a few instructions each.
struct RowStat {
  float m;    // running max
  int idx;    // first index attaining m
  float s;    // sum of exp(v - m)
};

B200_DEVINL void rowstat_init(RowStat& r) {
  r.m = -INFINITY;
  r.idx = 0x7fffffff;
  r.s = 0.f;
}

// Push one logit. A tie with the running max keeps the smaller index, so the result does not
// depend on the order in which rows arrive.
B200_DEVINL void rowstat_push(RowStat& r, float v, int idx) {
  if (v > r.m || (v == r.m && idx < r.idx)) {
    r.s = r.s * __expf(r.m - v) + 1.f;
    r.m = v;
    r.idx = idx;
  } else {
    r.s += __expf(v - r.m);
  }
}

// Merge two states in any order: larger max wins, equal max takes the smaller index.
B200_DEVINL RowStat rowstat_merge(const RowStat& a, const RowStat& b) {
  RowStat o;
  if (a.m > b.m || (a.m == b.m && a.idx <= b.idx)) {
    o.m = a.m;
    o.idx = a.idx;
  } else {
    o.m = b.m;
    o.idx = b.idx;
  }
  const float sa = (a.s > 0.f) ? a.s * __expf(a.m - o.m) : 0.f;
  const float sb = (b.s > 0.f) ? b.s * __expf(b.m - o.m) : 0.f;
  o.s = sa + sb;
  return o;
}

// Push 32 consecutive logits (indices idx0 .. idx0 + 31) at once: their max and first argmax
// by trees over independent values and the sum of exp by 32 independent exponentials, then one
// merge -- a short dependency chain instead of 32 dependent exponentials.
B200_DEVINL void rowstat_push32(RowStat& r, const float (&v)[32], int idx0) {
  float t[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) t[i] = fmaxf(v[i], v[i + 16]);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) t[i] = fmaxf(t[i], t[i + w]);
  }
  const float m = t[0];
  int ir = 31;
#pragma unroll
  for (int i = 31; i >= 0; --i) ir = (v[i] == m) ? i : ir;
  float e[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) e[i] = __expf(v[i] - m) + __expf(v[i + 16] - m);
#pragma unroll
  for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
    for (int i = 0; i < w; ++i) e[i] += e[i + w];
  }
  RowStat b;
  b.m = m;
  b.idx = idx0 + ir;
  b.s = e[0];
  r = rowstat_merge(r, b);
}

B200_DEVINL RowStat rowstat_shfl_xor(const RowStat& r, int mask) {
  RowStat o;
  o.m = __shfl_xor_sync(0xffffffffu, r.m, mask);
  o.idx = __shfl_xor_sync(0xffffffffu, r.idx, mask);
  o.s = __shfl_xor_sync(0xffffffffu, r.s, mask);
  return o;
}

}  // namespace b200

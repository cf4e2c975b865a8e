// Small-M lm_head GEMVs for B200 (sm_100a): FP8 128x128 block-scaled and W4 group-128.
//
//   FP8: y[m, n] = sum_kb xs[m,kb] * ws[n/128,kb] * sum_{k in kb} qx[m,k] * wq[n,k]
//        (the operand contract of fp8hip_gemm_w8a8 / hcq_gemm_fp8blk_nt_m16,
//        kernels/experimental/fp8skinny/hcq_fp8skinny.hip:1-50); with the activation quant
//        per_token_group_quant_fp8(x, 128) fused into the prologue (kernels/fp8_target_lmhead.py:73).
//   W4:  y[m, n] = sum_g scale[n,g] * sum_{k in g} f16(x[m,k]) * (q[n,k] - zero[n,g])
//        (r4d_gemm_w4a16_nt_m64's math, kernels/draft_w4_lmhead.py:4-50), fp32 accumulation.
//   Optional fused epilogue: per row m, max / first-index argmax / logsumexp over the N
//   outputs of this call (the local argmax of mtp.py.diff L211-214, plus the logsumexp).
//
// Decode M is 1..16 here, so the weight stream is the whole cost. Per CTA (one per SM):
//   * warp 0 lane 0 streams the CTA's contiguous range of 16-row strips with 1-D bulk async
//     copies (cp.async.bulk, L2 evict-first) into a ring of shared-memory stages; each stage
//     is one strip's run of 128-K blocks, contiguous in the packed layout, so one copy fills
//     it. Full / empty mbarriers carry the hand-off; every wait is bounded by %globaltimer
//     and reports a timeout through an error word instead of hanging.
//   * 4 consumer warps take whole strips in turn. A strip is 16 weight rows, which is the A
//     operand of a warp MMA: FP8 uses mma.sync m16n8k32 e4m3 (128-bit shared loads straight
//     into A fragments), W4 widens nibbles to f16 in registers with one lop3 + one hadd2 per
//     pair ((nibble | 0x6400) - (1024 + zero) is exact in f16) and uses m16n8k16 f16. The
//     activation (<= 16 tokens) is the B operand from shared memory. Block / group scales are
//     applied in fp32 once per 128-K block.
//   * the activation prologue (quantize or convert x into shared memory) runs on the
//     consumer warps while the producer already streams the first stages.
// The weight never passes through registers of more than one warp and never touches L1; the
// CTA keeps (stages x stage bytes), ~160 KB, of weight reads in flight.
//
// Packed layouts (their own, B200 format; codes / scales / zeros are the reference's):
//   FP8 wq: [N/16 strips][K/128][16 rows][128 B]; 16-byte chunk c of row r at chunk c^(r&7).
//   W4  wq: [N/16][K/128][2][8 g][4 t][4 words] u32; word w of lane (g,t) = codes of
//           k = 128kb + 32w + 8t + j, code j in nibble (j&1)*4 + (j>>1), offset binary.
//   W4  wsz: int32 [N/16, K/128, 16] = f16 scale | f16(-(1024 + zero)) << 16
//           (draft_w4_lmhead.py:47-48, unchanged).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace {

constexpr int NC_FP8 = 4;                // consumer warps of the FP8 GEMV
constexpr int NC_W4 = 8;                 // consumer warps of the W4 GEMV (more ALU per byte), M <= 8
constexpr int NC_W4_WIDE = 6;            // ... and for 8 < M <= 16, where the larger activation
                                         // region leaves fewer stages (see plan())
constexpr int MAXM = 16;                 // tokens per GEMV launch
constexpr int SMEM_CAP = 227 * 1024;
constexpr int MAX_STAGES = 16;
constexpr int FP8_KB_BYTES = 16 * 128;   // one strip x one 128-K block
constexpr int W4_KB_BYTES = 16 * 64;
constexpr int W4_SZ_BYTES = 16 * 4;     // per strip and 128-K block: 16 rows x (f16 scale | f16 -(1024+zero))
constexpr int W4S_SZ_BYTES = 16 * 2;    // symmetric format: 16 rows x bf16 scale (zero fixed at 8)
constexpr uint64_t WAIT_NS = 2000000000ull;   // 2 s bound on any pipeline wait

enum Kind { FP8_QUANT = 0, FP8_PREQ = 1, W4_BF16 = 2, W4_F16 = 3, W4S_BF16 = 4, W4S_F16 = 5 };
// W4 kinds: activation bf16 or f16; W4S = the symmetric format (codes q in 0..15 mean q - 8,
// one bf16 scale per row and 128-K group).
__host__ __device__ constexpr bool kind_w4(int k) { return k >= W4_BF16; }
__host__ __device__ constexpr bool kind_w4s(int k) { return k >= W4S_BF16; }
__host__ __device__ constexpr bool kind_bf16x(int k) { return k == W4_BF16 || k == W4S_BF16; }
__host__ __device__ constexpr int kind_sz_bytes(int k) { return kind_w4s(k) ? W4S_SZ_BYTES : W4_SZ_BYTES; }

__device__ int g_lmhead_err = 0;         // 1 = a pipeline wait timed out

struct Params {
  const void* x;
  const float* xs_in;
  int M, K, N, n_valid;
  long long vocab_offset;
  const uint8_t* w;
  const void* wscale;
  __nv_bfloat16* y;
  long long ldy;
  float* row_max;
  long long* row_arg;
  float* row_lse;
  uint8_t* qx_out;
  float* xs_out;
  char* ws;          // workspace base (nullptr: none)
  float* partial;
  int kps;           // 128-K blocks per stage (tcgen05 path: TMEM accumulators)
  int nstage;
  int stage_bytes;
  int xs_stride;     // bytes per activation row in shared memory
  int x_off, xs_off, ring_off;
  int pdl;           // 1: launched as the programmatic dependent of the activation kernel
  int kw;            // tcgen05 path: 128-K blocks per stage
  int cs_off;        // tcgen05 path: per-accumulator scale vectors in shared memory
  int tagged;        // GEMV: consumers check stage tags (the ring's slots are not owned)
  float* px;         // tcgen05 path: partial accumulators of blocks split along K
  int* flags;        // tcgen05 path: split pairs' tickets and ready flags
  // vocabulary-sharded combine fused into the statistics merge (peers == nullptr: none)
  char* const* peers;
  unsigned long long* counters;
  int rank, world, M_cap, m_base;
};

// Release / acquire on a gpu-scope counter (the in-kernel finish of split tcgen05 pairs).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int NC>
__device__ __forceinline__ void consumer_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(NC * 32) : "memory");
}

// Programmatic dependent launch: the dependent grid may start while its primary still runs;
// griddep_wait() blocks until the primary grid has completed and its writes are visible.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));   // (a & b) | c
  return d;
}

__device__ __forceinline__ uint32_t hadd2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t hfma2_u32(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Offset-binary nibbles -> (code - zero) as f16x2, exactly. nz holds f16(-(1024 + zero)) in
// both halves, nz64 = nz + 960 = f16(-(64 + zero)). Pairs 0 and 2 (nibbles 0 and 2 of each
// half-word): (w & 0x000F000F) | 0x6400 gives 1024 + code, plus nz. Pairs 1 and 3 are masked in
// place (0x00F0 | 0x6400 gives 1024 + 16 code) and fma'd by 1/16 and nz64: 64 + code - 64 - zero.
// Every value is a small integer, so each f16 operation is exact. One shift serves pairs 2, 3.
__device__ __forceinline__ void w4_dequant_word(uint32_t w, uint32_t nz, uint32_t nz64, uint32_t (&o)[4]) {
  const uint32_t w8 = w >> 8;
  o[0] = hadd2_u32(lop3_and_or(w, 0x000F000Fu, 0x64006400u), nz);
  o[1] = hfma2_u32(lop3_and_or(w, 0x00F000F0u, 0x64006400u), 0x2C002C00u, nz64);     // 1/16
  o[2] = hadd2_u32(lop3_and_or(w8, 0x000F000Fu, 0x64006400u), nz);
  o[3] = hfma2_u32(lop3_and_or(w8, 0x00F000F0u, 0x64006400u), 0x2C002C00u, nz64);
}

// ---- activation prologue -----------------------------------------------------------------
//
// FP8_QUANT: quantize x (bf16 [M, K]) per token group of 128 straight into shared memory
//   (bit-identical to b200_per_token_group_quant_fp8: s = max(amax, 1e-10) * (1/448)); used
//   when the caller gives no workspace.
// FP8_PREQ: e4m3 rows [M, K] (+ fp32 scales [M, K/128]) arrive by one bulk copy per row; with
//   p.pdl they were written by act_rows_kernel, this kernel's programmatic primary.
// W4_*: the raw activation rows arrive by one bulk copy per row and bf16 is rounded to f16 in
//   shared memory (round to nearest even, i.e. x.to(float16)).
// Rows >= M are zero (and their scales 0), so they add nothing to any accumulator.
template <int KIND, int NC>
__device__ void load_activation(const Params& p, char* sm, int rows_x, uint64_t* x_bar,
                                uint64_t deadline, bool* ok) {
  const int ctid = threadIdx.x - 32;            // consumer thread 0..NC*32-1
  const int KB = p.K / 128;
  uint8_t* X = reinterpret_cast<uint8_t*>(sm + p.x_off);
  float* xs = reinterpret_cast<float*>(sm + p.xs_off);
  if (KIND == FP8_QUANT) {
    const int half = ctid >> 4, hl = ctid & 15;  // half-warps, 16 lanes x 8 elements
    const unsigned hmask = 0xffffu << (16 * ((ctid >> 4) & 1));
    const int ngroups = rows_x * KB;
    for (int gi = half; gi < ngroups; gi += NC * 2) {
      const int m = gi / KB, kb = gi % KB;
      uint8_t* dst = X + m * p.xs_stride + kb * 128 + hl * 8;
      if (m >= p.M) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(0, 0);
        if (hl == 0) xs[m * KB + kb] = 0.f;
        continue;
      }
      const __nv_bfloat16* src = static_cast<const __nv_bfloat16*>(p.x) + (long long)m * p.K + kb * 128 + hl * 8;
      const uint4 r = *reinterpret_cast<const uint4*>(src);
      const __nv_bfloat16* rv = reinterpret_cast<const __nv_bfloat16*>(&r);
      float f[8];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        f[i] = __bfloat162float(rv[i]);
        amax = fmaxf(amax, fabsf(f[i]));
      }
#pragma unroll
      for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(hmask, amax, o));
      const float sc = fmaxf(amax, 1e-10f) * (1.0f / 448.0f);
      uint2 b;
      b.x = b200::pack4_e4m3(fmaxf(fminf(f[0] / sc, 448.f), -448.f), fmaxf(fminf(f[1] / sc, 448.f), -448.f),
                             fmaxf(fminf(f[2] / sc, 448.f), -448.f), fmaxf(fminf(f[3] / sc, 448.f), -448.f));
      b.y = b200::pack4_e4m3(fmaxf(fminf(f[4] / sc, 448.f), -448.f), fmaxf(fminf(f[5] / sc, 448.f), -448.f),
                             fmaxf(fminf(f[6] / sc, 448.f), -448.f), fmaxf(fminf(f[7] / sc, 448.f), -448.f));
      *reinterpret_cast<uint2*>(dst) = b;
      if (hl == 0) xs[m * KB + kb] = sc;
      if (p.qx_out != nullptr && blockIdx.x == 0) {
        *reinterpret_cast<uint2*>(p.qx_out + (long long)m * p.K + kb * 128 + hl * 8) = b;
        if (hl == 0) p.xs_out[m * KB + kb] = sc;
      }
    }
    return;
  }
  constexpr bool IS_W4 = kind_w4(KIND);
  const int row_bytes = IS_W4 ? 2 * p.K : p.K;
  if (p.pdl) griddep_wait();
  if (ctid == 0) {
    b200::mbar_arrive_expect_tx(x_bar, (uint32_t)(p.M * row_bytes));
    for (int m = 0; m < p.M; ++m)
      b200::bulk_g2s(X + m * p.xs_stride, static_cast<const uint8_t*>(p.x) + (long long)m * row_bytes,
                     row_bytes, x_bar);
  }
  // zero rows >= M while the copies fly; scales straight from global memory
  for (int i = ctid; i < (rows_x - p.M) * (row_bytes / 16); i += NC * 32) {
    const int m = p.M + i / (row_bytes / 16), c = i % (row_bytes / 16);
    *reinterpret_cast<uint4*>(X + m * p.xs_stride + c * 16) = make_uint4(0, 0, 0, 0);
  }
  if (!IS_W4)
    for (int i = ctid; i < rows_x * KB; i += NC * 32) xs[i] = (i / KB < p.M) ? p.xs_in[i] : 0.f;
  *ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(x_bar, 0, deadline));
  if (kind_bf16x(KIND)) {
    consumer_bar<NC>();                           // (every consumer warp reaches it)
    if (!*ok) return;
    for (int i = ctid; i < p.M * (p.K / 8); i += NC * 32) {
      const int m = i / (p.K / 8), c = i % (p.K / 8);
      uint4* q = reinterpret_cast<uint4*>(X + m * p.xs_stride + c * 16);
      const uint4 r = *q;
      const __nv_bfloat16* rv = reinterpret_cast<const __nv_bfloat16*>(&r);
      __half h[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __float2half_rn(__bfloat162float(rv[j]));
      *q = *reinterpret_cast<const uint4*>(h);
    }
  }
}

// ---- per-strip consumer math ----------------------------------------------------------------

// Shared-memory operands are read through plain pointers (not volatile asm), so the compiler
// can issue block j + 1's loads while block j's MMAs run; the stage's mbarrier wait, an asm
// with a memory clobber, still orders them after the copy has landed.
template <int NT8>
__device__ __forceinline__ void fp8_stage(const Params& p, const char* stage, const char* xbase,
                                          const float* xs, int kb0, int nkb, int strip,
                                          float (&tot)[NT8][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int KB = p.K / 128;
  const float* ws = static_cast<const float*>(p.wscale) + (long long)(strip >> 3) * KB;
  const float wsv = (lane < nkb) ? __ldg(ws + kb0 + lane) : 0.f;
  const int c0 = ((t ^ g) & 7) * 16, c1 = (((t + 4) ^ g) & 7) * 16;
#pragma unroll 2
  for (int j = 0; j < nkb; ++j) {
    const float sw = __shfl_sync(0xffffffffu, wsv, j);
    const char* tile = stage + j * FP8_KB_BYTES;
    const uint4 A0 = *reinterpret_cast<const uint4*>(tile + g * 128 + c0);
    const uint4 A1 = *reinterpret_cast<const uint4*>(tile + g * 128 + c1);
    const uint4 B0 = *reinterpret_cast<const uint4*>(tile + (g + 8) * 128 + c0);
    const uint4 B1 = *reinterpret_cast<const uint4*>(tile + (g + 8) * 128 + c1);
    const uint32_t wa[8] = {A0.x, A0.y, A0.z, A0.w, A1.x, A1.y, A1.z, A1.w};
    const uint32_t wb[8] = {B0.x, B0.y, B0.z, B0.w, B1.x, B1.y, B1.z, B1.w};
    const int kb = kb0 + j;
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt) {
      const char* xr = xbase + (8 * nt + g) * p.xs_stride + kb * 128;
      const uint4 X0 = *reinterpret_cast<const uint4*>(xr + t * 16);
      const uint4 X1 = *reinterpret_cast<const uint4*>(xr + (t + 4) * 16);
      const uint32_t xw[8] = {X0.x, X0.y, X0.z, X0.w, X1.x, X1.y, X1.z, X1.w};
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; ++s)
        b200::mma_e4m3_16832(acc, wa[2 * s], wb[2 * s], wa[2 * s + 1], wb[2 * s + 1], xw[2 * s], xw[2 * s + 1]);
      const float s0 = sw * xs[(8 * nt + 2 * t) * KB + kb];
      const float s1 = sw * xs[(8 * nt + 2 * t + 1) * KB + kb];
      tot[nt][0] = fmaf(acc[0], s0, tot[nt][0]);
      tot[nt][1] = fmaf(acc[1], s1, tot[nt][1]);
      tot[nt][2] = fmaf(acc[2], s0, tot[nt][2]);
      tot[nt][3] = fmaf(acc[3], s1, tot[nt][3]);
    }
  }
}

template <int NT8, bool SYM>
__device__ __forceinline__ void w4_stage(const Params& p, const char* stage, const char* xbase, int kb0,
                                         int nkb, float (&tot)[NT8][4]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const char* szbase = stage + p.kps * W4_KB_BYTES;
#pragma unroll 2
  for (int j = 0; j < nkb; ++j) {
    const char* tile = stage + j * W4_KB_BYTES;
    const uint4 A = *reinterpret_cast<const uint4*>(tile + (g * 4 + t) * 16);
    const uint4 B = *reinterpret_cast<const uint4*>(tile + ((8 + g) * 4 + t) * 16);
    float scA, scB;
    uint32_t nzA, nzB;
    if constexpr (SYM) {
      // bf16 scale; zero 8, so (nibble | 0x6400) + f16(-1032) = q - 8 exactly
      const unsigned short sa = *reinterpret_cast<const unsigned short*>(szbase + j * W4S_SZ_BYTES + g * 2);
      const unsigned short sb = *reinterpret_cast<const unsigned short*>(szbase + j * W4S_SZ_BYTES + (g + 8) * 2);
      scA = __uint_as_float((uint32_t)sa << 16);
      scB = __uint_as_float((uint32_t)sb << 16);
      nzA = nzB = 0xE408E408u;                          // f16(-1032) twice
    } else {
      const uint32_t szA = *reinterpret_cast<const uint32_t*>(szbase + j * W4_SZ_BYTES + g * 4);
      const uint32_t szB = *reinterpret_cast<const uint32_t*>(szbase + j * W4_SZ_BYTES + (g + 8) * 4);
      scA = __half2float(__ushort_as_half((unsigned short)(szA & 0xffffu)));
      scB = __half2float(__ushort_as_half((unsigned short)(szB & 0xffffu)));
      nzA = (szA >> 16) | (szA & 0xffff0000u);
      nzB = (szB >> 16) | (szB & 0xffff0000u);
    }
    const uint32_t wa[4] = {A.x, A.y, A.z, A.w}, wb[4] = {B.x, B.y, B.z, B.w};
    const uint32_t nzA64 = hadd2_u32(nzA, 0x63806380u), nzB64 = hadd2_u32(nzB, 0x63806380u);   // + 960
    const int kb = kb0 + j;
    float acc[NT8][4];
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      uint32_t pa[4], pb[4];
      w4_dequant_word(wa[w], nzA, nzA64, pa);
      w4_dequant_word(wb[w], nzB, nzB64, pb);
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) {
        const uint4 X = *reinterpret_cast<const uint4*>(xbase + (8 * nt + g) * p.xs_stride + (kb * 128 + 32 * w + 8 * t) * 2);
        b200::mma_f16_16816(acc[nt], pa[0], pb[0], pa[1], pb[1], X.x, X.y);
        b200::mma_f16_16816(acc[nt], pa[2], pb[2], pa[3], pb[3], X.z, X.w);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT8; ++nt) {
      tot[nt][0] = fmaf(acc[nt][0], scA, tot[nt][0]);
      tot[nt][1] = fmaf(acc[nt][1], scA, tot[nt][1]);
      tot[nt][2] = fmaf(acc[nt][2], scB, tot[nt][2]);
      tot[nt][3] = fmaf(acc[nt][3], scB, tot[nt][3]);
    }
  }
}

// ---- row statistics: CTA partial per token, merged by stats_merge_kernel ---------------------
// red[w * stride + m] holds warp w's state for token m (nred warps). The workspace partials
// are token-major ([m][slot], G slots) so the merge reads them coalesced.

// Write this CTA's merged state per token into partial slot `slot`. Every thread calls it
// after a barrier that published `red`.
__device__ __forceinline__ void stats_write_partial(const Params& p, const b200::RowStat* red, int stride,
                                                    int nred, int slot, int G) {
  if (threadIdx.x < p.M) {
    const int m = threadIdx.x;
    b200::RowStat r = red[m];
    for (int w = 1; w < nred; ++w) r = b200::rowstat_merge(r, red[w * stride + m]);
    float* dst = p.partial + ((long long)m * G + slot) * 3;
    dst[0] = r.m;
    dst[1] = __int_as_float(r.idx);
    dst[2] = r.s;
  }
}

// ---- the kernel ------------------------------------------------------------------------------

// Shared-memory header of the GEMV: full/empty barriers [0, 256), the activation barrier at
// 256, the stage tags of the ring slots from 320, per-warp row statistics from 384, the "last
// CTA" flag after them.
constexpr int GEMV_XBAR = 256;
constexpr int GEMV_TAGS = 320;
constexpr int GEMV_HDR_RED = 384;
__host__ __device__ constexpr int gemv_hdr(int nc) { return GEMV_HDR_RED + nc * MAXM * 12 + 16; }

template <int KIND, int NT8, bool STATS, int NC, bool TAGGED>
__global__ void __launch_bounds__(32 * (NC + 1), 1) gemv_kernel(Params p) {
  extern __shared__ __align__(128) char sm[];
  constexpr bool IS_W4 = kind_w4(KIND);
  constexpr int KB_BYTES = IS_W4 ? W4_KB_BYTES : FP8_KB_BYTES;
  constexpr int SZB = kind_sz_bytes(KIND);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.K / 128;
  const int CH = (KB + p.kps - 1) / p.kps;
  const int nstrips_total = p.N / 16;
  const int s0 = (int)(((long long)blockIdx.x * nstrips_total) / gridDim.x);
  const int s1 = (int)(((long long)(blockIdx.x + 1) * nstrips_total) / gridDim.x);
  const int nst = (s1 - s0) * CH;

  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* x_bar = reinterpret_cast<uint64_t*>(sm + GEMV_XBAR);
  int* tag = reinterpret_cast<int*>(sm + GEMV_TAGS);
  b200::RowStat* red = reinterpret_cast<b200::RowStat*>(sm + GEMV_HDR_RED);   // [NC][MAXM]
  char* ring = sm + p.ring_off;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nstage; ++i) {
      b200::mbar_init(&full[i], 1);
      b200::mbar_init(&empty[i], 1);
      tag[i] = -1;
    }
    b200::mbar_init(x_bar, 1);
    b200::fence_mbar_init();
  }
  __syncthreads();
  const uint64_t deadline = b200::globaltimer_ns() + WAIT_NS;
  if (STATS) griddep_launch_dependents();   // stats_merge_kernel may be scheduled

  b200::RowStat st[NT8][2];
#pragma unroll
  for (int nt = 0; nt < NT8; ++nt) {
    b200::rowstat_init(st[nt][0]);
    b200::rowstat_init(st[nt][1]);
  }

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = b200::l2_policy_evict_first();
      int issued = 0;
      bool ok = true;
      for (int q = 0; q < nst; ++q) {
        const int slot = q % p.nstage, round = q / p.nstage;
        if (round > 0 && !b200::mbar_wait_bounded(&empty[slot], (round - 1) & 1, deadline)) {
          ok = false;
          break;
        }
        if (TAGGED) b200::tag_publish(&tag[slot], q);
        const int strip = s0 + q / CH, ch = q % CH;
        const int kb0 = ch * p.kps, nkb = min(p.kps, KB - kb0);
        const long long blk = (long long)strip * KB + kb0;
        char* dst = ring + slot * p.stage_bytes;
        const uint32_t wbytes = nkb * KB_BYTES;
        const uint32_t sbytes = IS_W4 ? nkb * SZB : 0;
        b200::mbar_arrive_expect_tx(&full[slot], wbytes + sbytes);
        b200::bulk_g2s_stream(dst, p.w + blk * KB_BYTES, wbytes, &full[slot], pol);
        if (IS_W4)
          b200::bulk_g2s(dst + p.kps * W4_KB_BYTES,
                         static_cast<const uint8_t*>(p.wscale) + blk * SZB, sbytes, &full[slot]);
        ++issued;
      }
      if (!ok) atomicExch(&g_lmhead_err, 1);
      // never leave with copies in flight: the last use of every slot must have landed
      for (int q = max(0, issued - p.nstage); q < issued; ++q)
        b200::mbar_wait_bounded(&full[q % p.nstage], (q / p.nstage) & 1, deadline + WAIT_NS);
    }
    __syncwarp();
  } else {
    // ---------------- consumers ----------------
    const int cw = warp - 1;
    bool ok = true;
    load_activation<KIND, NC>(p, sm, 8 * NT8, x_bar, deadline, &ok);
    consumer_bar<NC>();
    ok = ok && __all_sync(0xffffffffu, ok);
    const char* xbase = sm + p.x_off;
    const float* xs = reinterpret_cast<const float*>(sm + p.xs_off);
    const int g = lane >> 2, t = lane & 3;
    for (int ls = cw; ls < s1 - s0 && ok; ls += NC) {
      const int strip = s0 + ls;
      float tot[NT8][4];
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) tot[nt][0] = tot[nt][1] = tot[nt][2] = tot[nt][3] = 0.f;
      for (int ch = 0; ch < CH; ++ch) {
        const int q = ls * CH + ch, slot = q % p.nstage;
        // (tagged ring) the stage is in its slot, so the parity wait cannot end on the slot's
        // previous round, whose copy may still be landing; then it has landed
        const bool got = (!TAGGED || b200::tag_wait_bounded(&tag[slot], q, deadline)) &&
                         b200::mbar_wait_bounded(&full[slot], (q / p.nstage) & 1, deadline);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const char* stage = ring + slot * p.stage_bytes;
        const int kb0 = ch * p.kps, nkb = min(p.kps, KB - kb0);
        if (IS_W4)
          w4_stage<NT8, kind_w4s(KIND)>(p, stage, xbase, kb0, nkb, tot);
        else
          fp8_stage<NT8>(p, stage, xbase, xs, kb0, nkb, strip, tot);
        __syncwarp();
        if (lane == 0) b200::mbar_arrive(&empty[slot]);
      }
      if (!ok) break;
      // epilogue: rows n0+g, n0+g+8 ; tokens 8nt+2t, 8nt+2t+1
      const int n0 = strip * 16;
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt) {
        const int m0 = 8 * nt + 2 * t, m1 = m0 + 1;
        if (p.y != nullptr) {
          if (m0 < p.M) {
            p.y[(long long)m0 * p.ldy + n0 + g] = __float2bfloat16_rn(tot[nt][0]);
            p.y[(long long)m0 * p.ldy + n0 + g + 8] = __float2bfloat16_rn(tot[nt][2]);
          }
          if (m1 < p.M) {
            p.y[(long long)m1 * p.ldy + n0 + g] = __float2bfloat16_rn(tot[nt][1]);
            p.y[(long long)m1 * p.ldy + n0 + g + 8] = __float2bfloat16_rn(tot[nt][3]);
          }
        }
        if (STATS) {
          const int ia = n0 + g, ib = n0 + g + 8;
          const int gia = (int)(ia + p.vocab_offset), gib = (int)(ib + p.vocab_offset);
          if (ia < p.n_valid) {
            b200::rowstat_push(st[nt][0], tot[nt][0], gia);
            b200::rowstat_push(st[nt][1], tot[nt][1], gia);
          }
          if (ib < p.n_valid) {
            b200::rowstat_push(st[nt][0], tot[nt][2], gib);
            b200::rowstat_push(st[nt][1], tot[nt][3], gib);
          }
        }
      }
    }
    if (!ok) atomicExch(&g_lmhead_err, 1);
    if (STATS) {
      // merge over the 8 row groups (lanes with equal t), then publish per consumer warp
#pragma unroll
      for (int nt = 0; nt < NT8; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int msk = 4; msk < 32; msk <<= 1)
            st[nt][h] = b200::rowstat_merge(st[nt][h], b200::rowstat_shfl_xor(st[nt][h], msk));
      if (g == 0) {
#pragma unroll
        for (int nt = 0; nt < NT8; ++nt) {
          red[cw * MAXM + 8 * nt + 2 * t] = st[nt][0];
          red[cw * MAXM + 8 * nt + 2 * t + 1] = st[nt][1];
        }
      }
    }
  }

  if (!STATS) return;
  __syncthreads();
  stats_write_partial(p, red, MAXM, NC, blockIdx.x, gridDim.x);
}

// ---- tcgen05 path: 9 <= M <= 64 tokens ----------------------------------------------------------
//
// At these row counts the GEMV's warp MMAs would issue-bound the SM, so the contraction moves
// to the 5th-generation tensor core: D[128 weight rows, T tokens] (fp32, in TMEM) = W tile
// (A, 128 x 128 K, shared memory) x X tile (B, T x 128 K). A 128x128 weight tile is exactly one
// block-scale block, so every tile gets its own TMEM accumulator and the two scales are applied
// in fp32 when the epilogue reads it back:  y[n, t] += ws[n/128, kb] * xs[t, kb] * D_kb[n, t].
//
// The weight stream has to keep about 170 KB in flight per SM (loaded-HBM latency is 3-4 us),
// while a stage is held about 1 us after it lands (its MMAs run about 85 ns each whatever T
// is). So a stage carries the two 128-row blocks of a block PAIR at one 128-K block -- one
// 32 KB tensor-map copy, a (byte, row, strip, kb) box of 16 strips landing as two swizzled
// [128 rows][128 B] tiles -- and ONE activation tile both use; five such stages fit.
//   warp 0 (1 lane): the two copies of each stage (weights; T x 128 B pre-tiled activation);
//   warps 1-2      : (warp 1 also allocates TMEM) lane 0 of warp 1 + s issues the 4
//                    tcgen05.mma kind::f8f6f4 (K = 32 each) of block 2p + s into its next TMEM
//                    accumulator and commits it; both commit each stage's empty barrier. A
//                    thread issues an MMA only every ~120 ns, so one issuer per block matters;
//   warps 3-10     : two groups of four (group s = block 2p + s; warp & 3 = TMEM lane
//                    quarter): tcgen05.ld of the accumulator, fp32 scale-accumulate in
//                    registers, and per finished block the bf16 logits (lane = row: each token
//                    is one coalesced 64-byte store per warp) and per token the (max, first
//                    argmax, sum exp) by warp reductions.
// TMEM holds 512 / T accumulators, so the MMAs run ahead of the epilogue by 256 / T stages.
// The activation is quantized once per call by act_tiles_kernel into the workspace, already
// swizzled.
//
// Work split (stream-K): a unit is one stage (block pair, 128-K block); CTA c takes the
// contiguous units [U c / G, U (c+1) / G) of all U = ceil(nblk/2) * K/128, so no CTA does more
// than one unit above the mean (whole blocks per CTA would run 1187 blocks on 148 SMs as 9
// against 8, and a 149-block vocabulary shard as 2 against 1). A pair shared by several CTAs
// is finished by whichever of them arrives last: at the end of its run of the pair each
// epilogue warp takes a ticket for its 32 rows; all but the last leave their fp32 partial and
// a ready flag, and the last adds the partials in K order and writes the rows. Only the last
// ever waits, and only for warps that took their tickets before it, which are running and
// wait for nothing, so the kernel needs no CTA to be resident at the same time as another.
// Per token, each CTA leaves (max, argmax, sum exp) over the blocks it wrote, which
// stats_merge_kernel (the programmatic dependent) merges. With an odd block count the last
// pair's second block lies beyond the tensor: the copy fills it with zeros and nothing of it
// is written.

constexpr int TC_ISSUERS = 2;                       // MMA-issuing warps, one per block of a pair
constexpr int TC_SCALE_WARP = 1 + TC_ISSUERS;     // writes the epilogue's per-unit scale vectors
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_THREADS = 32 * (2 + TC_ISSUERS + TC_EPI_WARPS);
constexpr int TC_MAX_STAGES = 8;
constexpr int TC_MAX_BUF = 16;
constexpr int TC_TILE_W = 128 * 128;
constexpr int TC_PAIR_W = 2 * TC_TILE_W;
constexpr int TC_HDR = 512;                         // barriers, TMEM slot
constexpr int TC_MAX_GRID = 160;                    // partial-accumulator slots are sized for it
// Split-pair bookkeeping in the workspace's flag region (ints, zeroed by act_tiles_kernel on
// every call): a ticket per (pair's first CTA, block of the pair), then a ready flag per (CTA,
// its first or last pair, block, 32-row quarter).
constexpr int TC_TICKET_OFF = 0;
constexpr int TC_READY_OFF = TC_MAX_GRID * 2;
constexpr int TC_FLAG_INTS = TC_READY_OFF + TC_MAX_GRID * 2 * 2 * 4;

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Named barrier of the four epilogue warps of group g (ids 2 and 3; 0 is __syncthreads).
__device__ __forceinline__ void group_bar(int g) {
  asm volatile("bar.sync %0, 128;" ::"r"(2 + g) : "memory");
}

// Does CTA c begin a block pair that continues in later CTAs (its last pair, split)? Then the
// pair's blocks have statistics slots of their own (see fp8_tc_kernel).
__host__ __device__ __forceinline__ bool tc_begins_split(long long LU, int G, int KBS, int c, int& pair) {
  const long long lu0 = LU * c / G, lu1 = LU * (c + 1) / G;
  pair = (int)((lu1 - 1) / KBS);
  return (lu1 % KBS) != 0 && lu0 <= (long long)pair * KBS;
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr & 0x3FFFFu) >> 4);      // start address, bits [0,14)
  d |= (uint64_t)1 << 16;                                // leading byte offset (unused here)
  d |= (uint64_t)(1024 >> 4) << 32;                      // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                                // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                                // layout: SWIZZLE_128B
  return d;
}

__device__ __forceinline__ void tc_mma_f8(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   b200::smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// (a0, a1) += (v0 * c0, v1 * c1): two fused multiply-adds, each rounded once (round to nearest),
// in one packed instruction.
__device__ __forceinline__ void ffma2(float& a0, float& a1, float v0, float v1, float c0, float c1) {
  unsigned long long a = ((unsigned long long)__float_as_uint(a1) << 32) | __float_as_uint(a0);
  const unsigned long long v = ((unsigned long long)__float_as_uint(v1) << 32) | __float_as_uint(v0);
  const unsigned long long c = ((unsigned long long)__float_as_uint(c1) << 32) | __float_as_uint(c0);
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(a) : "l"(v), "l"(c));
  a0 = __uint_as_float((uint32_t)a);
  a1 = __uint_as_float((uint32_t)(a >> 32));
}

// The registers a tcgen05.ld writes are valid only after tcgen05.wait::ld; passing each value
// through an empty volatile asm placed after the wait keeps the compiler from using it earlier.
template <int N>
__device__ __forceinline__ void tmem_values_after_wait(float (&v)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+f"(v[i]));
}

// x (bf16 [M, K]) -> per-token group-128 quant, written as tiles qt[kb][tpad rows][128 B] in the
// 128-byte-swizzled layout (rows >= M zero) + scales xt[kb][tpad]; with qx_in set, re-tile an
// already quantized e4m3 [M, K] + xs [M, K/128] instead. Same formula as the standalone quant.
// grid = (K/128, tpad/8), 128 threads: half a warp per (row, 128-K block).
__global__ void __launch_bounds__(128)
    act_tiles_kernel(const __nv_bfloat16* __restrict__ x, const uint8_t* __restrict__ qx_in,
                     const float* __restrict__ xs_in, int M, int K, int tpad,
                     uint8_t* __restrict__ qt, float* __restrict__ xt, uint8_t* __restrict__ qx_out,
                     float* __restrict__ xs_out, int* __restrict__ flags, int nflags) {
  griddep_launch_dependents();              // the GEMM may start streaming weights now
  // the GEMM's split-pair tickets and ready flags start every call at zero (this kernel is
  // stream-ordered after the previous call, and the GEMM touches them only after
  // griddepcontrol.wait)
  if (blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < nflags; i += blockDim.x) flags[i] = 0;
  const int KB = K / 128, kb = blockIdx.x;
  const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
  const unsigned hmask = 0xffffu << (16 * (hw & 1));
  const int m = blockIdx.y * 8 + hw;
  uint2 b = make_uint2(0, 0);
  float sc = 0.f;
  if (m < M) {
    if (qx_in != nullptr) {
      b = *reinterpret_cast<const uint2*>(qx_in + (long long)m * K + kb * 128 + hl * 8);
      sc = xs_in[m * KB + kb];
    } else {
      const uint4 r = *reinterpret_cast<const uint4*>(x + (long long)m * K + kb * 128 + hl * 8);
      const __nv_bfloat16* rv = reinterpret_cast<const __nv_bfloat16*>(&r);
      float f[8];
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        f[i] = __bfloat162float(rv[i]);
        amax = fmaxf(amax, fabsf(f[i]));
      }
#pragma unroll
      for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(hmask, amax, o));
      sc = fmaxf(amax, 1e-10f) * (1.0f / 448.0f);
      b.x = b200::pack4_e4m3(fmaxf(fminf(f[0] / sc, 448.f), -448.f), fmaxf(fminf(f[1] / sc, 448.f), -448.f),
                             fmaxf(fminf(f[2] / sc, 448.f), -448.f), fmaxf(fminf(f[3] / sc, 448.f), -448.f));
      b.y = b200::pack4_e4m3(fmaxf(fminf(f[4] / sc, 448.f), -448.f), fmaxf(fminf(f[5] / sc, 448.f), -448.f),
                             fmaxf(fminf(f[6] / sc, 448.f), -448.f), fmaxf(fminf(f[7] / sc, 448.f), -448.f));
      if (qx_out != nullptr) {
        *reinterpret_cast<uint2*>(qx_out + (long long)m * K + kb * 128 + hl * 8) = b;
        if (hl == 0) xs_out[m * KB + kb] = sc;
      }
    }
  }
  if (m < tpad) {
    uint8_t* tile = qt + ((long long)kb * tpad + m) * 128;
    *reinterpret_cast<uint2*>(tile + (((hl >> 1) ^ (m & 7)) * 16) + (hl & 1) * 8) = b;
    if (hl == 0) xt[kb * tpad + m] = sc;
  }
}

// x (bf16 [M, K]) -> e4m3 rows qr [M, K] + fp32 scales sr [M, K/128] (row-major, the
// per_token_group_quant_fp8 layout): the programmatic primary of the FP8 GEMV, which pulls the
// rows with one bulk copy each. grid = (K/128, ceil(M/8)), half a warp per (row, 128-K block).
__global__ void __launch_bounds__(128)
    act_rows_kernel(const __nv_bfloat16* __restrict__ x, int M, int K, uint8_t* __restrict__ qr,
                    float* __restrict__ sr) {
  griddep_launch_dependents();
  const int KB = K / 128, kb = blockIdx.x;
  const int hw = threadIdx.x >> 4, hl = threadIdx.x & 15;
  const unsigned hmask = 0xffffu << (16 * (hw & 1));
  const int m = blockIdx.y * 8 + hw;
  if (m >= M) return;                        // a whole half-warp leaves together
  const uint4 r = *reinterpret_cast<const uint4*>(x + (long long)m * K + kb * 128 + hl * 8);
  const __nv_bfloat16* rv = reinterpret_cast<const __nv_bfloat16*>(&r);
  float f[8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    f[i] = __bfloat162float(rv[i]);
    amax = fmaxf(amax, fabsf(f[i]));
  }
#pragma unroll
  for (int o = 8; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(hmask, amax, o));
  const float sc = fmaxf(amax, 1e-10f) * (1.0f / 448.0f);
  uint2 b;
  b.x = b200::pack4_e4m3(fmaxf(fminf(f[0] / sc, 448.f), -448.f), fmaxf(fminf(f[1] / sc, 448.f), -448.f),
                         fmaxf(fminf(f[2] / sc, 448.f), -448.f), fmaxf(fminf(f[3] / sc, 448.f), -448.f));
  b.y = b200::pack4_e4m3(fmaxf(fminf(f[4] / sc, 448.f), -448.f), fmaxf(fminf(f[5] / sc, 448.f), -448.f),
                         fmaxf(fminf(f[6] / sc, 448.f), -448.f), fmaxf(fminf(f[7] / sc, 448.f), -448.f));
  *reinterpret_cast<uint2*>(qr + (long long)m * K + kb * 128 + hl * 8) = b;
  if (hl == 0) sr[m * KB + kb] = sc;
}

// Units of one CTA: the contiguous run [lu0, lu1) of all LU = npairs * KBS units (stream-K);
// unit lu is (block pair lu / KBS, 128-K block lu % KBS). A pair shared with other CTAs is
// begun by one CTA and continued by the next ones' FIRST runs.
struct TcWork {
  int KBS, G, c;
  long long LU, lu0, lu1;
  __device__ int total() const { return (int)(lu1 - lu0); }
  __device__ void unit(int i, int& pair, int& j) const {
    const long long lu = lu0 + i;
    pair = (int)(lu / KBS);
    j = (int)(lu % KBS);
  }
  // CTA that processes unit lu (the largest c with LU*c/G <= lu). The host keeps LU * G below
  // 2^31, so the arithmetic is 32-bit.
  __device__ int owner(long long lu) const { return (((int)lu + 1) * G - 1) / (int)LU; }
};

__device__ __forceinline__ TcWork tc_work(int npairs, int KBS, int G, int c) {
  TcWork w;
  w.G = G;
  w.c = c;
  w.KBS = KBS;
  w.LU = (long long)npairs * KBS;
  w.lu0 = w.LU * w.c / w.G;
  w.lu1 = w.LU * (w.c + 1) / w.G;
  return w;
}

// Output of one finished 128-row block: lane = row n0 + lane of the warp's 32 rows, acc[t] its
// logit for token t. Sixteen tokens at a time pass through the warp's [16][33] shared tile
// `tr`, after which lane (tt = lane & 15, rg = lane >> 4) holds rows n0 + 16 rg .. + 15 of
// token 16 ch + tt: two 16-byte stores of bf16 logits; the max over the 32 rows, the first row
// at it and the sum of exp(v - max) by trees over independent values and one shuffle across
// the two row groups. Lane tt (< 16) folds token 16 ch + tt's block result into st[ch].
constexpr int TC_CHUNK = 16;

template <int TPAD, bool STATS>
__device__ __forceinline__ void tc_block_rows(const Params& p, const float (&acc)[TPAD], int n0, int lane,
                                              float* tr, b200::RowStat (&st)[TPAD / TC_CHUNK]) {
  const int tt = lane & 15, rg = lane >> 4;
#pragma unroll
  for (int ch = 0; ch < TPAD / TC_CHUNK; ++ch) {
    if (TC_CHUNK * ch < p.M) {
#pragma unroll
      for (int i = 0; i < TC_CHUNK; ++i) tr[i * 33 + lane] = acc[TC_CHUNK * ch + i];
      __syncwarp();
      float v[16];
#pragma unroll
      for (int r = 0; r < 16; ++r) v[r] = tr[tt * 33 + 16 * rg + r];
      __syncwarp();
      const int t = TC_CHUNK * ch + tt;
      const bool live = t < p.M;
      if (live && p.y != nullptr) {
        __nv_bfloat162 h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        uint4* dst = reinterpret_cast<uint4*>(p.y + (long long)t * p.ldy + n0 + 16 * rg);
        dst[0] = *reinterpret_cast<const uint4*>(&h[0]);
        dst[1] = *reinterpret_cast<const uint4*>(&h[4]);
      }
      if (STATS) {
        float mt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mt[i] = fmaxf(v[i], v[i + 8]);
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1) {
#pragma unroll
          for (int i = 0; i < w; ++i) mt[i] = fmaxf(mt[i], mt[i + w]);
        }
        const float m = fmaxf(mt[0], __shfl_xor_sync(0xffffffffu, mt[0], 16));
        int it[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) it[i] = (v[i] == m) ? i : ((v[i + 8] == m) ? i + 8 : 0x7fffffff);
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1) {
#pragma unroll
          for (int i = 0; i < w; ++i) it[i] = min(it[i], it[i + w]);
        }
        const int ir0 = (it[0] == 0x7fffffff) ? 0x7fffffff : 16 * rg + it[0];
        const int ir = min(ir0, __shfl_xor_sync(0xffffffffu, ir0, 16));
        float et[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) et[i] = __expf(v[i] - m) + __expf(v[i + 8] - m);
#pragma unroll
        for (int w = 4; w >= 1; w >>= 1) {
#pragma unroll
          for (int i = 0; i < w; ++i) et[i] += et[i + w];
        }
        const float e = et[0] + __shfl_xor_sync(0xffffffffu, et[0], 16);
        if (live && rg == 0) {
          b200::RowStat b;
          b.m = m;
          b.idx = (int)(n0 + p.vocab_offset) + ir;
          b.s = e;
          st[ch] = b200::rowstat_merge(st[ch], b);
        }
      }
    }
  }
}

template <int TPAD, bool STATS>
__global__ void __launch_bounds__(TC_THREADS, 1)
    fp8_tc_kernel(const __grid_constant__ CUtensorMap wmap, Params p, const uint8_t* __restrict__ qt,
                  const float* __restrict__ xt) {
  extern __shared__ char sm_raw[];
  const uint32_t raw = b200::smem_u32(sm_raw);
  char* sm = sm_raw + ((1024u - (raw & 1023u)) & 1023u);
  constexpr int XT_BYTES = TPAD * 128;
  constexpr int STAGE = TC_PAIR_W + XT_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = p.K / 128;
  const int nblk = p.N / 128;
  const TcWork wk = tc_work((nblk + 1) / 2, KB, gridDim.x, blockIdx.x);
  const int total = wk.total();
  const int nstage = p.nstage, nbuf = p.kps;          // kps carries the accumulator count here

  uint64_t* w_full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* w_empty = w_full + TC_MAX_STAGES;
  uint64_t* a_full = w_empty + TC_MAX_STAGES;
  uint64_t* a_empty = a_full + TC_MAX_BUF;
  uint64_t* xs_bar = a_empty + TC_MAX_BUF;
  uint64_t* done_bar = xs_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  int* s_ticket = reinterpret_cast<int*>(tmem_slot + 2);       // [2 groups][2 parities]
  float* xs_s = reinterpret_cast<float*>(sm + p.xs_off);       // [KB][TPAD]
  float* c_s = reinterpret_cast<float*>(sm + p.cs_off);        // [accumulator][TPAD]
  char* ring = sm + p.ring_off;
  b200::RowStat st[TPAD / TC_CHUNK];        // epilogue lanes l < 16: tokens 16 ch + l

  if (threadIdx.x == 0) {
    for (int i = 0; i < nstage; ++i) {
      b200::mbar_init(&w_full[i], 1);
      b200::mbar_init(&w_empty[i], TC_ISSUERS);
    }
    for (int i = 0; i < nbuf; ++i) {
      b200::mbar_init(&a_full[i], 2);              // the MMAs' commit + the scale vector
      b200::mbar_init(&a_empty[i], 4);             // the four warps of the buffer's group
    }
    b200::mbar_init(xs_bar, 1);
    b200::mbar_init(done_bar, TC_ISSUERS);
    b200::fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(
                     b200::smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint64_t deadline = b200::globaltimer_ns() + WAIT_NS;
  griddep_launch_dependents();              // stats_merge_kernel may be scheduled as SMs free up

  if (warp == 0) {
    // ---------------- producer ----------------
    // Weight tiles do not depend on the activation kernel (this grid's programmatic primary),
    // so the first ring of weight tiles is issued before griddepcontrol.wait; each stage's
    // activation tile (and the scales) only after it.
    if (lane == 0) {
      const uint64_t pol = b200::l2_policy_evict_first();
      const uint64_t wmap_addr = reinterpret_cast<uint64_t>(&wmap);
      auto issue_w = [&](int it) {
        const int s = it % nstage;
        int pr, kb;
        wk.unit(it, pr, kb);
        b200::mbar_arrive_expect_tx(&w_full[s], STAGE);
        asm volatile(
            "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
            " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(b200::smem_u32(ring + s * STAGE)),
            "l"(wmap_addr), "r"(0), "r"(0), "r"(pr * 16), "r"(kb), "r"(b200::smem_u32(&w_full[s])),
            "l"(pol)
            : "memory");
      };
      auto issue_x = [&](int it) {
        const int s = it % nstage;
        int pr, kb;
        wk.unit(it, pr, kb);
        b200::bulk_g2s(ring + s * STAGE + TC_PAIR_W, qt + (long long)kb * XT_BYTES, XT_BYTES, &w_full[s]);
      };
      const int first = min(nstage, total);
      for (int it = 0; it < first; ++it) issue_w(it);
      if (p.pdl) griddep_wait();
      b200::mbar_arrive_expect_tx(xs_bar, TPAD * KB * 4);
      b200::bulk_g2s(xs_s, xt, TPAD * KB * 4, xs_bar);
      for (int it = 0; it < first; ++it) issue_x(it);
      int issued = first;
      bool ok = true;
      for (int it = first; it < total; ++it) {
        const int s = it % nstage, round = it / nstage;
        if (!b200::mbar_wait_bounded(&w_empty[s], (round - 1) & 1, deadline)) {
          ok = false;
          break;
        }
        issue_w(it);
        issue_x(it);
        ++issued;
      }
      if (!ok) atomicExch(&g_lmhead_err, 1);
      for (int q = max(0, issued - nstage); q < issued; ++q)
        b200::mbar_wait_bounded(&w_full[q % nstage], (q / nstage) & 1, deadline + WAIT_NS);
      b200::mbar_wait_bounded(xs_bar, 0, deadline + WAIT_NS);
    }
    __syncwarp();
  } else if (warp <= TC_ISSUERS) {
    // ---------------- MMA issuers: issuer `me` computes block 2p + me of every stage --------
    // (one thread each, doing nothing else: its loop sets the pace of the whole pipeline)
    if (lane == 0) {
      const int me = warp - 1;
      const uint32_t idesc = (1u << 4)                        // D: f32
                             | ((uint32_t)(TPAD >> 3) << 17)  // N
                             | ((uint32_t)(128 >> 4) << 24);  // M = 128; A, B e4m3, K-major
      bool ok = true;
      for (int it = 0; it < total; ++it) {
        const int s = it % nstage;
        if (!b200::mbar_wait_bounded(&w_full[s], (it / nstage) & 1, deadline)) { ok = false; break; }
        const int kk = 2 * it + me, buf = kk % nbuf;
        if (kk >= nbuf && !b200::mbar_wait_bounded(&a_empty[buf], ((kk / nbuf) - 1) & 1, deadline)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t st = b200::smem_u32(ring + s * STAGE);
        const uint64_t ad = sw128_desc(st + me * TC_TILE_W), bd = sw128_desc(st + TC_PAIR_W);
        const uint32_t d = tmem + (uint32_t)(buf * TPAD);
#pragma unroll
        for (int k = 0; k < 4; ++k) tc_mma_f8(d, ad + 2 * k, bd + 2 * k, idesc, k > 0 ? 1u : 0u);
        tc_commit(&a_full[buf]);
        tc_commit(&w_empty[s]);
      }
      if (!ok) atomicExch(&g_lmhead_err, 1);
      tc_commit(done_bar);                                     // every issued MMA has landed
      b200::mbar_wait_bounded(done_bar, 0, deadline + WAIT_NS);
    }
    __syncwarp();
  } else if (warp == TC_SCALE_WARP) {
    // ---------------- scale vectors: for every accumulator, c[t] = ws[block, kb] * xs[kb][t],
    // written into the accumulator's slot ahead of the MMAs (the slot is free once the epilogue
    // has released the accumulator's previous use), so that the epilogue's per-unit work is one
    // fused multiply-add per logit. The accumulator is complete (a_full) when its MMAs have
    // landed AND its vector is written. Lane j holds the weight scales of units base + j, the
    // next 32 units' already in flight.
    const float* wsp = static_cast<const float*>(p.wscale);
    auto load32 = [&](int base, float (&w)[2]) {
      const int u = base + lane;
      int pr, kb;
      wk.unit(u, pr, kb);
#pragma unroll
      for (int me = 0; me < 2; ++me) {
        const int blk = 2 * pr + me;
        w[me] = (u < total && blk < nblk) ? __ldg(wsp + (long long)blk * KB + kb) : 0.f;
      }
    };
    float wcur[2], wnext[2];
    load32(0, wcur);
    load32(32, wnext);
    bool ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(xs_bar, 0, deadline));
    for (int it = 0; it < total && ok; ++it) {
      if ((it & 31) == 0 && it > 0) {
        wcur[0] = wnext[0];
        wcur[1] = wnext[1];
        load32(it + 32, wnext);
      }
      int pr, kb;
      wk.unit(it, pr, kb);
      const float* xk = xs_s + kb * TPAD;
#pragma unroll
      for (int me = 0; me < 2; ++me) {
        const int kk = 2 * it + me, buf = kk % nbuf;
        if (kk >= nbuf) ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(&a_empty[buf], ((kk / nbuf) - 1) & 1, deadline));
        if (!ok) break;
        const float sw = __shfl_sync(0xffffffffu, wcur[me], it & 31);
        float* c = c_s + buf * TPAD;
#pragma unroll
        for (int t = lane; t < TPAD; t += 32) c[t] = sw * xk[t];
        __syncwarp();
        if (lane == 0) b200::mbar_arrive(&a_full[buf]);
      }
    }
    if (!ok && lane == 0) atomicExch(&g_lmhead_err, 1);
  } else {
    // ---------------- epilogue: group g handles block 2p + g of each pair ----------------
    // After a timed-out wait the warps carry on without touching TMEM (so every warp still
    // reaches the final barrier) and the error word reports the call.
    const int ew = warp - 2 - TC_ISSUERS;     // 0..7
    const int g = ew >> 2;
    const int qd = warp & 3;                  // TMEM lane quarter this warp may access
    const int row = 32 * qd + lane;           // row of the 128-row block held by this lane
    float* tr = reinterpret_cast<float*>(sm + p.x_off) + ew * (TC_CHUNK * 33);
#pragma unroll
    for (int i = 0; i < TPAD / TC_CHUNK; ++i) b200::rowstat_init(st[i]);
    bool ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(xs_bar, 0, deadline));
    int nsplit = 0;                           // split pairs met so far (ticket buffer parity)
    for (int it = 0; it < total;) {
      int pr, j0;
      wk.unit(it, pr, j0);
      const int blk = 2 * pr + g;
      const bool real = blk < nblk;
      float acc[TPAD];
#pragma unroll
      for (int j = 0; j < TPAD; ++j) acc[j] = 0.f;
      int j1 = j0;
      for (;; ++it) {
        int p2, kb;
        if (it >= total) break;
        wk.unit(it, p2, kb);
        if (p2 != pr) break;
        j1 = kb;
        const int kk = 2 * it + g, buf = kk % nbuf;
        if (ok) ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(&a_full[buf], (kk / nbuf) & 1, deadline));
        if (!ok) continue;
        tc_fence_after();
        const uint32_t ta = tmem + ((uint32_t)(32 * qd) << 16) + (uint32_t)(buf * TPAD);
        const float4* c4 = reinterpret_cast<const float4*>(c_s + buf * TPAD);   // ws * xs per token
#pragma unroll
        for (int h = 0; h < TPAD / 32; ++h) {
          float v[32];
          tmem_ld32(ta + 32 * h, v);
          tmem_wait_ld();
          tmem_values_after_wait(v);
#pragma unroll
          for (int j = 0; j < 32; j += 4) {
            const float4 cv = c4[(32 * h + j) >> 2];
            ffma2(acc[32 * h + j], acc[32 * h + j + 1], v[j], v[j + 1], cv.x, cv.y);
            ffma2(acc[32 * h + j + 2], acc[32 * h + j + 3], v[j + 2], v[j + 3], cv.z, cv.w);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) b200::mbar_arrive(&a_empty[buf]);
      }
      if ((j0 != 0 || j1 != wk.KBS - 1) && real) {
        // The pair is split between CTAs (contiguous ones, c_first .. c_first + nseg - 1, each
        // covering one run of its 128-K blocks). Each block's group of four warps takes a
        // ticket; the group that arrives LAST finishes the block and the others leave their
        // fp32 partials (one per warp, with a ready flag). A group therefore waits only for
        // partials whose writers hold an earlier ticket, i.e. are already running and have
        // nothing left to wait for: no CTA depends on a CTA that has not started. The block is
        // the sum of the segments' partials in segment (K) order whoever finishes it, and its
        // per-token statistics go to a slot of the pair's own (not to the finishing CTA's), so
        // every output is independent of the arrival order.
        const long long u0 = (long long)pr * wk.KBS;
        const int c_first = wk.owner(u0);
        const int nseg = wk.owner(u0 + wk.KBS - 1) - c_first + 1, me = wk.c - c_first;
        if ((ew & 3) == 0 && lane == 0)
          s_ticket[2 * g + (nsplit & 1)] = ok ? atom_add_acq_rel_gpu(p.flags + TC_TICKET_OFF + c_first * 2 + g, 1) : -1;
        group_bar(g);
        const int t = s_ticket[2 * g + (nsplit & 1)];
        ++nsplit;
        if (t < 0) continue;                // a wait of this group ran out earlier
        float4* px4 = reinterpret_cast<float4*>(p.px);
        // partial slot of segment `s`: [T/4][128 rows][4] (each warp access one contiguous 512 B)
        auto slot = [&](int s) {
          const int cc = c_first + s;
          const int which = ((int)((wk.LU * cc / wk.G) / wk.KBS) == pr) ? 0 : 1;   // CTA cc's first pair?
          return (((long long)cc * 2 + which) * 2 + g) * 4 + qd;
        };
        auto publish = [&](long long sl) {
          float4* dst = px4 + (sl >> 2) * (TPAD / 4) * 128 + row;
#pragma unroll
          for (int j = 0; j < TPAD; j += 4) dst[(j >> 2) * 128] = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
        };
        if (t < nseg - 1) {
          const long long sl = slot(me);
          publish(sl);
          __threadfence();
          __syncwarp();
          if (lane == 0) st_release_gpu(p.flags + TC_READY_OFF + sl, 1);
          continue;
        }
        // Last: sum the segments in order. Segment 0 + this one is order-free (addition
        // commutes); from the third segment on, this warp's own partial joins the others in
        // memory so that the prefix is summed first.
        if (me >= 2) publish(slot(me));
        for (int s = 0; s < nseg && ok; ++s) {
          if (s == me && me < 2) continue;
          const long long sl = slot(s);
          if (s != me) {
            // every lane polls with its own acquire load, so each lane's reads follow the publish
            bool got;
            while (!(got = __all_sync(0xffffffffu, ld_acquire_gpu(p.flags + TC_READY_OFF + sl) != 0))) {
              if (__any_sync(0xffffffffu, b200::globaltimer_ns() > deadline)) break;   // warp-uniform
            }
            if (!got) {
              ok = false;
              break;
            }
          }
          const float4* src = px4 + (sl >> 2) * (TPAD / 4) * 128 + row;
          float4 v4[TPAD / 4];
#pragma unroll
          for (int j = 0; j < TPAD / 4; ++j) v4[j] = __ldcg(src + j * 128);
          const bool first = (me >= 2) && (s == 0);
#pragma unroll
          for (int j = 0; j < TPAD / 4; ++j) {
            acc[4 * j] = first ? v4[j].x : acc[4 * j] + v4[j].x;
            acc[4 * j + 1] = first ? v4[j].y : acc[4 * j + 1] + v4[j].y;
            acc[4 * j + 2] = first ? v4[j].z : acc[4 * j + 2] + v4[j].z;
            acc[4 * j + 3] = first ? v4[j].w : acc[4 * j + 3] + v4[j].w;
          }
        }
        // the block's rows, then its per-token statistics: each warp's (lanes < 16 hold tokens
        // 16 ch + lane) into its transpose tile, merged over the group's four warps in a fixed
        // order into the pair's slot G + 2 c_first + g
        b200::RowStat bs[TPAD / TC_CHUNK];
#pragma unroll
        for (int i = 0; i < TPAD / TC_CHUNK; ++i) b200::rowstat_init(bs[i]);
        if (ok) tc_block_rows<TPAD, STATS>(p, acc, blk * 128 + 32 * qd, lane, tr, bs);
        if (STATS) {
          if (lane < TC_CHUNK) {
#pragma unroll
            for (int i = 0; i < TPAD / TC_CHUNK; ++i) {
              float* e = tr + (TC_CHUNK * i + lane) * 3;
              e[0] = bs[i].m;
              e[1] = __int_as_float(bs[i].idx);
              e[2] = bs[i].s;
            }
          }
          group_bar(g);
          if ((ew & 3) == 0) {
            const float* tg = reinterpret_cast<const float*>(sm + p.x_off) + (4 * g) * (TC_CHUNK * 33);
            for (int tk = lane; tk < p.M; tk += 32) {
              b200::RowStat r;
              b200::rowstat_init(r);
              for (int w = 0; w < 4; ++w) {
                const float* e = tg + w * (TC_CHUNK * 33) + tk * 3;
                r = b200::rowstat_merge(r, b200::RowStat{e[0], __float_as_int(e[1]), e[2]});
              }
              float* dst = p.partial + ((long long)tk * 3 * wk.G + wk.G + 2 * c_first + g) * 3;
              dst[0] = r.m;
              dst[1] = __int_as_float(r.idx);
              dst[2] = r.s;
            }
          }
          group_bar(g);                     // the tiles are free again
        }
        continue;
      }
      if (real && ok) tc_block_rows<TPAD, STATS>(p, acc, blk * 128 + 32 * qd, lane, tr, st);
    }
    if (!ok) atomicExch(&g_lmhead_err, 1);
  }
  tc_fence_before();
  __syncthreads();                          // every copy has landed and every MMA completed
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
  if (STATS) {
    // the ring is idle now: the per-warp row statistics go there
    b200::RowStat* red = reinterpret_cast<b200::RowStat*>(ring);
    if (warp > TC_SCALE_WARP) {
      const int ew = warp - 2 - TC_ISSUERS;
      for (int i = 0; i < 64; i += 32) red[ew * 64 + i + lane] = b200::RowStat{-INFINITY, 0x7fffffff, 0.f};
      __syncwarp();
      if (lane < TC_CHUNK) {
#pragma unroll
        for (int i = 0; i < TPAD / TC_CHUNK; ++i) red[ew * 64 + TC_CHUNK * i + lane] = st[i];
      }
    }
    __syncthreads();
    stats_write_partial(p, red, 64, TC_EPI_WARPS, blockIdx.x, 3 * gridDim.x);
  }
}

// ---- vocabulary-sharded combine over NVLink peer memory ----------------------------------------
// Every rank owns a buffer in memory all ranks can address (torch symmetric memory):
// [2 parities][world source ranks][M_cap][4] uint64 words. Each word carries 32 bits of data in
// its low half and a 32-bit call tag in its high half (the low-latency "tagged word" form of a
// flag): a token's row is max bits, argmax low, argmax high, logsumexp bits. Every token m has
// its own call counter k = counters[m] (equal on every rank, since all make the same calls),
// and its call k has tag (uint32)(k + 1): the token's warp stores its row, tagged, into slot
// [k & 1][rank][m] of EVERY rank's buffer (8-byte relaxed system-scope stores over NVLink,
// each single-copy atomic), then reads slot [k & 1][r][m] of its own buffer for every rank r,
// re-reading -- bounded by %globaltimer -- each word whose tag is not yet this call's, and
// combines. A word's data and tag arrive together, so no fence and no separate arrival flag
// sit between the stores and the reads: the exchange costs one NVLink crossing. Tokens are
// independent of each other, so every token's exchange runs in its own warp. Double-buffering
// by parity makes reuse safe: a rank writes token m's parity k & 1 again at call k + 2 only
// after reading every rank's call k + 1 row of m, which each rank stores after it has
// finished call k of m. A tag never matches a stale word: the slot last held tag k - 1 (or
// zero before its first use, and tags are zero only after 2^32 calls).
constexpr long long P2P_WAIT_NS = 1000000000ull;
constexpr int P2P_WORDS = 4;                // per token row: max, argmax low, argmax high, lse
constexpr int P2P_MAX_WORLD = 64;

__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Token m's exchange and combine, run by one whole warp. (mx, arg, lse) is this rank's row; `w`
// is the warp's shared scratch for the world ranks' words. The global result: the max over
// ranks, the argmax of the first rank attaining it (shards are in vocabulary order, so the first
// global index), logsumexp = max + log sum_r exp(lse_r - max) in float64; a NaN max at any rank
// (a rank whose bounded wait ran out) makes max and logsumexp NaN and the argmax -1, as in
// combine_row_stats_kernel, and so does a rank whose row did not arrive in time. Lane 0 writes the outputs (each nullable) and advances the
// token's counter. Returns false when some rank's row did not arrive within the limit.
__device__ bool p2p_token(float mx, long long arg, float lse, int m, int M_cap, char* const* peers, int rank,
                          int world, unsigned long long* counters, float* out_mx, long long* out_arg,
                          float* out_lse, unsigned long long (*w)[P2P_WORDS]) {
  const int lane = threadIdx.x & 31;
  unsigned long long k = 0;
  if (lane == 0) k = counters[m];
  k = __shfl_sync(0xffffffffu, k, 0);
  const uint32_t tag32 = (uint32_t)(k + 1);
  const unsigned long long tag = (unsigned long long)tag32 << 32;
  const int par = (int)(k & 1);
  const unsigned long long a = (unsigned long long)arg;
  const unsigned long long row[P2P_WORDS] = {tag | __float_as_uint(mx), tag | (a & 0xffffffffull), tag | (a >> 32),
                                             tag | __float_as_uint(lse)};
  for (int q = lane; q < world; q += 32) {
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(peers[q]) +
                              (((long long)par * world + rank) * M_cap + m) * P2P_WORDS;
#pragma unroll
    for (int i = 0; i < P2P_WORDS; ++i) st_relaxed_sys(dst + i, row[i]);
  }
  const unsigned long long* g = reinterpret_cast<const unsigned long long*>(peers[rank]) +
                                (long long)par * world * M_cap * P2P_WORDS;
  const uint64_t deadline = b200::globaltimer_ns() + P2P_WAIT_NS;
  bool bad = false;
  for (int r = lane; r < world; r += 32) {
    const unsigned long long* src = g + ((long long)r * M_cap + m) * P2P_WORDS;
    unsigned long long v[P2P_WORDS];
#pragma unroll
    for (int i = 0; i < P2P_WORDS; ++i) v[i] = ld_relaxed_sys(src + i);     // all four in flight
#pragma unroll
    for (int i = 0; i < P2P_WORDS; ++i) {
      uint32_t n = 0;
      while (!bad && (uint32_t)(v[i] >> 32) != tag32) {
        if ((++n & 63u) == 0 && b200::globaltimer_ns() > deadline) bad = true;
        v[i] = ld_relaxed_sys(src + i);
      }
      w[r][i] = v[i];
    }
  }
  bad = __any_sync(0xffffffffu, bad);
  __syncwarp();
  if (lane == 0) {
    double gm = 0.0;
    long long garg = 0;
    bool nan = false;
    for (int r = 0; r < world; ++r) {
      const double x = (double)__uint_as_float((uint32_t)w[r][0]);
      nan = nan || (x != x);
      if (r == 0 || x > gm) {
        gm = x;
        garg = (long long)(((w[r][2] & 0xffffffffull) << 32) | (w[r][1] & 0xffffffffull));
      }
    }
    if (nan || bad) {                       // a rank's statistics are poisoned or missing
      gm = __longlong_as_double(0x7ff8000000000000ll);
      garg = -1;
    }
    double sum = 0.0;
    for (int r = 0; r < world; ++r) sum += exp((double)__uint_as_float((uint32_t)w[r][3]) - gm);
    if (out_mx) out_mx[m] = (float)gm;
    if (out_arg) out_arg[m] = garg;
    if (out_lse) out_lse[m] = (float)(gm + log(sum));
    counters[m] = k + 1;
  }
  __syncwarp();                             // `w` is free again for the warp's next token
  return !bad;
}

// The combine alone (the statistics come from an earlier kernel), launched as a programmatic
// dependent, so the statistics are read only after the kernel that writes them has completed.
// Warp w of the grid takes tokens w, w + W, w + 2W, ... in that order on every rank, so the
// row a warp waits for is stored by the same warp of the peer after the peer's previous token,
// whose row this warp has already stored; the grid (at most P2P_MAX_CTAS CTAs) is resident at
// once, so every warp makes progress.
constexpr int P2P_MAX_CTAS = 128;
__global__ void __launch_bounds__(128) p2p_combine_kernel(const float* __restrict__ mx, const long long* __restrict__ arg,
                                                          const float* __restrict__ lse, int M, int M_cap,
                                                          char* const* __restrict__ peers, int rank, int world,
                                                          unsigned long long* __restrict__ counters,
                                                          float* __restrict__ out_mx, long long* __restrict__ out_arg,
                                                          float* __restrict__ out_lse) {
  __shared__ unsigned long long s_w[4][P2P_MAX_WORLD][P2P_WORDS];
  griddep_wait();
  const int warp = threadIdx.x >> 5;
  bool ok = true;
  for (int m = blockIdx.x * 4 + warp; m < M; m += gridDim.x * 4)      // whole warps
    ok = p2p_token(mx[m], arg[m], lse[m], m, M_cap, peers, rank, world, counters, out_mx, out_arg, out_lse,
                   s_w[warp]) && ok;
  if (!ok && (threadIdx.x & 31) == 0) atomicExch(&g_lmhead_err, 2);
}

// Final (max, first argmax, logsumexp) of token blockIdx.x from its `nslots` partials: per warp
// the max, the smallest index attaining it and sum_i s_i exp(m_i - warp max) as independent
// terms, then the eight warps merged in order (one rescaling each); every reduction in a fixed
// order. 256 threads; the programmatic dependent of the GEMM kernel.
// With g_cta > 0 (the tcgen05 path) slots [0, g_cta) are the GEMM CTAs' and slots
// g_cta + 2c + g the blocks of the split pair CTA c begins (valid only where it begins one).
__global__ void __launch_bounds__(256) stats_merge_kernel(Params p, int nslots, int g_cta) {
  __shared__ float s_m[8];
  __shared__ int s_i[8];
  __shared__ float s_s[8];
  __shared__ long long s_arg;
  __shared__ unsigned long long s_w[P2P_MAX_WORLD][P2P_WORDS];
  const int m = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_launch_dependents();              // a peer-memory combine may launch behind it
  const float* base = p.partial + (long long)m * nslots * 3;
  const int KBS = p.K / 128, nblk = p.N / 128;
  const long long LU = (long long)((nblk + 1) / 2) * KBS;
  auto valid = [&](int i) {
    if (i >= nslots) return false;
    if (g_cta <= 0 || i < g_cta) return true;
    int pair;
    const int j = i - g_cta;
    return tc_begins_split(LU, g_cta, KBS, j >> 1, pair) && 2 * pair + (j & 1) < nblk;
  };
  // which of this thread's slots hold data depends only on the launch shape: decided while
  // the GEMM still runs, so that only the loads follow the wait
  bool v[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) v[k] = valid(threadIdx.x + 256 * k);
  griddep_wait();
  // the error word travels with the partials (one round trip), not after the reductions
  const int err = (threadIdx.x == 0) ? *reinterpret_cast<volatile int*>(&g_lmhead_err) : 0;
  float pm[2], ps[2];
  int pi[2];
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    const int i = threadIdx.x + 256 * k;
    pm[k] = v[k] ? __ldcg(base + 3 * i) : -INFINITY;
    pi[k] = v[k] ? __float_as_int(__ldcg(base + 3 * i + 1)) : 0x7fffffff;
    ps[k] = v[k] ? __ldcg(base + 3 * i + 2) : 0.f;
  }
  for (int i = threadIdx.x + 512; i < nslots; i += 256) {      // more than 512 slots: fold in
    if (!valid(i)) continue;
    const float mm = __ldcg(base + 3 * i), ss = __ldcg(base + 3 * i + 2);
    const int ii = __float_as_int(__ldcg(base + 3 * i + 1));
    b200::RowStat a{pm[1], pi[1], ps[1]}, b{mm, ii, ss};
    a = b200::rowstat_merge(a, b);
    pm[1] = a.m; pi[1] = a.idx; ps[1] = a.s;
  }
  // per warp: its max, the first index at it and the sum of exp(m_i - its max), each by a fixed
  // shuffle tree; thread 0 then merges the eight warps in order (one barrier)
  float wm = fmaxf(pm[0], pm[1]);
#pragma unroll
  for (int o = 16; o; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
  int id = 0x7fffffff;
#pragma unroll
  for (int k = 0; k < 2; ++k)
    if (pm[k] == wm && ps[k] > 0.f) id = min(id, pi[k]);
#pragma unroll
  for (int o = 16; o; o >>= 1) id = min(id, __shfl_xor_sync(0xffffffffu, id, o));
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < 2; ++k)
    if (ps[k] > 0.f) sum += ps[k] * __expf(pm[k] - wm);
#pragma unroll
  for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  if (lane == 0) {
    s_m[warp] = wm;
    s_i[warp] = id;
    s_s[warp] = sum;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mx = s_m[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) mx = fmaxf(mx, s_m[w]);
    float t = 0.f;
    int best = 0x7fffffff;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      if (s_s[w] > 0.f) t += s_s[w] * __expf(s_m[w] - mx);
      if (s_m[w] == mx) best = min(best, s_i[w]);
    }
    float lse = mx + logf(t);
    long long arg = best;
    // A pipeline wait that ran out (this call or an earlier one not yet cleared with
    // b200_lmhead_error(1)) leaves some blocks unwritten: the statistics say so instead of
    // carrying a plausible value (max and logsumexp NaN, argmax -1).
    if (err != 0) {
      mx = __int_as_float(0x7fffffff);
      lse = mx;
      arg = -1;
    }
    if (p.peers == nullptr) {
      if (p.row_max) p.row_max[m] = mx;
      if (p.row_arg) p.row_arg[m] = arg;
      if (p.row_lse) p.row_lse[m] = lse;
    } else {
      s_m[0] = mx;
      s_s[0] = lse;
      s_arg = arg;
    }
  }
  if (p.peers == nullptr) return;
  // vocabulary-sharded: this token's row meets every rank's over peer memory (warp 0)
  __syncthreads();
  if (warp == 0 &&
      !p2p_token(s_m[0], s_arg, s_s[0], p.m_base + m, p.M_cap, p.peers, p.rank, p.world, p.counters,
                 p.row_max ? p.row_max - p.m_base : nullptr, p.row_arg ? p.row_arg - p.m_base : nullptr,
                 p.row_lse ? p.row_lse - p.m_base : nullptr, s_w) &&
      lane == 0)
    atomicExch(&g_lmhead_err, 2);
}

// ---- vocabulary-sharded combine of the row statistics ---------------------------------------
// Each rank's (max, argmax, logsumexp) per token is packed as three float64 (exact for the
// index), all-gathered by NCCL, and combined: global max; argmax of the first rank attaining
// it (shards are in vocabulary order, so this is the first global index); logsumexp =
// max + log sum_r exp(lse_r - max). A NaN max at any rank (its statistics poisoned by a wait
// that ran out) gives NaN max and logsumexp and argmax -1.
__global__ void pack_row_stats_kernel(const float* __restrict__ mx, const long long* __restrict__ arg,
                                      const float* __restrict__ lse, int M, double* __restrict__ out) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  out[3 * m] = (double)mx[m];
  out[3 * m + 1] = (double)arg[m];
  out[3 * m + 2] = (double)lse[m];
}

__global__ void combine_row_stats_kernel(const double* __restrict__ g, int world, int M, float* __restrict__ mx,
                                         long long* __restrict__ arg, float* __restrict__ lse) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  double gm = g[3 * m];
  int first = 0;
  bool nan = gm != gm;
  for (int r = 1; r < world; ++r) {
    const double v = g[((long long)r * M + m) * 3];
    nan = nan || (v != v);
    if (v > gm) {
      gm = v;
      first = r;
    }
  }
  if (nan) gm = __longlong_as_double(0x7ff8000000000000ll);     // poisoned at some rank
  double s = 0.0;
  for (int r = 0; r < world; ++r) s += exp(g[((long long)r * M + m) * 3 + 2] - gm);
  if (mx) mx[m] = (float)gm;
  if (arg) arg[m] = nan ? -1 : (long long)g[((long long)first * M + m) * 3 + 1];
  if (lse) lse[m] = (float)(gm + log(s));
}

// ---- read-only stream control (hcq_stream_probe, hcq_fp8skinny.hip:206-224) -----------------
__global__ void __launch_bounds__(256) stream_probe_kernel(const uint4* __restrict__ w, size_t n16,
                                                           unsigned* __restrict__ out) {
  size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  unsigned acc = 0;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    const uint4 a = __ldcs(w + i), b = __ldcs(w + i + stride), c = __ldcs(w + i + 2 * stride),
                d = __ldcs(w + i + 3 * stride);
    acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
  }
  for (; i < n16; i += stride) {
    const uint4 a = __ldcs(w + i);
    acc ^= a.x ^ a.y ^ a.z ^ a.w;
  }
  if (acc == 0xdeadbeefu) out[0] = acc;      // never taken in practice; keeps every load live
}

// ---- host side -------------------------------------------------------------------------------

// ---- per-device host state, set up on first use (a call then costs launches, not queries) ----
constexpr int HOST_MAX_DEVICES = 64;

int current_device() {
  int dev = 0;
  return (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < HOST_MAX_DEVICES) ? dev : 0;
}

int num_sms() {
  static int cached[HOST_MAX_DEVICES] = {};
  const int dev = current_device();
  if (cached[dev] <= 0) {
    int n = 0;
    cached[dev] = (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) ? n : 148;
  }
  return cached[dev];
}

// Raise a kernel's dynamic shared-memory limit to the full 227 KB once per device, so later
// launches with any plan need no attribute call. `done` is the kernel's own flag array.
int allow_full_smem(const void* kern, bool (&done)[HOST_MAX_DEVICES]) {
  const int dev = current_device();
  if (done[dev]) return 0;
  const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_CAP);
  if (e != cudaSuccess) return (int)e;
  done[dev] = true;
  return 0;
}

// Fill in the GEMV's shared-memory plan; returns the dynamic smem bytes, or -1 if it cannot fit.
// Consumer warp c takes strips c, c + NC, ... of CH = ceil(KB / kps) stages each and waits on
// a slot by the parity of the stage's round. That wait must not end on the slot's previous
// round, whose copy may still be landing (issued is not enough: two bulk copies may complete
// out of order). When nstage is a multiple of NC * CH every slot is owned by one consumer,
// whose own previous stage that round was; otherwise (p.tagged: the kernel's TAGGED
// instantiation) the consumer first waits for its stage's tag in the slot, written by the
// producer only once the previous round was consumed. The plan asks nstage >= (NC - 1) * CH
// + 1, so that the producer, issuing in order, can have every consumer's next stage in flight.
int plan(Params& p, bool is_w4, int nt8, int nc, int sz_bytes) {
  const int KB = p.K / 128;
  const int rows_x = 8 * nt8;
  p.xs_stride = (is_w4 ? 2 * p.K : p.K) + 64;
  p.xs_off = (gemv_hdr(nc) + 15) & ~15;
  p.x_off = (p.xs_off + MAXM * KB * 4 + 127) & ~127;
  const int fixed = p.x_off + rows_x * p.xs_stride;
  const int per_kb = is_w4 ? (W4_KB_BYTES + sz_bytes) : FP8_KB_BYTES;
  // The largest stages (fewest, biggest bulk copies) that still give a safe ring.
  for (int kps = min(KB, 24); kps >= 1; --kps) {
    const int ch = (KB + kps - 1) / kps;
    const int sb = (kps * per_kb + 127) & ~127;
    const int ring_off = (fixed + 127) & ~127;
    const int nstage = min(MAX_STAGES, (SMEM_CAP - ring_off) / sb);
    if (nstage >= max(2, (nc - 1) * ch + 1)) {
      p.tagged = (nstage % (nc * ch)) != 0;
      p.kps = kps;
      p.stage_bytes = sb;
      p.nstage = nstage;
      p.ring_off = ring_off;
      return ring_off + nstage * sb;
    }
  }
  return -1;
}

// cudaLaunchKernelEx, optionally as the programmatic dependent of the previous kernel in the
// stream (which must be one of ours that only produces this launch's activation).
template <typename... Exp, typename... Act>
int launch_ex(void (*kern)(Exp...), dim3 grid, dim3 block, int smem, cudaStream_t stream, bool pdl,
              Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, std::forward<Act>(args)...);
  return (int)(e != cudaSuccess ? e : cudaGetLastError());
}

template <int KIND, int NT8, bool STATS>
int launch_one(Params p, cudaStream_t stream) {
  constexpr bool IS_W4 = kind_w4(KIND);
  constexpr int NC = IS_W4 ? (NT8 == 1 ? NC_W4 : NC_W4_WIDE) : NC_FP8;
  const int smem = plan(p, IS_W4, NT8, NC, IS_W4 ? kind_sz_bytes(KIND) : 0);
  if (smem < 0) return -8;
  auto kern = p.tagged ? gemv_kernel<KIND, NT8, STATS, NC, true> : gemv_kernel<KIND, NT8, STATS, NC, false>;
  static bool smem_set[2][HOST_MAX_DEVICES] = {};
  const int e = allow_full_smem((const void*)kern, smem_set[p.tagged ? 1 : 0]);
  if (e != 0) return e;
  const int grid = min(p.N / 16, num_sms());
  const int rc = launch_ex(kern, dim3(grid), dim3(32 * (NC + 1)), smem, stream, p.pdl != 0, p);
  if (rc != 0 || !STATS) return rc;
  return launch_ex(stats_merge_kernel, dim3(p.M), dim3(256), 0, stream, true, p, grid, 0);
}

template <int KIND, bool STATS>
int launch_m(const Params& p, cudaStream_t stream) {
  return (p.M <= 8) ? launch_one<KIND, 1, STATS>(p, stream) : launch_one<KIND, 2, STATS>(p, stream);
}

// Workspace: [0,16) reserved | [16, 16+1024*64*12) per-CTA row statistics |
// [QT_OFF, +QT_CAP) swizzled activation tiles (tcgen05) | [XT_OFF, +XT_CAP) their scales |
// [QR_OFF, +QR_CAP) quantized activation rows (GEMV) | [SR_OFF, +SR_CAP) their scales |
// [PX_OFF, +PX_CAP) fp32 partial accumulators of the tcgen05 block pairs split between CTAs:
// per CTA its first and its last pair, two [T/4][128][4] blocks each | [FLAG_OFF, +FLAG_CAP)
// (inside the gap before QT_OFF) the split pairs' tickets and ready flags.
constexpr long long PART_CAP = 1024LL * 64 * 12;
constexpr long long QT_OFF = 1 << 20, QT_CAP = 1 << 20;
constexpr long long XT_OFF = 2 << 20, XT_CAP = 64 << 10;
constexpr long long QR_OFF = XT_OFF + XT_CAP, QR_CAP = 256 << 10;
constexpr long long SR_OFF = QR_OFF + QR_CAP, SR_CAP = 16 << 10;
constexpr long long PX_OFF = SR_OFF + SR_CAP, PX_CAP = 4LL * TC_MAX_GRID * 128 * 64 * 4;
constexpr long long WORKSPACE_BYTES = PX_OFF + PX_CAP;
constexpr long long FLAG_OFF = 16 + PART_CAP, FLAG_CAP = TC_FLAG_INTS * 4;
static_assert(FLAG_OFF + FLAG_CAP <= QT_OFF, "workspace regions overlap");
static_assert(3LL * TC_MAX_GRID * 64 * 12 <= PART_CAP, "statistics slots: CTAs + split pairs' blocks");

// Shared-memory plan of the tcgen05 kernel: header, row statistics, activation scales, then
// as many pair stages (two weight tiles + one activation tile) as fit. Returns the dynamic
// smem bytes or -1.
int plan_tc(Params& p, int tpad) {
  const int KB = p.K / 128;
  const int nbuf = min(TC_MAX_BUF, 512 / tpad);             // TMEM accumulators
  p.xs_off = TC_HDR;
  p.cs_off = (p.xs_off + tpad * KB * 4 + 15) & ~15;         // nbuf x [tpad] fp32 scale vectors
  p.x_off = (p.cs_off + nbuf * tpad * 4 + 15) & ~15;        // 8 warps x [16][33] fp32 tiles
  p.ring_off = (p.x_off + TC_EPI_WARPS * TC_CHUNK * 33 * 4 + 1023) & ~1023;
  const int avail = SMEM_CAP - 1024 - p.ring_off;
  const int stage = TC_PAIR_W + tpad * 128;
  const int nstage = min(TC_MAX_STAGES, avail / stage);
  if (nstage < 2) return -1;
  p.kw = 1;
  p.nstage = nstage;
  p.kps = nbuf;
  return 1024 + p.ring_off + nstage * stage;
}

// 4-D view of the strip-packed weight for the tensor-map copy: (byte 128, row 16, strip, kb),
// the strip and kb strides swapped against memory order so that one (128, 16, 16, 1) box is the
// 128x128 tiles of two consecutive 128-row blocks at one 128-K block, each landing as
// [128 rows][128 B] already in the 128-byte-swizzled order (the pack stores it that way; the
// copy itself does not swizzle). Strips beyond N read as zeros.
int encode_strip_map(CUtensorMap* m, const void* w, int N, int K) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return -12;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const int KB = K / 128;
  cuuint64_t dims[4] = {128, 16, (cuuint64_t)(N / 16), (cuuint64_t)KB};
  cuuint64_t strides[3] = {128, (cuuint64_t)KB * 2048, 2048};
  cuuint32_t box[4] = {128, 16, 16, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(w), dims, strides, box,
                            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -12;
}

// The tensor map of a weight depends only on (address, N, K): keep the last few encodings, so
// repeated calls on the same head skip the encode.
int make_strip_map(CUtensorMap* m, const void* w, int N, int K) {
  struct Entry {
    const void* w;
    int N, K;
    CUtensorMap map;
  };
  constexpr int SLOTS = 16;
  static Entry cache[SLOTS];
  static int used = 0, next = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].w == w && cache[i].N == N && cache[i].K == K) {
      *m = cache[i].map;
      return 0;
    }
  const int rc = encode_strip_map(m, w, N, K);
  if (rc != 0) return rc;
  cache[next] = Entry{w, N, K, *m};
  next = (next + 1) % SLOTS;
  used = used < SLOTS ? used + 1 : SLOTS;
  return 0;
}

template <int TPAD, bool STATS>
int launch_tc_t(Params p, const uint8_t* qx_in, const float* xs_in, cudaStream_t stream) {
  const int KB = p.K / 128;
  if ((long long)KB * TPAD * 128 > QT_CAP || (long long)TPAD * KB * 4 > XT_CAP) return -8;
  if ((reinterpret_cast<uintptr_t>(p.w) & 127) != 0) return -10;
  if (p.y != nullptr && ((p.ldy % 8) != 0 || (reinterpret_cast<uintptr_t>(p.y) & 15) != 0)) return -10;
  const int smem = plan_tc(p, TPAD);
  if (smem < 0) return -8;
  CUtensorMap wmap;
  if (make_strip_map(&wmap, p.w, p.N, p.K) != 0) return -12;
  char* base = p.ws;
  uint8_t* qt = reinterpret_cast<uint8_t*>(base + QT_OFF);
  float* xt = reinterpret_cast<float*>(base + XT_OFF);
  p.px = reinterpret_cast<float*>(base + PX_OFF);
  const long long npairs = p.N / 256 + (p.N / 128) % 2, units = npairs * KB;
  // At most one pair per SM (a vocabulary shard of up to ~38k rows): one whole pair per CTA, so
  // no pair is split and no CTA pays the split pairs' ticket, partial exchange and second
  // finish, which at that size cost more than the SMs left idle. Otherwise stream-K over
  // every SM.
  const int cap = std::min(num_sms(), TC_MAX_GRID);
  const int grid = (int)(npairs <= cap ? npairs : std::min<long long>(units, cap));
  if (units * grid >= (1LL << 31)) return -8;               // the kernels' work arithmetic is 32-bit
  p.flags = reinterpret_cast<int*>(base + FLAG_OFF);
  int rc = launch_ex(act_tiles_kernel, dim3(KB, TPAD / 8), dim3(128), 0, stream, false,
                     static_cast<const __nv_bfloat16*>(qx_in ? nullptr : p.x), qx_in, xs_in, p.M,
                     p.K, TPAD, qt, xt, p.qx_out, p.xs_out, p.flags, TC_FLAG_INTS);
  if (rc != 0) return rc;
  auto kern = fp8_tc_kernel<TPAD, STATS>;
  static bool smem_set[HOST_MAX_DEVICES] = {};
  const int e = allow_full_smem((const void*)kern, smem_set);
  if (e != 0) return e;
  p.pdl = 1;
  rc = launch_ex(kern, dim3(grid), dim3(TC_THREADS), smem, stream, true, wmap, p, qt, xt);
  if (rc != 0) return rc;
  if (!STATS) return 0;
  return launch_ex(stats_merge_kernel, dim3(p.M), dim3(256), 0, stream, true, p, 3 * grid, grid);
}

template <bool STATS>
int launch_tc(const Params& p, const uint8_t* qx_in, const float* xs_in, cudaStream_t stream) {
  return (p.M <= 32) ? launch_tc_t<32, STATS>(p, qx_in, xs_in, stream)
                     : launch_tc_t<64, STATS>(p, qx_in, xs_in, stream);
}

// Runs M in token chunks, one weight pass each. With a workspace, FP8 takes 64-token chunks:
// from TC_MIN_M tokens the tcgen05 kernel, below it the GEMV fed by act_rows_kernel (both as
// programmatic dependents of their activation kernel). Without one, 16-token GEMV chunks.
// (From 9 tokens the GEMV's warp MMAs, two n-tiles per strip, cost more than the tcgen05
// pipeline: 90 against 82 us for the 151936 x 2560 head at M = 12-16.)
constexpr int TC_MIN_M = 9;
template <int KIND>
int run_chunks(Params p, int x_elem_bytes, cudaStream_t stream) {
  const int M = p.M, KB = p.K / 128;
  const bool stats = (p.row_max || p.row_arg || p.row_lse || p.peers);
  const bool is_fp8 = (KIND == FP8_QUANT || KIND == FP8_PREQ);
  const bool have_ws = p.ws != nullptr;
  const bool tc_ok = is_fp8 && have_ws && (long long)KB * 64 * 128 <= QT_CAP;
  const int chunk = tc_ok ? 64 : MAXM;
  for (int m0 = 0; m0 < M; m0 += chunk) {
    Params q = p;
    q.M = min(chunk, M - m0);
    q.x = static_cast<const char*>(p.x) + (long long)m0 * p.K * x_elem_bytes;
    if (p.xs_in) q.xs_in = p.xs_in + (long long)m0 * KB;
    if (p.y) q.y = p.y + (long long)m0 * p.ldy;
    if (p.row_max) q.row_max = p.row_max + m0;
    if (p.row_arg) q.row_arg = p.row_arg + m0;
    if (p.row_lse) q.row_lse = p.row_lse + m0;
    if (p.qx_out) q.qx_out = p.qx_out + (long long)m0 * p.K;
    if (p.xs_out) q.xs_out = p.xs_out + (long long)m0 * KB;
    q.m_base = p.m_base + m0;
    int rc;
    if (tc_ok && q.M >= TC_MIN_M) {
      const uint8_t* qx_in = (KIND == FP8_PREQ) ? static_cast<const uint8_t*>(q.x) : nullptr;
      rc = stats ? launch_tc<true>(q, qx_in, q.xs_in, stream) : launch_tc<false>(q, qx_in, q.xs_in, stream);
    } else if (KIND == FP8_QUANT && have_ws && (long long)MAXM * p.K <= QR_CAP) {
      // quantize the rows once (the programmatic primary), then the GEMV on e4m3 rows
      char* base = p.ws;
      uint8_t* qr = q.qx_out ? q.qx_out : reinterpret_cast<uint8_t*>(base + QR_OFF);
      float* sr = q.xs_out ? q.xs_out : reinterpret_cast<float*>(base + SR_OFF);
      rc = launch_ex(act_rows_kernel, dim3(KB, (q.M + 7) / 8), dim3(128), 0, stream, false,
                     static_cast<const __nv_bfloat16*>(q.x), q.M, q.K, qr, (float*)sr);
      if (rc != 0) return rc;
      q.x = qr;
      q.xs_in = sr;
      q.qx_out = nullptr;
      q.xs_out = nullptr;
      q.pdl = 1;
      rc = stats ? launch_m<FP8_PREQ, true>(q, stream) : launch_m<FP8_PREQ, false>(q, stream);
    } else {
      rc = stats ? launch_m<KIND, true>(q, stream) : launch_m<KIND, false>(q, stream);
    }
    if (rc != 0) return rc;
  }
  return 0;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// The peer-memory combine fused into a head's statistics merge (peers == nullptr: none).
struct Combine {
  void* const* peers = nullptr;
  unsigned long long* counters = nullptr;
  int rank = 0, world = 1, M_cap = 0;
  bool valid(int M) const {
    return M <= M_cap && world >= 1 && world <= P2P_MAX_WORLD && rank >= 0 && rank < world;
  }
  void apply(Params& p) const {
    p.peers = reinterpret_cast<char* const*>(peers);
    p.counters = counters;
    p.rank = rank;
    p.world = world;
    p.M_cap = M_cap;
    p.m_base = 0;
  }
};

}  // namespace

extern "C" {

// Bytes of caller-owned workspace the fused entries need. It needs no initialisation (every
// call writes what it reads); calls that share a workspace must not overlap on the GPU.
long long b200_lmhead_workspace_bytes(void) { return WORKSPACE_BYTES; }

// Reads (and with reset != 0 clears) the device error word: 1 = a pipeline wait timed out.
// Synchronous; for tests and diagnostics only.
int b200_lmhead_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_lmhead_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(g_lmhead_err, &z, sizeof(int));
  }
  return v;
}

// Fused FP8 target lm_head: x bf16 [M, K] is quantized per token group of 128 in the prologue
// (bit-identical to b200_per_token_group_quant_fp8), then y = (qx*xs) @ (wq*ws)^T over the
// N rows of this weight, and per row m: row_max / row_arg (first index, + vocab_offset) /
// row_lse = log sum exp. Every output pointer is nullable. qx_out / xs_out (nullable) receive
// the quantized activation. wq / ws in the B200 packed layout (see the file header).
// Returns 0, -1 bad M, -2 N % 128, -3 K % 128, -8 does not fit shared memory, -9 workspace
// too small / missing when stats are asked for, -10 misaligned pointer, else a CUDA error.
static int fp8_lmhead_impl(const void* x, int M, int K, const void* wq, const float* ws, int N,
                           long long vocab_offset, void* y, long long ldy, float* row_max, long long* row_arg,
                           float* row_lse, void* qx_out, float* xs_out, void* workspace,
                           long long workspace_bytes, const Combine& cb, cudaStream_t stream) {
  if (M < 0) return -1;
  if (N <= 0 || N % 128) return -2;
  if (K <= 0 || K % 128) return -3;
  if (cb.peers != nullptr && !cb.valid(M)) return -14;
  if (M == 0) return 0;
  const bool stats = row_max || row_arg || row_lse || cb.peers != nullptr;
  if (stats && (workspace == nullptr || workspace_bytes < WORKSPACE_BYTES)) return -9;
  if (!aligned16(x) || !aligned16(wq) || (qx_out && !aligned16(qx_out))) return -10;
  Params p{};
  cb.apply(p);
  p.x = x; p.M = M; p.K = K; p.N = N; p.n_valid = N; p.vocab_offset = vocab_offset;
  p.w = static_cast<const uint8_t*>(wq); p.wscale = ws;
  p.y = static_cast<__nv_bfloat16*>(y); p.ldy = ldy > 0 ? ldy : N;
  p.row_max = row_max; p.row_arg = row_arg; p.row_lse = row_lse;
  p.qx_out = static_cast<uint8_t*>(qx_out); p.xs_out = xs_out;
  p.ws = static_cast<char*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + 16);
  return run_chunks<FP8_QUANT>(p, 2, stream);
}

int b200_fp8_lmhead(const void* x, int M, int K, const void* wq, const float* ws, int N,
                    long long vocab_offset, void* y, long long ldy, float* row_max, long long* row_arg,
                    float* row_lse, void* qx_out, float* xs_out, void* workspace,
                    long long workspace_bytes, cudaStream_t stream) {
  return fp8_lmhead_impl(x, M, K, wq, ws, N, vocab_offset, y, ldy, row_max, row_arg, row_lse, qx_out, xs_out,
                         workspace, workspace_bytes, Combine{}, stream);
}

// b200_fp8_lmhead on this rank's vocabulary shard with the combine of the per-token statistics
// over NVLink peer memory fused into its last kernel (the b200_p2p_combine_row_stats exchange
// and its `peers` / `counters` / M_cap, M <= M_cap): row_max / row_arg / row_lse receive the
// GLOBAL (max, first argmax, logsumexp) over all ranks' shards. Logits, when asked for, are
// this shard's. Same returns as b200_fp8_lmhead, plus -14 bad combine arguments.
int b200_fp8_lmhead_combined(const void* x, int M, int K, const void* wq, const float* ws, int N,
                             long long vocab_offset, void* y, long long ldy, float* row_max, long long* row_arg,
                             float* row_lse, void* qx_out, float* xs_out, void* workspace,
                             long long workspace_bytes, void* const* peers, int rank, int world,
                             unsigned long long* counters, int M_cap, cudaStream_t stream) {
  if (peers == nullptr || counters == nullptr) return -14;
  return fp8_lmhead_impl(x, M, K, wq, ws, N, vocab_offset, y, ldy, row_max, row_arg, row_lse, qx_out, xs_out,
                         workspace, workspace_bytes, Combine{peers, counters, rank, world, M_cap}, stream);
}

// fp8hip_gemm_w8a8_launch(qx, w, xs, ws, y, M, N, K, stream) -- the closed fp8hip GEMM's ABI
// (tests/k3/test_fp8sk.py:13-34): pre-quantized e4m3 qx [M, K] with fp32 xs [M, K/128],
// w / ws as above, y bf16 [M, N].
int fp8hip_gemm_w8a8_launch(void* qx, void* w, void* xs, void* ws, void* y, int M, int N, int K,
                            void* stream) {
  if (M < 0) return -1;
  if (N <= 0 || N % 128) return -2;
  if (K <= 0 || K % 128) return -3;
  if (M == 0) return 0;
  if (!aligned16(qx) || !aligned16(w)) return -10;
  Params p{};
  p.x = qx; p.xs_in = static_cast<const float*>(xs); p.M = M; p.K = K; p.N = N; p.n_valid = N;
  p.w = static_cast<const uint8_t*>(w); p.wscale = ws;
  p.y = static_cast<__nv_bfloat16*>(y); p.ldy = N;
  return run_chunks<FP8_PREQ>(p, 1, static_cast<cudaStream_t>(stream));
}

// hcq_gemm_fp8blk_nt_m16 (kernels/experimental/fp8skinny/hcq_fp8skinny.hip:168-197): same
// operands, M <= 16, the reference's precondition codes -1..-7 checked on its launch knobs
// (WV, SK, NPW); the B200 kernel then runs its own launch plan.
int hcq_gemm_fp8blk_nt_m16(void* a, void* as, void* w, void* ws, void* c, int M, int K, int N,
                           int WV, int SK, int NPW, void* stream) {
  if (M < 1 || M > MAXM) return -1;
  if (N % 128) return -2;
  if (K % 128) return -3;
  if (SK < 1 || (K / 128) % SK) return -4;
  if (WV < 1 || WV * SK * 32 > 1024) return -5;
  if (NPW != 1 && NPW != 2 && NPW != 4) return -6;
  const long long smem = ((long long)WV * NPW * SK * 256 + 16LL * (K / 128)) * 4;
  if (smem > 64 * 1024) return -7;
  const int rc = fp8hip_gemm_w8a8_launch(a, w, as, ws, c, M, N, K, stream);
  return rc == 0 ? 0 : (rc > 0 ? rc : -8);
}

int hcq_gemm_fp8blk_nt_m16_max_m(void) { return MAXM; }

// Pack this rank's per-token (max, argmax, logsumexp) as [M][3] float64 for the all-gather.
int b200_pack_row_stats(const float* row_max, const long long* row_arg, const float* row_lse, int M,
                        double* out, cudaStream_t stream) {
  if (M < 0) return -1;
  if (M == 0) return 0;
  pack_row_stats_kernel<<<(M + 127) / 128, 128, 0, stream>>>(row_max, row_arg, row_lse, M, out);
  return (int)cudaGetLastError();
}

// Combine `world` gathered [M][3] float64 blocks (rank-major, shards in vocabulary order) into
// the global per-token max, first argmax and logsumexp; each output is nullable.
int b200_combine_row_stats(const double* gathered, int world, int M, float* row_max, long long* row_arg,
                           float* row_lse, cudaStream_t stream) {
  if (M < 0 || world <= 0) return -1;
  if (M == 0) return 0;
  combine_row_stats_kernel<<<(M + 127) / 128, 128, 0, stream>>>(gathered, world, M, row_max, row_arg, row_lse);
  return (int)cudaGetLastError();
}

// Bytes of the per-rank peer-addressable buffer b200_p2p_combine_row_stats and the combined
// heads need.
long long b200_p2p_combine_bytes(int world, int M_cap) {
  return 2LL * world * M_cap * P2P_WORDS * 8;
}

// The vocabulary-sharded combine in one kernel over NVLink peer memory (see above). `peers` is
// a DEVICE array of `world` pointers, peers[q] = rank q's buffer as this GPU addresses it
// (zeroed before the first call); `counters` is this rank's DEVICE array of M_cap per-token
// call counters (zeroed before the first call, shared with the combined heads below). Every
// rank must make the same sequence of calls with the same M; a call with M == 0 does nothing.
// A peer whose row of a token does not arrive within 1 s sets the error word to 2
// (b200_lmhead_error) and that token's outputs are not meaningful.
// Returns 0, -1 bad sizes (M > M_cap, world outside 1..64, rank outside the world), else the
// launch's cudaError_t.
int b200_p2p_combine_row_stats(const float* row_max, const long long* row_arg, const float* row_lse, int M,
                               int M_cap, void* const* peers, int rank, int world,
                               unsigned long long* counters, float* out_max, long long* out_arg,
                               float* out_lse, cudaStream_t stream) {
  if (M < 0 || M > M_cap || world <= 0 || world > P2P_MAX_WORLD || rank < 0 || rank >= world) return -1;
  if (M == 0) return 0;
  return launch_ex(p2p_combine_kernel, dim3(std::min((M + 3) / 4, P2P_MAX_CTAS)), dim3(128), 0, stream, true,
                   row_max, row_arg, row_lse,
                   M, M_cap, reinterpret_cast<char* const*>(peers), rank, world, counters, out_max, out_arg,
                   out_lse);
}

// Read-only control: streams `bytes` from w with 16-byte loads over `wgs` CTAs of 256.
int hcq_stream_probe(void* w, long long bytes, int wgs, void* out, void* stream) {
  if (bytes % 16) return -1;
  if (wgs < 1) return -2;
  stream_probe_kernel<<<wgs, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(w), (size_t)(bytes / 16), static_cast<unsigned*>(out));
  return (int)cudaGetLastError();
}

// Fused W4 draft lm_head: x [M, K] (dtype 0 = bf16, converted to f16 in the kernel exactly as
// x.to(float16); 1 = f16), packed wq / wsz over N_pad rows (multiple of 16); rows >= n_valid
// are padding (written to y, excluded from the row statistics). Same outputs as
// b200_fp8_lmhead. Returns 0, -1 bad M, -2 N_pad % 16, -3 K % 128, -8 smem, -9 workspace,
// -10 alignment, -11 bad dtype.
static int w4_lmhead_impl(bool sym, const void* x, int x_dtype, int M, int K, const void* wq, const void* wsz,
                   int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                   float* row_max, long long* row_arg, float* row_lse, void* workspace,
                   long long workspace_bytes, const Combine& cb, cudaStream_t stream) {
  if (M < 0) return -1;
  if (N_pad <= 0 || N_pad % 16) return -2;
  if (K <= 0 || K % 128) return -3;
  if (x_dtype != 0 && x_dtype != 1) return -11;
  if (cb.peers != nullptr && !cb.valid(M)) return -14;
  if (M == 0) return 0;
  const bool stats = row_max || row_arg || row_lse || cb.peers != nullptr;
  if (stats && (workspace == nullptr || workspace_bytes < WORKSPACE_BYTES)) return -9;
  if (!aligned16(x) || !aligned16(wq) || !aligned16(wsz)) return -10;
  Params p{};
  cb.apply(p);
  p.x = x; p.M = M; p.K = K; p.N = N_pad;
  p.n_valid = (n_valid > 0 && n_valid < N_pad) ? n_valid : N_pad;
  p.vocab_offset = vocab_offset;
  p.w = static_cast<const uint8_t*>(wq); p.wscale = wsz;
  p.y = static_cast<__nv_bfloat16*>(y); p.ldy = ldy > 0 ? ldy : N_pad;
  p.row_max = row_max; p.row_arg = row_arg; p.row_lse = row_lse;
  p.ws = static_cast<char*>(workspace);
  p.partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + 16);
  if (sym) return x_dtype == 0 ? run_chunks<W4S_BF16>(p, 2, stream) : run_chunks<W4S_F16>(p, 2, stream);
  return x_dtype == 0 ? run_chunks<W4_BF16>(p, 2, stream) : run_chunks<W4_F16>(p, 2, stream);
}

int b200_w4_lmhead(const void* x, int x_dtype, int M, int K, const void* wq, const void* wsz,
                   int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                   float* row_max, long long* row_arg, float* row_lse, void* workspace,
                   long long workspace_bytes, cudaStream_t stream) {
  return w4_lmhead_impl(false, x, x_dtype, M, K, wq, wsz, N_pad, n_valid, vocab_offset, y, ldy, row_max,
                        row_arg, row_lse, workspace, workspace_bytes, Combine{}, stream);
}

// b200_w4_lmhead (sym = 0) or b200_w4_lmhead_sym (sym = 1) on this rank's vocabulary shard with
// the peer-memory combine of the statistics fused in, as b200_fp8_lmhead_combined: the row
// outputs are the GLOBAL (max, first argmax, logsumexp). Returns as those, plus -14.
int b200_w4_lmhead_combined(int sym, const void* x, int x_dtype, int M, int K, const void* wq, const void* wsz,
                            int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                            float* row_max, long long* row_arg, float* row_lse, void* workspace,
                            long long workspace_bytes, void* const* peers, int rank, int world,
                            unsigned long long* counters, int M_cap, cudaStream_t stream) {
  if (peers == nullptr || counters == nullptr) return -14;
  return w4_lmhead_impl(sym != 0, x, x_dtype, M, K, wq, wsz, N_pad, n_valid, vocab_offset, y, ldy, row_max,
                        row_arg, row_lse, workspace, workspace_bytes, Combine{peers, counters, rank, world, M_cap},
                        stream);
}

// The same head for the symmetric format: `wscale` holds bf16 scales [N_pad/16, K/128, 16]
// (strip, 128-K group, row in strip); a code q in 0..15 stands for (q - 8) * scale.
int b200_w4_lmhead_sym(const void* x, int x_dtype, int M, int K, const void* wq, const void* wscale,
                       int N_pad, int n_valid, long long vocab_offset, void* y, long long ldy,
                       float* row_max, long long* row_arg, float* row_lse, void* workspace,
                       long long workspace_bytes, cudaStream_t stream) {
  return w4_lmhead_impl(true, x, x_dtype, M, K, wq, wscale, N_pad, n_valid, vocab_offset, y, ldy, row_max,
                        row_arg, row_lse, workspace, workspace_bytes, Combine{}, stream);
}

static int g_w4_last_rc = 0;

// r4d_gemm_w4a16_nt_m64 (ABI bound at kernels/draft_w4_lmhead.py:118-127): f16 a [M, K],
// packed wq / wsz, bf16 c [M, N] with N = n_pad. WV/SK/MB/NPW/NT are the AMD launch knobs;
// they are accepted and ignored (the B200 kernel plans its own launch). Returns nothing,
// like the reference; the status of the last call is r4d_gemm_w4a16_nt_m64_last_error().
void r4d_gemm_w4a16_nt_m64(long a, long wq, long wsz, long c, int M, int K, int N, int WV, int SK,
                           int MB, int NPW, int NT, long stream) {
  (void)WV; (void)SK; (void)MB; (void)NPW; (void)NT;
  if (M < 1 || M > 64) {
    g_w4_last_rc = -1;
    return;
  }
  g_w4_last_rc = b200_w4_lmhead(reinterpret_cast<const void*>(a), 1, M, K,
                                reinterpret_cast<const void*>(wq), reinterpret_cast<const void*>(wsz), N,
                                N, 0, reinterpret_cast<void*>(c), N, nullptr, nullptr, nullptr, nullptr,
                                0, reinterpret_cast<cudaStream_t>(stream));
}

int r4d_gemm_w4a16_nt_m64_last_error(void) { return g_w4_last_rc; }
int r4d_gemm_w4a16_nt_m64_max_m(void) { return 64; }
int r4d_gemm_w4a16_nt_m64_group(void) { return 128; }

}  // extern "C"

// ---- FP8 lm_head with built-in scratch (allocates nothing) ----------------------------------
//
// b200_fp8_lmhead needs a caller-owned workspace. Some callers cannot hand one over: a plain C
// or ctypes binding that has no device allocator of its own, or code running where an
// allocation is not allowed (a caching allocator's hook, a memory-capped pool). For those the
// scratch lives in one file-scope device array of STATIC_SCRATCH_BYTES (about 23.4 MB per
// device, reserved when the library's device code is loaded).

namespace {

constexpr long long STATIC_SCRATCH_BYTES = WORKSPACE_BYTES;
constexpr int STATIC_SCRATCH_MAX_K = 16384;     // tcgen05 tiles and GEMV rows both fit
constexpr int STATIC_SCRATCH_MAX_DEVICES = 64;
static_assert((long long)(STATIC_SCRATCH_MAX_K / 128) * 64 * 128 <= QT_CAP, "tile region");
static_assert((long long)MAXM * STATIC_SCRATCH_MAX_K <= QR_CAP, "row region");

static __device__ __align__(256) unsigned char g_static_scratch[STATIC_SCRATCH_BYTES];
void* g_static_scratch_ptr[STATIC_SCRATCH_MAX_DEVICES] = {};
unsigned long long g_static_scratch_ctx[STATIC_SCRATCH_MAX_DEVICES] = {};
std::mutex g_static_scratch_mu;

// Unique id of the context current on this thread, 0 when there is none or the driver entry
// points are unavailable. Ids are never reused within a process, so a device reset (which
// destroys the context the array's address belongs to) shows up as a new id.
unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(fn);
  });
  CUcontext ctx = nullptr;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of this device's copy of the array. It is looked up with that device
// current (cudaGetSymbolAddress; the name itself is only a host-side stand-in) and kept
// together with the id of the context it belongs to; a call that finds another context
// current (after cudaDeviceReset, say) looks it up again. Returns 0, -13 device index beyond
// the table, or the CUDA error.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= STATIC_SCRATCH_MAX_DEVICES) return -13;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  const unsigned long long ctx = current_context_id();
  if (g_static_scratch_ptr[dev] == nullptr || ctx == 0 || ctx != g_static_scratch_ctx[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_static_scratch);   // makes the primary context current
    if (e != cudaSuccess) return (int)e;
    g_static_scratch_ptr[dev] = ptr;
    g_static_scratch_ctx[dev] = current_context_id();
  }
  *out = g_static_scratch_ptr[dev];
  return 0;
}

}  // namespace

extern "C" {

// b200_fp8_lmhead with the library's own scratch instead of a workspace argument; same
// operands, outputs and return codes, plus -9 K > STATIC_SCRATCH_MAX_K and -13 device index
// >= 64. The first call on each device (and the first after a device reset) looks the
// scratch's address up, so make it before capturing a stream. The array keeps the previous
// call's bytes: the split-pair tickets and ready flags, the only part that must start at zero,
// are zeroed by each call's first kernel, and every other byte is written before it is read.
// One array serves every stream of a device, so calls that overlap on the GPU race on it: run
// them in order.
int b200_fp8_lmhead_static_scratch(const void* x, int M, int K, const void* wq, const float* ws,
                                   int N, long long vocab_offset, void* y, long long ldy,
                                   float* row_max, long long* row_arg, float* row_lse, void* qx_out,
                                   float* xs_out, cudaStream_t stream) {
  if (M < 0) return -1;
  if (N <= 0 || N % 128) return -2;
  if (K <= 0 || K % 128) return -3;
  if (K > STATIC_SCRATCH_MAX_K) return -9;
  if (M == 0) return 0;
  void* scratch = nullptr;
  const int rc = static_scratch(&scratch);
  if (rc != 0) return rc;
  return b200_fp8_lmhead(x, M, K, wq, ws, N, vocab_offset, y, ldy, row_max, row_arg, row_lse,
                         qx_out, xs_out, scratch, STATIC_SCRATCH_BYTES, stream);
}

}  // extern "C"

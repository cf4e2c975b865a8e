// Grouped MoE GEMM with MXFP4 expert weights and FP8 activations for sm_100a: the contract of
// the closed r4d_gemm_moe_mxfp4a8_nt_b16 the reference's MoE layer calls twice per projection,
// once over the resident ("hot") experts and once over the rest ("cold")
// (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff L584-606, op at
// L454-500; semantics restated from the reference's own harness, tests/k1/moe_ref_harness.py):
//
//   for every block b < num_post_pad / 16 with e = expert_ids[b] >= 0, and every row id
//   i = sorted_ids[16 b + r] < mtk (larger ids are padding):
//     y[i, n] = tw[i] * xs[i / top_k] * sum_k qx[i / top_k, k] * W_e[n, k]
//   W_e[n, k] = e2m1(code[e, n, k]) * 2^(s[e, n, k / 32] - 127)   (E8M0 scales)
//   tw is the routed weight of the row (absent: 1). Rows not named are left untouched.
//
// Decode shapes are small (a few routed rows per expert, 1 to 16 per block), so the weight
// stream is the whole cost: each (block, 16-row strip of the expert's N outputs) is one unit
// of work, and a CTA (one per SM) takes a contiguous run of the units of the live blocks,
// whose count it reads on the device (so the launch is the same for every call and graph
// capturable). Per CTA:
//   * warp 0 lane 0 streams each unit's strip -- its nibbles for every 32-K group in one run,
//     then its E8M0 scales -- with two 1-D bulk copies into a ring of shared-memory stages,
//     and each block's activation rows (one bulk copy per live row) into the activation buffer
//     once the consumers are done with the previous block's;
//   * 4 consumer warps take the units in turn (unit q of the CTA to warp q % 4; the ring has a
//     multiple of 4 stages, so a slot's previous use always belongs to the same warp, which
//     finished it before waiting on the slot again: the barrier's phase parity is never
//     ambiguous). The strip is the A operand of mma.sync
//     m16n8k16 f16: a lane's 8 bytes per group are its A fragments for two MMAs, and each
//     e2m1 code becomes an f16 exactly (code bits shifted into place give e2m1 * 2^-14; one
//     multiply by 2^(14 - (wref - s)) folds the group's scale, exactly while the result is
//     representable in f16). The activation bytes become f16 exactly (cvt e4m3x2). fp32
//     accumulation; the epilogue multiplies by 2^(wref - 127) (exact), the token's scale and
//     the routed weight, and stores bf16.
//   * rows beyond the block's live ones skip their MMA tile when all of 8..15 are padding.
// Every wait is bounded (2 s) and reports a timeout through the error word instead of hanging.
//
// Packed layouts (B200 formats; codes and scales are the checkpoint's):
//   wq   uint8 [E][N/16 strips][K/32 groups][32 lanes][8 bytes]; lane (g, t) of a group holds
//        two 32-bit words, word h for k in [16 h, 16 h + 16): its nibble pair p (bits 4p and
//        16 + 4p) is row (g + 8 (p & 1)), k = 16 h + 2 t + 8 (p >> 1) and that k + 1.
//   ws   uint8 [E][N/16][K/32][16 rows] E8M0 exponents (the reference's ws_t, regrouped).
//   wref uint8 [E][N] per-row reference exponent, the maximum of the row's scales.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

namespace {

constexpr int MOE_BLOCK = 16;             // rows per aligned block (moe_align block size)
constexpr int MOE_GROUP = 32;             // K per E8M0 exponent
constexpr int MOE_NC = 4;                 // consumer warps
constexpr int MOE_THREADS = 32 * (1 + MOE_NC);
constexpr int MOE_MAX_STAGES = 16;
constexpr int MOE_SMEM_CAP = 227 * 1024;
constexpr int MOE_HDR = 512;              // barriers and the two buffers' row ids
constexpr uint64_t MOE_WAIT_NS = 2000000000ull;

__device__ int g_moe_err = 0;             // 1 = a pipeline wait timed out

struct MoeParams {
  const uint8_t* qx;       // e4m3 [tokens, K]; row i of the GEMM reads token i / top_k
  const float* xs;         // fp32 [tokens]
  const uint8_t* wq;
  const uint8_t* ws;
  const uint8_t* wref;
  __nv_bfloat16* y;        // [mtk, N]
  const int* sorted;       // [em]
  const int* eids;         // [em / 16]
  const int* npad;         // [1]
  const float* tw;         // [mtk] or nullptr
  int em, mtk, top_k, K, N;
  int nstage, stage_bytes, xrow, x_off, ring_off;
};

// e2m1 nibble pairs at bits (0..3, 16..19) of w -> f16x2 of e2m1 * 2^-14, exactly: the three
// magnitude bits land in f16 bits 9..11 (the f16 with that exponent/mantissa pattern is the
// e2m1 value scaled by 2^-14, subnormals included) and the sign bit in bit 15.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t w) {
  return ((w & 0x00070007u) << 9) | ((w & 0x00080008u) << 12);
}

__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(v));
  return d;
}

// f16 bits of 2^x for an integer x (subnormal below 2^-14, 0 below 2^-24, capped at 2^15).
__device__ __forceinline__ uint32_t pow2_f16_bits(int x) {
  const int e = x + 15;
  if (e >= 31) return 0x7800u;            // 2^15 (not reached: the group exponent never exceeds wref)
  if (e >= 1) return (uint32_t)e << 10;
  if (e >= -9) return 1u << (e + 9);
  return 0u;
}

// 2^x as fp32 for -149 <= x <= 127 (exact powers of two).
__device__ __forceinline__ float pow2_f32(int x) {
  if (x >= -126) return __int_as_float((x + 127) << 23);
  return __int_as_float(1 << (x + 149));
}

__global__ void __launch_bounds__(MOE_THREADS, 1) moe_mxfp4_kernel(MoeParams p) {
  extern __shared__ __align__(128) char sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + MOE_MAX_STAGES;
  uint64_t* xfull = empty + MOE_MAX_STAGES;          // the activation buffer: rows landed
  uint64_t* xempty = xfull + 1;                      // ... and released by the consumers
  int* rowid = reinterpret_cast<int*>(xempty + 1);   // [16] the block's row ids (-1: padding)
  char* ring = sm + p.ring_off;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NS = p.N / 16, NG = p.K / MOE_GROUP;
  const int wbytes = NG * 256, sbytes = NG * 16;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nstage; ++i) {
      b200::mbar_init(&full[i], 1);
      b200::mbar_init(&empty[i], 1);
    }
    b200::mbar_init(xfull, 1);
    b200::mbar_init(xempty, MOE_NC);
    b200::fence_mbar_init();
  }
  __syncthreads();
  const uint64_t deadline = b200::globaltimer_ns() + MOE_WAIT_NS;

  // the units of the live blocks, split evenly over the CTAs
  const int live = min(max(p.npad[0], 0), p.em) / MOE_BLOCK;
  const long long units = (long long)live * NS;
  const int u0 = (int)(units * blockIdx.x / gridDim.x), u1 = (int)(units * (blockIdx.x + 1) / gridDim.x);

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = b200::l2_policy_evict_first();
      bool ok = true;
      int q = 0, nb = 0, cur_b = -1;
      for (int u = u0; u < u1 && ok; ++u) {
        const int b = u / NS, s = u - b * NS;
        const int e = p.eids[b];
        if (e < 0) continue;
        if (b != cur_b) {                   // a new block: its activation rows, once released
          if (nb >= 1 && !b200::mbar_wait_bounded(xempty, (nb - 1) & 1, deadline)) {
            ok = false;
            break;
          }
          int ids[MOE_BLOCK], nlive = 0;
#pragma unroll
          for (int r = 0; r < MOE_BLOCK; ++r) {
            const int id = p.sorted[b * MOE_BLOCK + r];
            ids[r] = (id >= 0 && id < p.mtk) ? id : -1;
            rowid[r] = ids[r];
            nlive += ids[r] >= 0;
          }
          char* X = sm + p.x_off;
          b200::mbar_arrive_expect_tx(xfull, (uint32_t)(nlive * p.K));
#pragma unroll
          for (int r = 0; r < MOE_BLOCK; ++r)
            if (ids[r] >= 0)
              b200::bulk_g2s(X + r * p.xrow, p.qx + (long long)(ids[r] / p.top_k) * p.K, (uint32_t)p.K, xfull);
          cur_b = b;
          ++nb;
        }
        const int slot = q % p.nstage;
        if (q >= p.nstage && !b200::mbar_wait_bounded(&empty[slot], ((q / p.nstage) - 1) & 1, deadline)) {
          ok = false;
          break;
        }
        char* dst = ring + slot * p.stage_bytes;
        const long long strip = (long long)e * NS + s;
        b200::mbar_arrive_expect_tx(&full[slot], (uint32_t)(wbytes + sbytes));
        b200::bulk_g2s_stream(dst, p.wq + strip * wbytes, (uint32_t)wbytes, &full[slot], pol);
        b200::bulk_g2s(dst + wbytes, p.ws + strip * sbytes, (uint32_t)sbytes, &full[slot]);
        ++q;
      }
      if (!ok) atomicExch(&g_moe_err, 1);
      // never leave with copies in flight: the last use of every slot must have landed
      for (int r = max(0, q - p.nstage); r < q; ++r)
        b200::mbar_wait_bounded(&full[r % p.nstage], (r / p.nstage) & 1, deadline + MOE_WAIT_NS);
      if (nb >= 1) b200::mbar_wait_bounded(xfull, (nb - 1) & 1, deadline + MOE_WAIT_NS);
    }
    __syncwarp();
    return;
  }

  // ---------------- consumers: unit q of the CTA's sequence goes to warp q % 4 ----------------
  const int cw = warp - 1, g = lane >> 2, t = lane & 3;
  bool ok = true;
  int q = 0, nb = 0, cur_b = -1, ntile = 2;
  int rid[MOE_BLOCK / 4];                   // this lane's epilogue rows: 8 nt + 2 t + c
  for (int u = u0; u < u1 && ok; ++u) {
    const int b = u / NS, s = u - b * NS;
    const int e = p.eids[b];
    if (e < 0) continue;
    if (b != cur_b) {
      if (nb > 0) {                          // done with the previous block's activation
        __syncwarp();
        if (lane == 0) b200::mbar_arrive(xempty);
      }
      ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(xfull, nb & 1, deadline));
      if (!ok) break;
      ntile = 1;
      for (int r = 8; r < MOE_BLOCK; ++r) ntile = rowid[r] >= 0 ? 2 : ntile;
#pragma unroll
      for (int j = 0; j < MOE_BLOCK / 4; ++j) rid[j] = rowid[8 * (j >> 1) + 2 * t + (j & 1)];
      cur_b = b;
      ++nb;
    }
    const int myq = q++;
    if ((myq & (MOE_NC - 1)) != cw) continue;
    const int slot = myq % p.nstage;
    ok = __all_sync(0xffffffffu, b200::mbar_wait_bounded(&full[slot], (myq / p.nstage) & 1, deadline));
    if (!ok) break;
    const int n0 = s * 16;
    const int wr0 = p.wref[(long long)e * p.N + n0 + g], wr1 = p.wref[(long long)e * p.N + n0 + g + 8];
    const char* stg = ring + slot * p.stage_bytes;
    const uint8_t* sc = reinterpret_cast<const uint8_t*>(stg + wbytes);
    const char* X = sm + p.x_off;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll 2
    for (int gi = 0; gi < NG; ++gi) {
      const uint2 wv = *reinterpret_cast<const uint2*>(stg + gi * 256 + lane * 8);
      const uint32_t h0 = pow2_f16_bits(14 - (wr0 - (int)sc[gi * 16 + g]));
      const uint32_t h1 = pow2_f16_bits(14 - (wr1 - (int)sc[gi * 16 + g + 8]));
      const uint32_t s0 = h0 | (h0 << 16), s1 = h1 | (h1 << 16);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t wd = h ? wv.y : wv.x;
        const uint32_t a0 = hmul2_u32(e2m1x2_to_f16x2(wd), s0);
        const uint32_t a1 = hmul2_u32(e2m1x2_to_f16x2(wd >> 4), s1);
        const uint32_t a2 = hmul2_u32(e2m1x2_to_f16x2(wd >> 8), s0);
        const uint32_t a3 = hmul2_u32(e2m1x2_to_f16x2(wd >> 12), s1);
        const int k = gi * MOE_GROUP + 16 * h + 2 * t;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          if (nt >= ntile) break;
          const char* xr = X + (8 * nt + g) * p.xrow + k;
          const uint32_t b0 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(xr));
          const uint32_t b1 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(xr + 8));
          b200::mma_f16_16816(acc[nt], a0, a1, a2, a3, b0, b1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) b200::mbar_arrive(&empty[slot]);
    // epilogue: weight rows n0 + g (c0, c1) and n0 + g + 8 (c2, c3); block rows 8 nt + 2 t (+1)
    const float f0 = pow2_f32(wr0 - 127), f1 = pow2_f32(wr1 - 127);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      if (nt >= ntile) break;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int id = rid[2 * nt + c];
        if (id < 0) continue;
        float sx = p.xs[id / p.top_k];
        if (p.tw != nullptr) sx *= p.tw[id];
        __nv_bfloat16* yr = p.y + (long long)id * p.N + n0 + g;
        yr[0] = __float2bfloat16_rn(acc[nt][c] * f0 * sx);
        yr[8] = __float2bfloat16_rn(acc[nt][2 + c] * f1 * sx);
      }
    }
  }
  if (!ok) atomicExch(&g_moe_err, 1);
}

int moe_num_sms() {
  static int cached = 0;
  if (cached <= 0) {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cached = (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) ? n : 148;
  }
  return cached;
}

int g_moe_last_rc = 0;

}  // namespace

extern "C" {

// Bytes of dynamic shared memory the grouped GEMM needs for reduction depth K, or -1 when K
// does not fit (the ring needs a multiple of 4 stages, at least 4, beside the activation
// buffer of 16 rows).
int b200_moe_gemm_smem_bytes(int K) {
  if (K <= 0 || K % MOE_GROUP) return -1;
  const int xrow = K + 16;                                   // padded: conflict-free row reads
  const int x_off = MOE_HDR;
  const int ring_off = (x_off + MOE_BLOCK * xrow + 127) & ~127;
  const int stage = ((K / MOE_GROUP) * (256 + 16) + 127) & ~127;
  const int nstage = std::min(MOE_MAX_STAGES, (MOE_SMEM_CAP - ring_off) / stage) / MOE_NC * MOE_NC;
  if (nstage < MOE_NC) return -1;
  return ring_off + nstage * stage;
}

// r4d_gemm_moe_mxfp4a8_nt_b16 (the closed kernel's ABI, bound with ctypes by the reference's
// MoE layer, r4d_mxfp4_moe.py.lru.diff L454-500; argument order as tests/k1/moe_ref_harness.py
// passes it): qx e4m3 [tokens, K], x_scale fp32 [tokens], wq / ws / wref in the B200 packed
// layouts above (indexed by expert_ids: the hot call passes the resident slots' copies, the
// cold call the full tensors), c bf16 [mtk, N], sorted_ids int32 [em], expert_ids int32
// [em / 16], num_post_pad int32 [1] (read on the device), topk_weights fp32 [mtk] or 0.
// wv / sk / npw are the gfx1201 launch knobs: accepted (the Python wrapper checks them as the
// reference does) and ignored. Returns nothing, like the reference; the status of the last
// call is r4d_gemm_moe_mxfp4a8_nt_b16_last_error(): 0, -1 em < 16 / mtk < 0 / top_k < 1,
// -2 N % 16, -3 K % 32 or K too deep for shared memory, -10 misaligned pointer, else a CUDA
// error.
void r4d_gemm_moe_mxfp4a8_nt_b16(long qx, long x_scale, long wq, long ws, long wref, long c, long sorted_ids,
                                 long expert_ids, long num_post_pad, long topk_weights, int em, int mtk,
                                 int top_k, int K, int N, int wv, int sk, int npw, long stream) {
  (void)wv; (void)sk; (void)npw;
  if (em < MOE_BLOCK || mtk < 0 || top_k < 1) { g_moe_last_rc = -1; return; }
  if (N <= 0 || N % 16) { g_moe_last_rc = -2; return; }
  const int smem = b200_moe_gemm_smem_bytes(K);
  if (smem < 0) { g_moe_last_rc = -3; return; }
  if ((qx & 15) || (wq & 15) || (ws & 15)) { g_moe_last_rc = -10; return; }
  if (mtk == 0) { g_moe_last_rc = 0; return; }
  MoeParams p{};
  p.qx = reinterpret_cast<const uint8_t*>(qx);
  p.xs = reinterpret_cast<const float*>(x_scale);
  p.wq = reinterpret_cast<const uint8_t*>(wq);
  p.ws = reinterpret_cast<const uint8_t*>(ws);
  p.wref = reinterpret_cast<const uint8_t*>(wref);
  p.y = reinterpret_cast<__nv_bfloat16*>(c);
  p.sorted = reinterpret_cast<const int*>(sorted_ids);
  p.eids = reinterpret_cast<const int*>(expert_ids);
  p.npad = reinterpret_cast<const int*>(num_post_pad);
  p.tw = reinterpret_cast<const float*>(topk_weights);
  p.em = em;
  p.mtk = mtk;
  p.top_k = top_k;
  p.K = K;
  p.N = N;
  p.xrow = K + 16;
  p.x_off = MOE_HDR;
  p.ring_off = (p.x_off + MOE_BLOCK * p.xrow + 127) & ~127;
  p.stage_bytes = ((K / MOE_GROUP) * (256 + 16) + 127) & ~127;
  p.nstage = std::min(MOE_MAX_STAGES, (MOE_SMEM_CAP - p.ring_off) / p.stage_bytes) / MOE_NC * MOE_NC;
  static bool smem_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !smem_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(moe_mxfp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               MOE_SMEM_CAP);
    if (e != cudaSuccess) { g_moe_last_rc = (int)e; return; }
    smem_set[dev] = true;
  }
  moe_mxfp4_kernel<<<moe_num_sms(), MOE_THREADS, smem, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  g_moe_last_rc = (int)cudaGetLastError();
}

int r4d_gemm_moe_mxfp4a8_nt_b16_last_error(void) { return g_moe_last_rc; }
int r4d_gemm_moe_mxfp4a8_nt_b16_block(void) { return MOE_BLOCK; }
int r4d_gemm_moe_mxfp4a8_nt_b16_group(void) { return MOE_GROUP; }

// Reads (and with reset != 0 clears) the grouped GEMM's device error word: 1 = a pipeline wait
// timed out. Synchronous; for tests and diagnostics.
int b200_moe_gemm_error(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_moe_err, sizeof(int)) != cudaSuccess) return -1;
  if (reset) {
    const int z = 0;
    cudaMemcpyToSymbol(g_moe_err, &z, sizeof(int));
  }
  return v;
}

}  // extern "C"

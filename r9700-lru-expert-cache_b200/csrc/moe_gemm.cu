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
// stream is the whole cost. A 16-row strip of an expert's N outputs is one record (its codes
// for every 32-K group, then its E8M0 exponents); a unit of work is a block and a run of R
// consecutive strips of its expert (R a power of two, records of R strips <= 24 KB: 1 strip at
// K = 2560, 8 at K = 320), so that each unit is ONE bulk copy of 16-24 KB -- a bulk copy costs
// the copy engine about a quarter microsecond however small, so several KB-sized copies per
// unit would cap the stream. A CTA (one per SM) takes a contiguous run of the units of the
// live blocks, whose count it reads on the device (so the launch is the same for every call
// and graph capturable). Per CTA:
//   * warp 0 lane 0 streams each unit's records into a ring of shared-memory stages, and each
//     block's activation rows (one bulk copy per live row) into the activation buffer once the
//     consumers are done with the previous block's -- meanwhile the new block's weights keep
//     streaming, so a block boundary does not drain the ring;
//   * 8 consumer warps take the units in turn (unit q of the CTA to warp q % 8; the ring has a
//     multiple of 8 stages, so a slot's previous use always belongs to the same warp, which
//     finished it before waiting on the slot again: the barrier's phase parity is never
//     ambiguous). The strip is the A operand of mma.sync m16n8k16 f16: each byte of a lane's 8
//     per group is one A register's two codes, which cvt.rn.f16x2.e2m1x2 turns into the two
//     e2m1 values exactly; the activation bytes become f16 exactly too (cvt e4m3x2). Each group's
//     two MMAs start from zero (32 products, fp32), and the group's sum is scaled by its
//     exponent 2^(s - 127) in fp32 (exact) into the row's total -- no f16 range limit on the
//     exponents. The epilogue multiplies by the token's scale and the routed weight and stores
//     bf16.
//   * rows beyond the block's live ones skip their MMA tile when all of 8..15 are padding.
// Every wait is bounded (2 s) and reports a timeout through the error word instead of hanging.
//
// Packed layouts (B200 formats; codes and scales are the checkpoint's):
//   wq   uint8 [E][N/16 strips][272 K/32]: per strip the codes [K/32 groups][32 lanes][8 bytes],
//        byte 4 h + r of lane (g, t) holding A register r of k-half h: row g + 8 (r & 1),
//        k = 16 h + 2 t + 8 (r >> 1) in its low nibble and k + 1 in its high nibble; then the
//        E8M0 exponents [16 rows][K/32].
//   ws, wref: the checkpoint's exponents [E, N, K/32] and their per-row maximum [E, N], part
//        of the reference's argument list; this kernel reads both from wq's records.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <algorithm>

#include "common.cuh"

extern "C" int b200_moe_gemm_smem_bytes(int K);

namespace {

constexpr int MOE_BLOCK = 16;             // rows per aligned block (moe_align block size)
constexpr int MOE_GROUP = 32;             // K per E8M0 exponent
constexpr int MOE_NC = 16;                // consumer warps
constexpr int MOE_OCT = 8;                // ... in teams (team_plan); the ring is a multiple of 8
constexpr int MOE_THREADS = 32 * (1 + MOE_NC);
constexpr int MOE_MAX_STAGES = 32;
constexpr int MOE_SMEM_CAP = 227 * 1024;
constexpr int MOE_HDR = 640;              // barriers (66 x 8 B) and the block's row ids (64 B)
constexpr int MOE_XCH = MOE_NC * 8 * 32 * 4;    // 8 partial sums per lane of each consumer warp
constexpr uint64_t MOE_WAIT_NS = 2000000000ull;

__device__ int g_moe_err = 0;             // 1 = a pipeline wait timed out

// One expert set's call: its weights and its aligned blocks. A launch takes one set (the
// reference's per-call entry) or two (the hot and the cold call of a projection at once).
struct MoeSet {
  const uint8_t* wq;
  const int* sorted;       // [em]
  const int* eids;         // [em / 16]
  const int* npad;         // [1]
  int em;
};

struct MoeParams {
  const uint8_t* qx;       // e4m3 [tokens, K]; row i of the GEMM reads token i / top_k
  const float* xs;         // fp32 [tokens]
  __nv_bfloat16* y;        // [mtk, N]
  const float* tw;         // [mtk] or nullptr
  MoeSet set[2];
  int nsets;
  int mtk, top_k, K, N;
  int nstage, stage_bytes, xrow, x_off, ring_off, run;   // run = R strips per unit
  int xch_off;                                            // the teams' exchange buffers
};

// Shared-memory plan for reduction depth K: a 16-row activation buffer (rows padded by 16 B:
// conflict-free fragment reads), then a ring of stages of R strip records, R the largest power
// of two with R records <= 24 KB, the stage count a multiple of the consumer warps.
struct MoePlan {
  int xrow, x_off, ring_off, run, stage_bytes, nstage, smem;
};

inline MoePlan moe_plan(int K) {
  MoePlan m{};
  const int rec = (K / MOE_GROUP) * 272;
  m.xrow = K + 16;
  m.x_off = MOE_HDR;
  m.ring_off = (m.x_off + MOE_BLOCK * m.xrow + 127) & ~127;
  m.run = 1;
  while (2 * m.run * rec <= 24 * 1024) m.run *= 2;
  m.stage_bytes = (m.run * rec + 127) & ~127;
  const int xch = MOE_XCH;
  m.nstage = std::min(MOE_MAX_STAGES, (MOE_SMEM_CAP - m.ring_off - xch) / m.stage_bytes) / MOE_OCT * MOE_OCT;
  m.smem = m.ring_off + m.nstage * m.stage_bytes + xch;
  return m;
}

// The four bytes of w, each two e2m1 codes (low nibble first), -> four f16x2, exactly.
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t& d0, uint32_t& d1, uint32_t& d2,
                                                uint32_t& d3) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\tcvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(d0), "=r"(d1), "=r"(d2), "=r"(d3) : "r"(w));
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t d;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(v));
  return d;
}

// Consumer teams for R strips per unit: a strip of 2 x 32 K (R < 8) is shared by two warps
// (wps = 2), and a team holds R such pairs, at least one; with R >= 8 every warp takes whole
// strips (wps = 1) in teams of 8 (16 for R >= 16). TS warps per team, NT = 16 / TS teams (a
// divisor of the ring's stage count, which is a multiple of 8).
// With few units per CTA (decode at a token or two: up to 4), the split runs 8 ways (teams of
// 8, wps = 8 / R) so that a unit's groups spread over more warps.
__host__ __device__ __forceinline__ void team_plan(int run, int upc, int& TS, int& NT, int& wps) {
  if (run < MOE_OCT && upc <= 4) {
    wps = MOE_OCT / run;
    TS = MOE_OCT;
  } else {
    wps = run < MOE_OCT ? 2 : 1;
    TS = run < MOE_OCT ? 2 * run : (run >= 2 * MOE_OCT ? MOE_NC : MOE_OCT);
  }
  NT = MOE_NC / TS;
}

// True on all TS warps of consumer team tm iff v is true on every lane of all of them: the
// team's warps leave their loop together, so none is left alone at a team barrier (ids 1..8).
__device__ __forceinline__ bool team_all(int tm, int TS, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.and.pred p, %2, %3, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(1 + tm), "r"(32 * TS)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void team_sync(int tm, int TS) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + tm), "r"(32 * TS) : "memory");
}

// One 16-row strip against the block's NT x 8 activation rows, groups [g0, g1): per 32-K group, the
// lane's 8 code bytes -> 8 f16x2 A registers, two MMAs from zero, and the group's sums scaled
// by 2^(s - 127) (fp32 bits s << 23; E8M0 0 gives 0) into tot. tot[nt][0..1]: row g,
// tot[nt][2..3]: row g + 8, block rows 8 nt + 2 t and + 1.
template <int NT>
__device__ __forceinline__ void strip_dot(const char* stg, const char* X, int xrow, int NG, int g0, int g1,
                                          int lane, float (&tot)[2][4]) {
  const int g = lane >> 2, t = lane & 3;
  const uint8_t* sc0 = reinterpret_cast<const uint8_t*>(stg + NG * 256) + g * NG;
  const uint8_t* sc1 = sc0 + 8 * NG;
  const char* xb = X + g * xrow + 2 * t;
#pragma unroll 2
  for (int gi = g0; gi < g1; ++gi) {
    const uint2 wv = *reinterpret_cast<const uint2*>(stg + gi * 256 + lane * 8);
    const float m0 = __uint_as_float((uint32_t)sc0[gi] << 23), m1 = __uint_as_float((uint32_t)sc1[gi] << 23);
    uint32_t a[2][4];
    e2m1x8_to_f16x2(wv.x, a[0][0], a[0][1], a[0][2], a[0][3]);
    e2m1x8_to_f16x2(wv.y, a[1][0], a[1][1], a[1][2], a[1][3]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const char* xr = xb + 8 * nt * xrow + gi * MOE_GROUP;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t b0 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(xr + 16 * h));
        const uint32_t b1 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(xr + 16 * h + 8));
        b200::mma_f16_16816(c, a[h][0], a[h][1], a[h][2], a[h][3], b0, b1);
      }
      tot[nt][0] = fmaf(m0, c[0], tot[nt][0]);
      tot[nt][1] = fmaf(m0, c[1], tot[nt][1]);
      tot[nt][2] = fmaf(m1, c[2], tot[nt][2]);
      tot[nt][3] = fmaf(m1, c[3], tot[nt][3]);
    }
  }
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
  const int NS = p.N / 16, NG = p.K / MOE_GROUP, rec = NG * 272;
  const int NR = (NS + p.run - 1) / p.run;           // runs (units) per block

  // the units of the live blocks of both sets (set 0's blocks first), split evenly over the
  // CTAs; global block gb < live0 is set 0's block gb, else set 1's block gb - live0
  const int live0 = min(max(p.set[0].npad[0], 0), p.set[0].em) / MOE_BLOCK;
  const int live1 = p.nsets > 1 ? min(max(p.set[1].npad[0], 0), p.set[1].em) / MOE_BLOCK : 0;
  const long long units = (long long)(live0 + live1) * NR;
  const int u0 = (int)(units * blockIdx.x / gridDim.x), u1 = (int)(units * (blockIdx.x + 1) / gridDim.x);
  const int upc = (int)((units + gridDim.x - 1) / gridDim.x);
  auto block_set = [&](int gb, int& lb) -> const MoeSet& {
    lb = gb < live0 ? gb : gb - live0;
    return p.set[gb < live0 ? 0 : 1];
  };

  if (threadIdx.x == 0) {
    int ts, nt, wps0;
    team_plan(p.run, upc, ts, nt, wps0);
    for (int i = 0; i < p.nstage; ++i) {
      b200::mbar_init(&full[i], 1);
      b200::mbar_init(&empty[i], ts);       // every warp of the unit's team
    }
    b200::mbar_init(xfull, 1);
    b200::mbar_init(xempty, MOE_NC);
    b200::fence_mbar_init();
  }
  __syncthreads();
  const uint64_t deadline = b200::globaltimer_ns() + MOE_WAIT_NS;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      const uint64_t pol = b200::l2_policy_evict_first();
      bool ok = true;
      int q = 0, nb = 0, pend = -1, b = u0 / NR, s = u0 - b * NR, e = -1, cur_b = -1;
      const uint8_t* wsrc = nullptr;          // the current block's set's weights
      // block blk's row ids and activation rows into the buffer (its previous user released it)
      auto load_x = [&](int blk) {
        int ids[MOE_BLOCK], nlive = 0, lb;
        const MoeSet& bs = block_set(blk, lb);
#pragma unroll
        for (int r = 0; r < MOE_BLOCK; ++r) {
          const int id = bs.sorted[lb * MOE_BLOCK + r];
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
        ++nb;
      };
      // A new block's weights stream on while the consumers finish the previous block; its
      // activation rows go as soon as they release the buffer (checked inside every slot wait,
      // so the producer never waits on a slot whose consumer waits for those rows).
      auto service = [&]() {
        if (pend >= 0 && b200::mbar_test_wait(xempty, (nb - 1) & 1)) {
          load_x(pend);
          pend = -1;
        }
      };
      for (int u = u0; u < u1; ++u, ++s) {
        if (s == NR) {
          s = 0;
          ++b;
        }
        if (b != cur_b) {
          cur_b = b;
          int lb;
          const MoeSet& bs = block_set(b, lb);
          e = bs.eids[lb];
          wsrc = bs.wq;
          if (e < 0) continue;
          if (pend >= 0) {                  // every unit before it is issued: this wait ends
            if (!b200::mbar_wait_bounded(xempty, (nb - 1) & 1, deadline)) {
              ok = false;
              break;
            }
            load_x(pend);
            pend = -1;
          }
          if (nb == 0) {
            load_x(b);
          } else {
            pend = b;
            service();
          }
        }
        if (e < 0) continue;
        const int slot = q % p.nstage;
        if (q >= p.nstage) {
          const uint32_t par = ((q / p.nstage) - 1) & 1;
          uint32_t n = 0;
          bool got;
          while (!(got = b200::mbar_try_wait(&empty[slot], par))) {
            service();
            if ((++n & 15u) == 0 && b200::globaltimer_ns() > deadline) break;
          }
          if (!got) {
            ok = false;
            break;
          }
        }
        char* dst = ring + slot * p.stage_bytes;
        const int s0 = s * p.run, ns = min(p.run, NS - s0);
        const uint32_t bytes = (uint32_t)(ns * rec);
        b200::mbar_arrive_expect_tx(&full[slot], bytes);
        b200::bulk_g2s_stream(dst, wsrc + ((long long)e * NS + s0) * rec, bytes, &full[slot], pol);
        ++q;
      }
      if (ok && pend >= 0) {
        if (b200::mbar_wait_bounded(xempty, (nb - 1) & 1, deadline))
          load_x(pend);
        else
          ok = false;
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

  // ---- consumers: teams of TS warps (team_plan); unit q of the CTA's sequence goes to team
  // q % NT. Within a unit the team's warps split the work: with wps = 1 each warp takes whole
  // strips; with wps = 2 two warps share a strip, each taking half of its 32-K groups, and
  // their partial sums meet in shared memory, where each of the two reduces and stores half of
  // the values. (Few large strips per unit: small teams, so that more units are in flight; many
  // small strips: a strip per warp and no reduction.)
  int TS, NT, wps;
  team_plan(p.run, upc, TS, NT, wps);
  const int cw = warp - 1, tm = cw / TS, wi = cw - tm * TS, g = lane >> 2, t = lane & 3;
  float* part = reinterpret_cast<float*>(sm + p.xch_off) + tm * TS * 256;   // [TS warps][8 values][32]
  const int sj = wi / wps, sp = wi - sj * wps;             // this warp's strip in the unit, its part
  bool ok = true;
  int q = 0, nb = 0, ntile = 2, b = u0 / NR, s = u0 - b * NR, e = -1, cur_b = -1;
  int rid[MOE_BLOCK / 4];                   // this lane's epilogue rows: 8 nt + 2 t + c
  float rs = 0.f;                           // lane r < 16: block row r's token scale x routed weight
  for (int u = u0; u < u1; ++u, ++s) {
    if (s == NR) {
      s = 0;
      ++b;
    }
    if (b != cur_b) {
      cur_b = b;
      int lb;
      e = block_set(b, lb).eids[lb];
      if (e < 0) continue;
      if (nb > 0) {                          // done with the previous block's activation
        __syncwarp();
        if (lane == 0) b200::mbar_arrive(xempty);
      }
      ok = team_all(tm, TS, b200::mbar_wait_bounded(xfull, nb & 1, deadline));
      if (!ok) break;
      ntile = 1;
      for (int r = 8; r < MOE_BLOCK; ++r) ntile = rowid[r] >= 0 ? 2 : ntile;
#pragma unroll
      for (int j = 0; j < MOE_BLOCK / 4; ++j) rid[j] = rowid[8 * (j >> 1) + 2 * t + (j & 1)];
      rs = 0.f;
      const int my = rowid[lane & 15];
      if (lane < MOE_BLOCK && my >= 0) {
        rs = p.xs[my / p.top_k];
        if (p.tw != nullptr) rs *= p.tw[my];
      }
      ++nb;
    }
    if (e < 0) continue;
    const int myq = q++;
    if (myq % NT != tm) continue;
    const int slot = myq % p.nstage;
    ok = team_all(tm, TS, b200::mbar_wait_bounded(&full[slot], (myq / p.nstage) & 1, deadline));
    if (!ok) break;
    const int s0 = s * p.run, ns = min(p.run, NS - s0);
    float sx[2][2];                          // block rows 8 nt + 2 t + c
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int c = 0; c < 2; ++c) sx[nt][c] = __shfl_sync(0xffffffffu, rs, 8 * nt + 2 * t + c);
    if (wps == 1) {
      // whole strips per warp: compute, then store straight from the registers
      for (int j = wi; j < ns; j += TS) {
        const char* stg = ring + slot * p.stage_bytes + j * rec;
        float tot[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        if (ntile == 1)
          strip_dot<1>(stg, sm + p.x_off, p.xrow, NG, 0, NG, lane, tot);
        else
          strip_dot<2>(stg, sm + p.x_off, p.xrow, NG, 0, NG, lane, tot);
        const int n0 = (s0 + j) * 16;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          if (nt >= ntile) break;
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int id = rid[2 * nt + c];
            if (id < 0) continue;
            __nv_bfloat16* yr = p.y + (long long)id * p.N + n0 + g;
            yr[0] = __float2bfloat16_rn(tot[nt][c] * sx[nt][c]);
            yr[8] = __float2bfloat16_rn(tot[nt][2 + c] * sx[nt][c]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) b200::mbar_arrive(&empty[slot]);
    } else {
      // wps warps per strip: each its share of the groups; partials through shared memory
      float tot[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      if (sj < ns) {
        const char* stg = ring + slot * p.stage_bytes + sj * rec;
        const int ga = NG * sp / wps, gb = NG * (sp + 1) / wps;
        if (ntile == 1)
          strip_dot<1>(stg, sm + p.x_off, p.xrow, NG, ga, gb, lane, tot);
        else
          strip_dot<2>(stg, sm + p.x_off, p.xrow, NG, ga, gb, lane, tot);
      }
      __syncwarp();
      if (lane == 0) b200::mbar_arrive(&empty[slot]);
#pragma unroll
      for (int v = 0; v < 8; ++v) part[(wi * 8 + v) * 32 + lane] = tot[v >> 2][v & 3];
      team_sync(tm, TS);
      if (sj < ns) {
        const int n0 = (s0 + sj) * 16;
        for (int v = sp; v < 4 * ntile; v += wps) {        // value v: tile nt = v / 4, c = v % 4
          float acc = 0.f;
          for (int w = 0; w < wps; ++w) acc += part[((sj * wps + w) * 8 + v) * 32 + lane];
          const int nt = v >> 2, c = v & 3;
          // (selects, not indexing: the arrays stay in registers)
          const int id = nt ? ((c & 1) ? rid[3] : rid[2]) : ((c & 1) ? rid[1] : rid[0]);
          const float f = nt ? ((c & 1) ? sx[1][1] : sx[1][0]) : ((c & 1) ? sx[0][1] : sx[0][0]);
          if (id >= 0)
            p.y[(long long)id * p.N + n0 + g + 8 * (c >> 1)] = __float2bfloat16_rn(acc * f);
        }
      }
      team_sync(tm, TS);                     // the partials are read before the next unit's
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

// Checks, plan and launch for one or two expert sets; 0, -1 em < 16 / mtk < 0 / top_k < 1,
// -2 N % 16, -3 K % 32 or K too deep for shared memory, -10 misaligned qx / weights, else a
// CUDA error.
int moe_launch(const void* qx, const float* x_scale, void* c, const float* tw, const MoeSet* sets, int nsets,
               int mtk, int top_k, int K, int N, cudaStream_t stream) {
  for (int i = 0; i < nsets; ++i)
    if (sets[i].em < MOE_BLOCK) return -1;
  if (mtk < 0 || top_k < 1) return -1;
  if (N <= 0 || N % 16) return -2;
  const int smem = b200_moe_gemm_smem_bytes(K);
  if (smem < 0) return -3;
  if ((reinterpret_cast<uintptr_t>(qx) & 15) || (reinterpret_cast<uintptr_t>(sets[0].wq) & 15)) return -10;
  if (mtk == 0) return 0;
  MoeParams p{};
  p.qx = static_cast<const uint8_t*>(qx);
  p.xs = x_scale;
  p.y = static_cast<__nv_bfloat16*>(c);
  p.tw = tw;
  for (int i = 0; i < nsets; ++i) p.set[i] = sets[i];
  p.nsets = nsets;
  p.mtk = mtk;
  p.top_k = top_k;
  p.K = K;
  p.N = N;
  const MoePlan m = moe_plan(K);
  p.xrow = m.xrow;
  p.x_off = m.x_off;
  p.ring_off = m.ring_off;
  p.run = m.run;
  p.stage_bytes = m.stage_bytes;
  p.nstage = m.nstage;
  p.xch_off = m.ring_off + m.nstage * m.stage_bytes;
  static bool smem_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !smem_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(moe_mxfp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               MOE_SMEM_CAP);
    if (e != cudaSuccess) return (int)e;
    smem_set[dev] = true;
  }
  moe_mxfp4_kernel<<<moe_num_sms(), MOE_THREADS, smem, stream>>>(p);
  return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

// Bytes of dynamic shared memory the grouped GEMM needs for reduction depth K, or -1 when K
// does not fit (the ring needs at least one stage per consumer warp beside the activation
// buffer of 16 rows).
int b200_moe_gemm_smem_bytes(int K) {
  if (K <= 0 || K % MOE_GROUP || K > 32768) return -1;
  const MoePlan m = moe_plan(K);
  return m.nstage < MOE_OCT ? -1 : m.smem;
}

// r4d_gemm_moe_mxfp4a8_nt_b16 (the closed kernel's ABI, bound with ctypes by the reference's
// MoE layer, r4d_mxfp4_moe.py.lru.diff L454-500; argument order as tests/k1/moe_ref_harness.py
// passes it): qx e4m3 [tokens, K], x_scale fp32 [tokens], wq in the B200 packed layout above
// (indexed by expert_ids: the hot call passes the resident slots' copies, the cold call the
// full tensors; ws and wref are accepted and not read), c bf16 [mtk, N], sorted_ids int32 [em], expert_ids int32
// [em / 16], num_post_pad int32 [1] (read on the device), topk_weights fp32 [mtk] or 0.
// wv / sk / npw are the gfx1201 launch knobs: accepted (the Python wrapper checks them as the
// reference does) and ignored. Returns nothing, like the reference; the status of the last
// call is r4d_gemm_moe_mxfp4a8_nt_b16_last_error(): 0, -1 em < 16 / mtk < 0 / top_k < 1,
// -2 N % 16, -3 K % 32 or K too deep for shared memory, -10 misaligned qx / wq, else a CUDA
// error.
void r4d_gemm_moe_mxfp4a8_nt_b16(long qx, long x_scale, long wq, long ws, long wref, long c, long sorted_ids,
                                 long expert_ids, long num_post_pad, long topk_weights, int em, int mtk,
                                 int top_k, int K, int N, int wv, int sk, int npw, long stream) {
  (void)ws; (void)wref; (void)wv; (void)sk; (void)npw;
  MoeSet one{reinterpret_cast<const uint8_t*>(wq), reinterpret_cast<const int*>(sorted_ids),
             reinterpret_cast<const int*>(expert_ids), reinterpret_cast<const int*>(num_post_pad), em};
  g_moe_last_rc = moe_launch(reinterpret_cast<const void*>(qx), reinterpret_cast<const float*>(x_scale),
                             reinterpret_cast<void*>(c), reinterpret_cast<const float*>(topk_weights), &one, 1,
                             mtk, top_k, K, N, reinterpret_cast<cudaStream_t>(stream));
}

// The projection's hot and cold calls in one launch (see include/b200_moe_gemm.h).
int b200_moe_gemm_hot_cold(const void* qx, const float* x_scale, const void* wq_hot, const void* wq_cold, void* c,
                           const int* sorted_hot, const int* eids_hot, const int* npad_hot, int em_hot,
                           const int* sorted_cold, const int* eids_cold, const int* npad_cold, int em_cold,
                           const float* topk_weights, int mtk, int top_k, int K, int N, cudaStream_t stream) {
  if ((reinterpret_cast<uintptr_t>(wq_cold) & 15)) return -10;
  MoeSet two[2] = {{static_cast<const uint8_t*>(wq_hot), sorted_hot, eids_hot, npad_hot, em_hot},
                   {static_cast<const uint8_t*>(wq_cold), sorted_cold, eids_cold, npad_cold, em_cold}};
  return moe_launch(qx, x_scale, c, topk_weights, two, 2, mtk, top_k, K, N, stream);
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

// Device-side LRU expert-slot cache for B200 (sm_100a): librlu.so.
//
// Drop-in for the three entry points of kernels/lru/r4d_lru.hip (r4d_lru_manage,
// r4d_lru_fused, r4d_lru_gather: same names, argument order, return codes). One CTA per
// MoE layer runs the whole cache update; nothing here allocates, syncs with the host or
// uses an order-dependent atomic on the state, so a captured CUDA graph keeps adapting and
// replicas that see the same routing hold identical caches.
//
// What a call computes (the reference semantics, r4d_lru.hip:187-269):
//   step += 1; mark the experts routed this step (ids outside [0, E) ignored);
//   more than max_distinct distinct experts -> read-through, nothing else changes;
//   routed + resident -> the slot's stamp becomes the new step;
//   routed + missing  -> the first max_inserts misses in ascending expert id each take the
//   evictable slot with the next smallest key (stamp << 20 | slot), evictable meaning the
//   slot's expert is not routed this step; table / map_cold / slot_expert / slot_stamp and
//   the (expert, slot) miss list are rewritten, n_miss = victims installed.
//
// How B200 does it:
//   * 512 threads; the state of one layer (slot -> expert, stamps, keys, expert flags and,
//     for E <= 4096, the expert -> slot table) is mirrored in shared memory on entry with
//     every global load issued up front, so the call pays about one global latency.
//   * counts and the expert-id-ordered miss enumeration are warp shuffles plus one
//     shared-memory exchange of 16 warp totals (one barrier per block scan).
//   * victims: every evictable slot ranks its key against the shared key array in one
//     pass (the reference's batched branch, r4d_lru.hip:155-172); a key is unique, so rank
//     r < nins names the r-th victim. That is the serial argmin loop's answer by the
//     argument at r4d_lru.hip:82-93, for every nins.
//   * the fused kernel adds both moe_align_block_size outputs from the rewritten table.
//     Placement inside a bucket is a stable counting sort (ascending token index) for
//     EVERY mk: warp match_any gives the in-warp rank, warps advance the bucket cursors in
//     order. That is the reference's order for mk <= 256 and a valid instance of its
//     atomic-cursor order above.
//   * guards: table entries >= S and slot_expert entries >= E (undefined in the reference)
//     are skipped; writes past L / NB are dropped.
#include <cuda_runtime.h>
#include <utility>
#include <stdint.h>

#include "common.cuh"

namespace {

constexpr int NT = 512;
constexpr int NW = NT / 32;
constexpr int MAXS = 1024;                // slots mirrored in shared memory (r4d_lru.hip:76)
constexpr int MAXINS = 1024;              // victim table depth (r4d_lru.hip:77)
constexpr int MAXE_FUSED = 1024;          // r4d_lru.hip:328
constexpr int TAB_SMEM_MAX = 4096;        // expert table mirrored in smem up to this E
constexpr int MAXE_MANAGE = 65536;        // expert flags live in smem (E bytes)
constexpr int SLOT_BITS = 20;             // r4d_lru.hip:29
constexpr int SLOT_MASK = (1 << SLOT_BITS) - 1;
constexpr long long KEY_MAX = 0x7fffffffffffffffLL;
constexpr unsigned KEY32_MAX = 0xffffffffu;
constexpr int AGE_BITS = 21;              // 32-bit keys: (2^21 - 1 - age) << 11 | slot
constexpr int IDS_REG = 4;                // topk ids kept in registers: mk <= IDS_REG * NT
constexpr int SEL_MAX = 16;               // warp-selection victim path: nins <= SEL_MAX (measured: its
                                          // nins serial rounds beat ranking every key up to ~16)
constexpr int SMALL_MK = 128;             // direct-ranking align path: mk <= SMALL_MK (measured at
                                          // mk = 200: the block-barrier placement is 0.4 us faster)

// Shared-memory carve-up (bytes), all offsets 16-byte aligned.
struct Smem {
  int off_red, off_flags, off_tab, off_se, off_st, off_k64, off_k32, off_vic, off_missE, off_cand;
  int off_cnt_h, off_cum_h, off_cnt_c, off_cum_c, off_key, off_tc, total;
};

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

__host__ __device__ inline Smem smem_layout(int E, int S, bool tab_smem, bool fused) {
  Smem L;
  const int S4 = (S + 3) & ~3;
  int o = 0;
  L.off_red = o;   o += align16(8 * NW * (int)sizeof(int));
  L.off_flags = o; o += align16(E);
  L.off_tab = o;   o += tab_smem ? align16(E * 4) : 0;
  L.off_se = o;    o += align16(S * 4);
  L.off_st = o;    o += align16(S * 8);
  L.off_k64 = o;   o += align16(S4 * 8);
  L.off_k32 = o;   o += align16(S4 * 4);
  L.off_vic = o;   o += align16(MAXINS * 4);
  L.off_missE = o; o += align16(MAXINS * 4);
  L.off_cand = o;  o += align16(NW * SEL_MAX * 4);
  if (fused) {
    L.off_cnt_h = o; o += align16(S * 4);
    L.off_cum_h = o; o += align16(S * 4);
    L.off_cnt_c = o; o += align16(E * 4);
    L.off_cum_c = o; o += align16(E * 4);
    L.off_key = o;   o += align16(SMALL_MK * 4);
    L.off_tc = o;    o += align16(SMALL_MK * 4);
  } else {
    L.off_cnt_h = L.off_cum_h = L.off_cnt_c = L.off_cum_c = L.off_key = L.off_tc = 0;
  }
  L.total = o;
  return L;
}

// Two-value block reduction in one barrier: per warp, a sum of `a` and an inclusive scan of
// `b`; returns the block sum of a, the exclusive prefix of b, and the block total of b.
// `ra`, `rb` hold NW ints each and must not be reused before the next barrier.
__device__ __forceinline__ void block_sum_exscan(int a, int b, int* ra, int* rb, int* sum_a,
                                                 int* pre_b, int* tot_b) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int wa = __reduce_add_sync(0xffffffffu, a);
  const int inc = b200::warp_inclusive_scan(b);
  if (l == 31) {
    ra[w] = wa;
    rb[w] = inc;
  }
  __syncthreads();
  // lane i < NW of every warp picks up warp i's totals; shuffles combine them
  const int xa = (l < NW) ? ra[l] : 0, xb = (l < NW) ? rb[l] : 0;
  const int sa = __reduce_add_sync(0xffffffffu, xa);
  const int tb = __reduce_add_sync(0xffffffffu, xb);
  const int before = __reduce_add_sync(0xffffffffu, (l < w) ? xb : 0);
  *sum_a = sa;
  *pre_b = before + inc - b;
  *tot_b = tb;
}

// Programmatic dependent launch: each update kernel is launched so that it may start while the
// kernel ahead of it in the stream is still running; it waits for that kernel (completion and
// memory visibility) before touching any memory, and lets the next kernel launch at once, so
// back-to-back updates overlap one launch latency with the previous update's work.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... Exp, typename... Act>
cudaError_t launch_pdl(void (*kern)(Exp...), int threads, int smem, cudaStream_t stream, Act&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Act>(args)...);
}

struct ManageArgs {
  const int* topk;
  int mk, E, S, max_distinct, max_inserts;
  int* table;
  int* map_cold;
  int* slot_expert;
  long long* slot_stamp;
  unsigned char* routed;
  long long* step;
  int* miss;
  int* n_miss;
};

// The manager, shared by both kernels. Every thread of the block calls it and every thread
// returns (no divergent exit). Six barriers. With FUSED the bucket counters are zeroed in the
// first phase; on return the final expert -> slot table is in s_tab (TAB_SMEM).
template <bool TAB_SMEM, bool FUSED>
__device__ void manage_core(const ManageArgs& a, char* sm, const Smem& L, int (&ids)[IDS_REG]) {
  const int tid = threadIdx.x;
  const int E = a.E, S = a.S, mk = a.mk;
  const int S4 = (S + 3) & ~3;
  unsigned char* flags = reinterpret_cast<unsigned char*>(sm + L.off_flags);
  int* s_tab = reinterpret_cast<int*>(sm + L.off_tab);
  int* s_se = reinterpret_cast<int*>(sm + L.off_se);
  long long* s_st = reinterpret_cast<long long*>(sm + L.off_st);
  long long* s_k64 = reinterpret_cast<long long*>(sm + L.off_k64);
  unsigned* s_k32 = reinterpret_cast<unsigned*>(sm + L.off_k32);
  int* s_vic = reinterpret_cast<int*>(sm + L.off_vic);
  int* s_missE = reinterpret_cast<int*>(sm + L.off_missE);
  int* red = reinterpret_cast<int*>(sm + L.off_red);

  // ---- 1. every independent global load up front; clear the flags ------------------------
  const long long st = a.step[0] + 1;
#pragma unroll
  for (int k = 0; k < IDS_REG; ++k) {
    const int i = k * NT + tid;
    ids[k] = (i < mk) ? a.topk[i] : -1;
  }
  for (int i = tid; i < S; i += NT) {
    s_se[i] = a.slot_expert[i];
    s_st[i] = a.slot_stamp[i];
  }
  if (TAB_SMEM)
    for (int i = tid; i < E; i += NT) s_tab[i] = a.table[i];
  for (int i = tid; i < E; i += NT) flags[i] = 0;
  if (FUSED) {
    int* cnt_h = reinterpret_cast<int*>(sm + L.off_cnt_h);
    int* cnt_c = reinterpret_cast<int*>(sm + L.off_cnt_c);
    for (int i = tid; i < S; i += NT) cnt_h[i] = 0;
    for (int i = tid; i < E; i += NT) cnt_c[i] = 0;
  }
  __syncthreads();                                                          // B1

  // ---- 2. mark the routed experts -------------------------------------------------------
#pragma unroll
  for (int k = 0; k < IDS_REG; ++k) {
    const int e = ids[k];
    if (e >= 0 && e < E) flags[e] = 1;
  }
  for (int i = IDS_REG * NT + tid; i < mk; i += NT) {
    const int e = a.topk[i];
    if (e >= 0 && e < E) flags[e] = 1;
  }
  __syncthreads();                                                          // B2

  // ---- 3. distinct count, hit stamps (shared copy only), misses in expert-id order ------
  const int C = (E + NT - 1) / NT;
  const int lo = min(tid * C, E), hi = min(lo + C, E);
  int cnt = 0, local = 0;
  for (int e = lo; e < hi; ++e) {
    const int f = flags[e];
    a.routed[e] = (unsigned char)f;
    if (!f) continue;
    ++cnt;
    const int s = TAB_SMEM ? s_tab[e] : a.table[e];
    if (s < 0)
      ++local;
    else if (s < S)
      s_st[s] = st;                 // written back only if the call is not a read-through
  }
  int total_cnt, base, total;
  block_sum_exscan(cnt, local, red, red + NW, &total_cnt, &base, &total);   // B3
  if (total_cnt > a.max_distinct) {                 // read-through: only step / n_miss change
    if (tid == 0) {
      a.step[0] = st;
      a.n_miss[0] = 0;
    }
    return;
  }
  const int nins = min(total, a.max_inserts);
  if (nins > 0) {
    int j = base;
    for (int e = lo; e < hi && j < nins; ++e) {
      if (!flags[e]) continue;
      const int s = TAB_SMEM ? s_tab[e] : a.table[e];
      if (s >= 0) continue;
      s_missE[j] = e;
      a.miss[2 * j] = e;
      ++j;
    }
  }
  if (nins <= 0) {
    for (int i = tid; i < S; i += NT) a.slot_stamp[i] = s_st[i];
    if (tid == 0) {
      a.step[0] = st;
      a.n_miss[0] = 0;
    }
    return;
  }

  // ---- 4. victim keys: (stamp << 20) | slot, and the order-equivalent 32-bit form ---------
  // ((2^21 - 1 - (step - stamp)) << 11) | slot, valid when every evictable stamp is within
  // 2^21 steps of the current one (checked; otherwise the 64-bit keys are ranked).
  int nev = 0, nofit = 0;
  for (int i = tid; i < S4; i += NT) {
    long long k64 = KEY_MAX;
    unsigned k32 = KEY32_MAX;
    if (i < S) {
      const int se = s_se[i];
      const bool busy = (se >= 0 && se < E && flags[se]);
      if (!busy) {
        const long long stamp = s_st[i];
        const long long age = st - stamp;
        k64 = (stamp << SLOT_BITS) | (long long)i;
        if (age >= 0 && age < (1LL << AGE_BITS))
          k32 = ((unsigned)((1LL << AGE_BITS) - 1 - age) << 11) | (unsigned)i;
        else
          ++nofit;
        ++nev;
      }
    }
    s_k64[i] = k64;
    s_k32[i] = k32;
  }
  int nev_total, dummy, nofit_total;
  block_sum_exscan(nev, nofit, red + 2 * NW, red + 3 * NW, &nev_total, &dummy, &nofit_total);  // B4
  const int nact = min(nins, nev_total);

  // ---- 5. victims: the nins smallest keys, victim r = the slot of the r-th smallest --------
  // Keys are unique (the slot is in the low bits), so ranks are well defined. Few inserts
  // (nins <= SEL_MAX, 32-bit keys, S <= 1024): each warp takes its 64 keys and pulls out its own
  // nins smallest with warp min-reductions; the block's nins smallest are among those
  // candidates, so ranking the candidates against one another names the victims.
  if (nofit_total == 0 && nins <= SEL_MAX) {
    unsigned* cand = reinterpret_cast<unsigned*>(sm + L.off_cand);
    const int w = tid >> 5, l = tid & 31;
    const int i0 = 32 * w + l, i1 = 32 * (w + NW) + l;
    const unsigned ka = (i0 < S) ? s_k32[i0] : KEY32_MAX;
    const unsigned kb = (i1 < S) ? s_k32[i1] : KEY32_MAX;
    unsigned lo2 = min(ka, kb), hi2 = max(ka, kb);
    for (int r = 0; r < nins; ++r) {
      const unsigned m = __reduce_min_sync(0xffffffffu, lo2);
      if (l == 0) cand[w * nins + r] = m;
      if (lo2 == m) {                       // the (unique) owner moves to its next key
        lo2 = hi2;
        hi2 = KEY32_MAX;
      }
    }
    __syncthreads();
    const int nc = NW * nins;               // a multiple of 16, so uint4 reads cover it
    for (int c = tid; c < nc; c += NT) {
      const unsigned k = cand[c];
      if (k == KEY32_MAX) continue;
      const uint4* cv = reinterpret_cast<const uint4*>(cand);
      int r = 0;
#pragma unroll 8
      for (int j = 0; j < (nc >> 2); ++j) {
        const uint4 q = cv[j];
        r += (q.x < k) + (q.y < k) + (q.z < k) + (q.w < k);
      }
      if (r < nins) s_vic[r] = (int)(k & 0x7ffu);
    }
  } else if (nofit_total == 0) {
    const unsigned k0 = (tid < S) ? s_k32[tid] : KEY32_MAX;
    const unsigned k1 = (tid + NT < S) ? s_k32[tid + NT] : KEY32_MAX;
    if (k0 != KEY32_MAX || k1 != KEY32_MAX) {
      const uint4* kv = reinterpret_cast<const uint4*>(s_k32);
      int r0 = 0, r1 = 0;
      if (S <= NT) {
#pragma unroll 8
        for (int j = 0; j < (S4 >> 2); ++j) {
          const uint4 q = kv[j];
          r0 += (q.x < k0) + (q.y < k0) + (q.z < k0) + (q.w < k0);
        }
      } else {
#pragma unroll 4
        for (int j = 0; j < (S4 >> 2); ++j) {
          const uint4 q = kv[j];
          r0 += (q.x < k0) + (q.y < k0) + (q.z < k0) + (q.w < k0);
          r1 += (q.x < k1) + (q.y < k1) + (q.z < k1) + (q.w < k1);
        }
      }
      if (k0 != KEY32_MAX && r0 < nins) s_vic[r0] = tid;
      if (k1 != KEY32_MAX && r1 < nins) s_vic[r1] = tid + NT;
    }
  } else {
    const long long k0 = (tid < S) ? s_k64[tid] : KEY_MAX;
    const long long k1 = (tid + NT < S) ? s_k64[tid + NT] : KEY_MAX;
    if (k0 != KEY_MAX || k1 != KEY_MAX) {
      const longlong2* kv = reinterpret_cast<const longlong2*>(s_k64);
      int r0 = 0, r1 = 0;
#pragma unroll 4
      for (int j = 0; j < (S4 >> 1); ++j) {
        const longlong2 q = kv[j];
        r0 += (q.x < k0) + (q.y < k0);
        r1 += (q.x < k1) + (q.y < k1);
      }
      if (k0 != KEY_MAX && r0 < nins) s_vic[r0] = tid;
      if (k1 != KEY_MAX && r1 < nins) s_vic[r1] = tid + NT;
    }
  }
  __syncthreads();                                                          // B5

  // ---- 6. install the victims in parallel (r4d_lru.hip:102-117) -----------------------------
  // victim slots are distinct, missing experts are distinct, and an evicted expert is not
  // routed while every inserted one is, so no two threads touch the same entry.
  for (int r = tid; r < nact; r += NT) {
    const int sl = s_vic[r];
    const int e = s_missE[r];
    const int old = s_se[sl];
    if (old >= 0 && old < E) {
      if (TAB_SMEM) s_tab[old] = -1;
      a.table[old] = -1;
      a.map_cold[old] = old;
    }
    s_se[sl] = e;
    s_st[sl] = st;
    if (TAB_SMEM) s_tab[e] = sl;
    a.table[e] = sl;
    a.map_cold[e] = -1;
    a.miss[2 * r + 1] = sl;
  }
  __syncthreads();                                                          // B6
  for (int i = tid; i < S; i += NT) {
    a.slot_expert[i] = s_se[i];
    a.slot_stamp[i] = s_st[i];
  }
  if (tid == 0) {
    a.step[0] = st;
    a.n_miss[0] = nact;
  }
}

template <bool TAB_SMEM>
__global__ void __launch_bounds__(NT) lru_manage_kernel(ManageArgs a) {
  extern __shared__ __align__(16) char sm[];
  const Smem L = smem_layout(a.E, a.S, TAB_SMEM, false);
  int ids[IDS_REG];
  pdl_enter();
  manage_core<TAB_SMEM, false>(a, sm, L, ids);
}

struct FusedArgs {
  ManageArgs m;
  int bs, L, NB;
  int* sorted_hot;
  int* eids_hot;
  int* npad_hot;
  int* sorted_cold;
  int* eids_cold;
  int* npad_cold;
};

// One side's padding: sorted_ids sentinels after each bucket's tokens and the bucket id of
// each of its blocks, for the buckets [lo, hi) this thread owns; then the counts become the
// placement cursors (same owner, so no other thread reads them meanwhile).
__device__ __forceinline__ int fill_side(int lo, int hi, int* cnt, int* cum, int run, int bs,
                                         int mk, int Lcap, int NBcap, int* sorted, int* eids) {
  for (int b = lo; b < hi; ++b) {
    const int c = cnt[b];
    const int pad = (c + bs - 1) / bs * bs;
    cum[b] = run;
    for (int p = run + c; p < run + pad && p < Lcap; ++p) sorted[p] = mk;
    for (int blk = run / bs; blk < (run + pad) / bs && blk < NBcap; ++blk) eids[blk] = b;
    cnt[b] = run;
    run += pad;
  }
  return run;
}

__global__ void __launch_bounds__(NT) lru_fused_kernel(FusedArgs f) {
  extern __shared__ __align__(16) char sm[];
  const ManageArgs& a = f.m;
  const int E = a.E, S = a.S, mk = a.mk, bs = f.bs;
  const Smem L = smem_layout(E, S, true, true);
  const int tid = threadIdx.x;
  int ids[IDS_REG];
  pdl_enter();

  // ---- the manager (single exit: every output below is always written) ------------------
  // Its last barrier orders the table installs before the reads below; on its early exits
  // the shared table is unchanged since its second barrier, and the counters were zeroed in
  // its first phase.
  manage_core<true, true>(a, sm, L, ids);

  const int* s_tab = reinterpret_cast<const int*>(sm + L.off_tab);
  int* cnt_h = reinterpret_cast<int*>(sm + L.off_cnt_h);
  int* cum_h = reinterpret_cast<int*>(sm + L.off_cum_h);
  int* cnt_c = reinterpret_cast<int*>(sm + L.off_cnt_c);
  int* cum_c = reinterpret_cast<int*>(sm + L.off_cum_c);
  int* red = reinterpret_cast<int*>(sm + L.off_red);

  // bucket key of token i: slot (hot) or MAXS + expert (cold); -1 = ignored
  auto bucket_of = [&](int e) -> int {
    if (e < 0 || e >= E) return -1;
    const int s = s_tab[e];
    return ((unsigned)s < (unsigned)S) ? s : (MAXS + e);
  };
  auto padded = [&](int c) { return (c + bs - 1) / bs * bs; };

  if (mk <= SMALL_MK) {
    // ---- few routed ids (decode): every token ranks itself directly --------------------------
    // Token i's slot in its side's sorted list = (padded sizes of that side's buckets with a
    // smaller key) + (tokens of its own bucket with a smaller index): the same stable order as
    // the counting sort below, from two O(mk) passes per token and no bucket scans. Padding
    // sentinels go in first, in parallel; the token writes come two barriers later.
    int* s_key = reinterpret_cast<int*>(sm + L.off_key);
    int* s_tc = reinterpret_cast<int*>(sm + L.off_tc);
    for (int p = tid; p < f.L; p += NT) {
      f.sorted_hot[p] = mk;
      f.sorted_cold[p] = mk;
    }
    // keys padded to a multiple of 4 with -1 so the passes read int4 vectors
    const int key = (tid < mk) ? bucket_of(ids[0]) : -1;
    const int mk4 = (mk + 3) & ~3;
    if (tid < mk4) s_key[tid] = key;
    __syncthreads();
    int cnt = 0, eqb = 0;
    const int4* kv = reinterpret_cast<const int4*>(s_key);
    if (key >= 0) {
#pragma unroll 4
      for (int j = 0; j < (mk4 >> 2); ++j) {
        const int4 q = kv[j];
        const int j0 = 4 * j;
        const int a0 = q.x == key, a1 = q.y == key, a2 = q.z == key, a3 = q.w == key;
        cnt += a0 + a1 + a2 + a3;
        eqb += (j0 < tid ? a0 : 0) + (j0 + 1 < tid ? a1 : 0) + (j0 + 2 < tid ? a2 : 0) + (j0 + 3 < tid ? a3 : 0);
      }
    }
    // s_tc[j]: the padded size of token j's bucket if j is the bucket's first token, else 0
    if (tid < mk4) s_tc[tid] = (key >= 0 && eqb == 0) ? padded(cnt) : 0;
    __syncthreads();
    int ph = 0, pc = 0;
    if (key >= 0) {
      const bool hot = key < MAXS;
      // same side and a smaller key: hot keys are < MAXS <= cold keys, so for a cold token
      // the hot keys must be excluded explicitly
      const int lo_key = hot ? 0 : MAXS;
      const int4* pv = reinterpret_cast<const int4*>(s_tc);
      int before = 0;
#pragma unroll 4
      for (int j = 0; j < (mk4 >> 2); ++j) {
        const int4 q = kv[j], pq = pv[j];
        before += ((q.x >= lo_key && q.x < key) ? pq.x : 0) + ((q.y >= lo_key && q.y < key) ? pq.y : 0) +
                  ((q.z >= lo_key && q.z < key) ? pq.z : 0) + ((q.w >= lo_key && q.w < key) ? pq.w : 0);
      }
      const int pos = before + eqb;
      if (pos < f.L) (hot ? f.sorted_hot : f.sorted_cold)[pos] = tid;
      if (eqb == 0) {                       // first token of its bucket: the bucket's block ids
        const int bkt = hot ? key : key - MAXS, pn = padded(cnt);
        int* eids = hot ? f.eids_hot : f.eids_cold;
        for (int blk = before / bs; blk < (before + pn) / bs && blk < f.NB; ++blk) eids[blk] = bkt;
        (hot ? ph : pc) = pn;
      }
    }
    int tot_h, tot_c, unused;
    block_sum_exscan(ph, pc, red + 6 * NW, red + 7 * NW, &tot_h, &unused, &tot_c);
    if (tid == 0) {
      f.npad_hot[0] = tot_h;
      f.npad_cold[0] = tot_c;
    }
    for (int blk = tot_h / bs + tid; blk < f.NB; blk += NT) f.eids_hot[blk] = -1;
    for (int blk = tot_c / bs + tid; blk < f.NB; blk += NT) f.eids_cold[blk] = -1;
    return;
  }

  // ---- counts (shared atomics: the counts do not depend on the order) --------------------
#pragma unroll
  for (int k = 0; k < IDS_REG; ++k) {
    const int b = bucket_of(ids[k]);
    if (b >= 0) atomicAdd(b < MAXS ? &cnt_h[b] : &cnt_c[b - MAXS], 1);
  }
  for (int i = IDS_REG * NT + tid; i < mk; i += NT) {
    const int b = bucket_of(a.topk[i]);
    if (b >= 0) atomicAdd(b < MAXS ? &cnt_h[b] : &cnt_c[b - MAXS], 1);
  }
  __syncthreads();

  // ---- block-padded exclusive scans of both sides in one barrier --------------------------
  const int Ch = (S + NT - 1) / NT, Cc = (E + NT - 1) / NT;
  const int lh = min(tid * Ch, S), hh = min(lh + Ch, S);
  const int lc = min(tid * Cc, E), hc = min(lc + Cc, E);
  int sh = 0, sc = 0;
  for (int b = lh; b < hh; ++b) sh += (cnt_h[b] + bs - 1) / bs * bs;
  for (int b = lc; b < hc; ++b) sc += (cnt_c[b] + bs - 1) / bs * bs;
  int eh, ec, tot_h, tot_c;
  {
    const int w = tid >> 5, l = tid & 31;
    const int ih = b200::warp_inclusive_scan(sh), ic = b200::warp_inclusive_scan(sc);
    if (l == 31) {
      red[4 * NW + w] = ih;
      red[5 * NW + w] = ic;
    }
    __syncthreads();
    int bh = 0, bc = 0;
    tot_h = tot_c = 0;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int xh = red[4 * NW + i], xc = red[5 * NW + i];
      bh += (i < w) ? xh : 0;
      bc += (i < w) ? xc : 0;
      tot_h += xh;
      tot_c += xc;
    }
    eh = bh + ih - sh;
    ec = bc + ic - sc;
  }
  if (tid == 0) {
    f.npad_hot[0] = tot_h;
    f.npad_cold[0] = tot_c;
  }

  // ---- expert_ids, padding sentinels, tails; counts become cursors -------------------------
  fill_side(lh, hh, cnt_h, cum_h, eh, bs, mk, f.L, f.NB, f.sorted_hot, f.eids_hot);
  fill_side(lc, hc, cnt_c, cum_c, ec, bs, mk, f.L, f.NB, f.sorted_cold, f.eids_cold);
  for (int p = tot_h + tid; p < f.L; p += NT) f.sorted_hot[p] = mk;
  for (int p = tot_c + tid; p < f.L; p += NT) f.sorted_cold[p] = mk;
  for (int blk = tot_h / bs + tid; blk < f.NB; blk += NT) f.eids_hot[blk] = -1;
  for (int blk = tot_c / bs + tid; blk < f.NB; blk += NT) f.eids_cold[blk] = -1;
  __syncthreads();

  // ---- stable placement: warp match_any ranks, warps advance the cursors in order --------
  const int warp = tid >> 5;
  const unsigned lt = b200::lanemask_lt();
  for (int base = 0, k = 0; base < mk; base += NT, ++k) {
    const int i = base + tid;
    int e = -1;
    if (i < mk) {
      if (k < IDS_REG) {
#pragma unroll
        for (int q = 0; q < IDS_REG; ++q)
          if (q == k) e = ids[q];
      } else {
        e = a.topk[i];
      }
    }
    const int key = bucket_of(e);
    for (int w = 0; w < NW && base + w * 32 < mk; ++w) {
      if (warp == w) {
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & lt);
        int* cur = nullptr;
        if (key >= 0) {
          cur = key < MAXS ? &cnt_h[key] : &cnt_c[key - MAXS];
          const int pos = *cur + rank;
          if (pos < f.L) (key < MAXS ? f.sorted_hot : f.sorted_cold)[pos] = i;
        }
        __syncwarp();
        if (key >= 0 && rank == 0) *cur = *cur + __popc(peers);
      }
      __syncthreads();
    }
  }
}

// ---- gather: copy the six per-expert slabs of every miss into its slot ---------------------
struct GatherArgs {
  uint4* d[6];
  const uint4* s[6];
  int v[6];          // 16-byte vectors per expert
  const int* miss;
  const int* n_miss;
};

constexpr int GNT = 256;   // r4d_lru.hip:28 (block = 256)
constexpr int GUNROLL = 4;

// grid = (chunks, lanes): block (c, j) copies misses j, j + lanes, ...; each slab is split
// over the `chunks` blocks by a grid-stride loop of 16-byte accesses (r4d_lru.hip:271-301),
// unrolled so each thread keeps several host-link reads in flight.
__global__ void __launch_bounds__(GNT) lru_gather_kernel(GatherArgs g) {
  const int nm = g.n_miss[0];
  const int stride = gridDim.x * GNT;
  const int start = blockIdx.x * GNT + threadIdx.x;
  for (int j = blockIdx.y; j < nm; j += gridDim.y) {
    const int e = g.miss[2 * j];
    const int sl = g.miss[2 * j + 1];
    if (e < 0 || sl < 0) continue;
#pragma unroll
    for (int b = 0; b < 6; ++b) {
      const int V = g.v[b];
      const uint4* __restrict__ p = g.s[b] + (size_t)e * (size_t)V;
      uint4* __restrict__ q = g.d[b] + (size_t)sl * (size_t)V;
      int i = start;
      for (; i + (GUNROLL - 1) * stride < V; i += GUNROLL * stride) {
        uint4 t[GUNROLL];
#pragma unroll
        for (int u = 0; u < GUNROLL; ++u) t[u] = p[i + u * stride];
#pragma unroll
        for (int u = 0; u < GUNROLL; ++u) q[i + u * stride] = t[u];
      }
      for (; i < V; i += stride) q[i] = p[i];
    }
  }
}


}  // namespace

extern "C" {

// r4d_lru.hip:579-589
int r4d_lru_manage(const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts,
                   int* table, int* map_cold, int* slot_expert, long long* slot_stamp,
                   unsigned char* routed, long long* step, int* miss, int* n_miss,
                   cudaStream_t stream) {
  if (E <= 0 || S <= 0 || S > MAXS || S > SLOT_MASK) return -1;
  if (max_inserts < 0 || max_inserts > MAXINS) return -1;
  if (E > MAXE_MANAGE) return -1;
  ManageArgs a{topk_ids, mk, E, S, max_distinct, max_inserts, table, map_cold,
               slot_expert, slot_stamp, routed, step, miss, n_miss};
  const bool tab = E <= TAB_SMEM_MAX;
  const Smem L = smem_layout(E, S, tab, false);
  if (L.total > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(tab ? (const void*)lru_manage_kernel<true>
                                             : (const void*)lru_manage_kernel<false>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
    if (e != cudaSuccess) return (int)e;
  }
  const cudaError_t e = tab ? launch_pdl(lru_manage_kernel<true>, NT, L.total, stream, a)
                            : launch_pdl(lru_manage_kernel<false>, NT, L.total, stream, a);
  return (int)(e != cudaSuccess ? e : cudaGetLastError());
}

// r4d_lru.hip:596-610. L and NB must be exactly what vLLM's moe_align_block_size wrapper
// allocates: L = mk < E ? min(mk*bs, mk + E*(bs-1)) : mk + E*(bs-1), NB = ceil(L / bs).
int r4d_lru_fused(const int* topk_ids, int mk, int E, int S, int max_distinct, int max_inserts,
                  int* table, int* map_cold, int* slot_expert, long long* slot_stamp,
                  unsigned char* routed, long long* step, int* miss, int* n_miss, int bs, int L,
                  int NB, int* sorted_hot, int* eids_hot, int* npad_hot, int* sorted_cold,
                  int* eids_cold, int* npad_cold, cudaStream_t stream) {
  if (E <= 0 || E > MAXE_FUSED || S <= 0 || S > MAXS || S > SLOT_MASK) return -1;
  if (bs <= 0 || L <= 0 || NB <= 0 || mk < 0) return -1;
  if (max_inserts < 0 || max_inserts > MAXE_FUSED) return -1;
  FusedArgs f{{topk_ids, mk, E, S, max_distinct, max_inserts, table, map_cold, slot_expert,
               slot_stamp, routed, step, miss, n_miss},
              bs, L, NB, sorted_hot, eids_hot, npad_hot, sorted_cold, eids_cold, npad_cold};
  const Smem Ls = smem_layout(E, S, true, true);
  if (Ls.total > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute((const void*)lru_fused_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, Ls.total);
    if (e != cudaSuccess) return (int)e;
  }
  const cudaError_t e = launch_pdl(lru_fused_kernel, NT, Ls.total, stream, f);
  return (int)(e != cudaSuccess ? e : cudaGetLastError());
}

// r4d_lru.hip:612-629. Sizes are BYTES per expert for each of the six buffers; each must be
// a positive multiple of 16. Sources may be mapped pinned host memory (UVA).
int r4d_lru_gather(void* d0, const void* s0, long b0, void* d1, const void* s1, long b1, void* d2,
                   const void* s2, long b2, void* d3, const void* s3, long b3, void* d4,
                   const void* s4, long b4, void* d5, const void* s5, long b5, const int* miss,
                   const int* n_miss, int chunks, int lanes, cudaStream_t stream) {
  const long bs[6] = {b0, b1, b2, b3, b4, b5};
  for (int i = 0; i < 6; i++)
    if (bs[i] <= 0 || bs[i] % 16) return -1;
  if (chunks <= 0 || lanes <= 0) return -1;
  GatherArgs g;
  void* ds[6] = {d0, d1, d2, d3, d4, d5};
  const void* ss[6] = {s0, s1, s2, s3, s4, s5};
  for (int i = 0; i < 6; i++) {
    if (bs[i] / 16 > 0x7fffffffL) return -1;
    g.d[i] = (uint4*)ds[i];
    g.s[i] = (const uint4*)ss[i];
    g.v[i] = (int)(bs[i] / 16);
  }
  g.miss = miss;
  g.n_miss = n_miss;
  lru_gather_kernel<<<dim3(chunks, lanes), GNT, 0, stream>>>(g);
  return (int)cudaGetLastError();
}

// Device pointer of a pinned host buffer (the UVA source the gather reads); mirrors the
// hipHostGetDevicePointer call of tests/lru/test_lru.py:42-50.
int r4d_lru_host_device_pointer(void* host, void** dev) {
  return (int)cudaHostGetDevicePointer(dev, host, 0);
}

}  // extern "C"

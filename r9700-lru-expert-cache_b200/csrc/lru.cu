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
constexpr int IDS_REG = 4;                // topk ids kept in registers: mk <= IDS_REG * NT

// Shared-memory carve-up (bytes), all offsets 16-byte aligned.
struct Smem {
  int off_flags, off_tab, off_se, off_st, off_key, off_vic, off_missE;
  int off_cnt_h, off_cum_h, off_cnt_c, off_cum_c, off_red, total;
};

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

__host__ __device__ inline Smem smem_layout(int E, int S, bool tab_smem, bool fused) {
  Smem L;
  int o = 0;
  L.off_red = o;   o += align16(4 * 64 * (int)sizeof(int));
  L.off_flags = o; o += align16(E);
  L.off_tab = o;   o += tab_smem ? align16(E * 4) : 0;
  L.off_se = o;    o += align16(S * 4);
  L.off_st = o;    o += align16(S * 8);
  L.off_key = o;   o += align16(S * 8);
  L.off_vic = o;   o += align16(MAXINS * 4);
  L.off_missE = o; o += align16(MAXINS * 4);
  if (fused) {
    L.off_cnt_h = o; o += align16(S * 4);
    L.off_cum_h = o; o += align16((S + 1) * 4);
    L.off_cnt_c = o; o += align16(E * 4);
    L.off_cum_c = o; o += align16((E + 1) * 4);
  } else {
    L.off_cnt_h = L.off_cum_h = L.off_cnt_c = L.off_cum_c = 0;
  }
  L.total = o;
  return L;
}

// Block sum of one int per thread; `red` holds NW ints. One barrier; every thread returns
// the total. `red` must not be reused before the next barrier.
__device__ __forceinline__ int block_sum(int v, int* red) {
  v = __reduce_add_sync(0xffffffffu, v);
  if (b200::lane_id() == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  int t = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) t += red[w];
  return t;
}

// Exclusive block scan of one int per thread; one barrier; `red` holds NW ints.
__device__ __forceinline__ int block_exscan(int v, int* red, int* total) {
  const int inc = b200::warp_inclusive_scan(v);
  const int w = threadIdx.x >> 5;
  if (b200::lane_id() == 31) red[w] = inc;
  __syncthreads();
  int before = 0, t = 0;
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    const int x = red[i];
    before += (i < w) ? x : 0;
    t += x;
  }
  *total = t;
  return before + inc - v;
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

// The manager, shared by both kernels. Every thread of the block calls it and every
// thread returns (no early exit), so the fused kernel can carry on. On return the final
// expert -> slot table is in s_tab when TAB_SMEM.
template <bool TAB_SMEM>
__device__ void manage_core(const ManageArgs& a, char* sm, const Smem& L, int (&ids)[IDS_REG]) {
  const int tid = threadIdx.x;
  const int E = a.E, S = a.S, mk = a.mk;
  unsigned char* flags = reinterpret_cast<unsigned char*>(sm + L.off_flags);
  int* s_tab = reinterpret_cast<int*>(sm + L.off_tab);
  int* s_se = reinterpret_cast<int*>(sm + L.off_se);
  long long* s_st = reinterpret_cast<long long*>(sm + L.off_st);
  long long* s_key = reinterpret_cast<long long*>(sm + L.off_key);
  int* s_vic = reinterpret_cast<int*>(sm + L.off_vic);
  int* s_missE = reinterpret_cast<int*>(sm + L.off_missE);
  int* red = reinterpret_cast<int*>(sm + L.off_red);

  // ---- issue every independent global load up front ----------------------------------
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
  __syncthreads();

  // ---- mark the routed experts ----------------------------------------------------------
#pragma unroll
  for (int k = 0; k < IDS_REG; ++k) {
    const int e = ids[k];
    if (e >= 0 && e < E) flags[e] = 1;
  }
  for (int i = IDS_REG * NT + tid; i < mk; i += NT) {
    const int e = a.topk[i];
    if (e >= 0 && e < E) flags[e] = 1;
  }
  __syncthreads();

  // ---- distinct count, and the per-thread miss count over a contiguous expert chunk ----
  const int C = (E + NT - 1) / NT;
  const int lo = tid * C, hi = min(lo + C, E);
  int cnt = 0, local = 0;
  for (int e = lo; e < hi; ++e) {
    const int f = flags[e];
    a.routed[e] = (unsigned char)f;              // the reference leaves its scratch this way
    cnt += f;
    if (f) {
      const int s = TAB_SMEM ? s_tab[e] : a.table[e];
      local += (s < 0);
    }
  }
  cnt = block_sum(cnt, red);
  if (cnt > a.max_distinct) {                    // read-through: only step / n_miss change
    if (tid == 0) {
      a.step[0] = st;
      a.n_miss[0] = 0;
    }
    return;
  }

  // ---- hits refresh their stamp; misses enumerated in expert-id order ------------------
  for (int e = lo; e < hi; ++e) {
    if (!flags[e]) continue;
    const int s = TAB_SMEM ? s_tab[e] : a.table[e];
    if (s >= 0 && s < S) s_st[s] = st;
  }
  int total = 0;
  const int base = block_exscan(local, red + NW, &total);
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

  // ---- victim keys: (stamp << 20) | slot, or KEY_MAX when the slot's expert is routed ----
  int nev = 0;
  for (int i = tid; i < S; i += NT) {
    const int se = s_se[i];
    const bool busy = (se >= 0 && se < E && flags[se]);
    s_key[i] = busy ? KEY_MAX : ((s_st[i] << SLOT_BITS) | (long long)i);
    nev += busy ? 0 : 1;
  }
  nev = block_sum(nev, red + 2 * NW);           // the barrier also publishes s_key / s_missE
  const int nact = min(nins, nev);

  // ---- rank every evictable key against the whole array: rank r < nins -> victim r ------
  {
    const int i0 = tid, i1 = tid + NT;
    const long long k0 = (i0 < S) ? s_key[i0] : KEY_MAX;
    const long long k1 = (i1 < S) ? s_key[i1] : KEY_MAX;
    int r0 = 0, r1 = 0;
    const longlong2* kv = reinterpret_cast<const longlong2*>(s_key);
    const int S2 = S >> 1;
#pragma unroll 4
    for (int j = 0; j < S2; ++j) {
      const longlong2 p = kv[j];
      r0 += (p.x < k0) + (p.y < k0);
      r1 += (p.x < k1) + (p.y < k1);
    }
    if (S & 1) {
      const long long p = s_key[S - 1];
      r0 += (p < k0);
      r1 += (p < k1);
    }
    if (k0 != KEY_MAX && r0 < nins) s_vic[r0] = i0;
    if (k1 != KEY_MAX && r1 < nins) s_vic[r1] = i1;
  }
  __syncthreads();

  // ---- install the victims in parallel (r4d_lru.hip:102-117) -----------------------------
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
  __syncthreads();
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
  manage_core<TAB_SMEM>(a, sm, L, ids);
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

// One side's block-padded bucket bookkeeping: pad fills of sorted_ids and expert_ids for the
// buckets [lo, hi) this thread owns (the non-padding slots are written by placement).
__device__ __forceinline__ void fill_side(int lo, int hi, const int* cnt, const int* cum, int bs,
                                          int mk, int Lcap, int NBcap, int* sorted, int* eids) {
  for (int b = lo; b < hi; ++b) {
    const int c0 = cum[b], c1 = cum[b + 1];
    for (int p = c0 + cnt[b]; p < c1 && p < Lcap; ++p) sorted[p] = mk;
    for (int blk = c0 / bs; blk < c1 / bs && blk < NBcap; ++blk) eids[blk] = b;
  }
}

__global__ void __launch_bounds__(NT) lru_fused_kernel(FusedArgs f) {
  extern __shared__ __align__(16) char sm[];
  const ManageArgs& a = f.m;
  const int E = a.E, S = a.S, mk = a.mk, bs = f.bs;
  const Smem L = smem_layout(E, S, true, true);
  const int tid = threadIdx.x;
  int ids[IDS_REG];

  // ---- phase 0: the manager (single exit: every output below is always written) --------
  manage_core<true>(a, sm, L, ids);
  __syncthreads();

  const int* s_tab = reinterpret_cast<const int*>(sm + L.off_tab);
  int* cnt_h = reinterpret_cast<int*>(sm + L.off_cnt_h);
  int* cum_h = reinterpret_cast<int*>(sm + L.off_cum_h);
  int* cnt_c = reinterpret_cast<int*>(sm + L.off_cnt_c);
  int* cum_c = reinterpret_cast<int*>(sm + L.off_cum_c);
  int* red = reinterpret_cast<int*>(sm + L.off_red);

  for (int i = tid; i < S; i += NT) cnt_h[i] = 0;
  for (int i = tid; i < E; i += NT) cnt_c[i] = 0;
  __syncthreads();

  // bucket key of token i: slot (hot) or MAXS + expert (cold); -1 = ignored
  auto bucket_of = [&](int e) -> int {
    if (e < 0 || e >= E) return -1;
    const int s = s_tab[e];
    return ((unsigned)s < (unsigned)S) ? s : (MAXS + e);
  };

  // ---- phase 2: counts (smem atomics: the counts do not depend on the order) -------------
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

  // ---- phase 3: block-padded exclusive scans of both sides in one block scan ------------
  const int Ch = (S + NT - 1) / NT, Cc = (E + NT - 1) / NT;
  const int lh = min(tid * Ch, S), hh = min(lh + Ch, S);
  const int lc = min(tid * Cc, E), hc = min(lc + Cc, E);
  int sh = 0, sc = 0;
  for (int b = lh; b < hh; ++b) sh += (cnt_h[b] + bs - 1) / bs * bs;
  for (int b = lc; b < hc; ++b) sc += (cnt_c[b] + bs - 1) / bs * bs;
  int tot_h = 0, tot_c = 0;
  const int eh = block_exscan(sh, red, &tot_h);
  const int ec = block_exscan(sc, red + NW, &tot_c);
  {
    int run = eh;
    for (int b = lh; b < hh; ++b) {
      cum_h[b] = run;
      run += (cnt_h[b] + bs - 1) / bs * bs;
    }
    run = ec;
    for (int b = lc; b < hc; ++b) {
      cum_c[b] = run;
      run += (cnt_c[b] + bs - 1) / bs * bs;
    }
    if (tid == 0) {
      cum_h[S] = tot_h;
      cum_c[E] = tot_c;
      f.npad_hot[0] = tot_h;
      f.npad_cold[0] = tot_c;
    }
  }
  __syncthreads();

  // ---- phase 4: expert_ids and padding sentinels; tail past npad --------------------------
  fill_side(lh, hh, cnt_h, cum_h, bs, mk, f.L, f.NB, f.sorted_hot, f.eids_hot);
  fill_side(lc, hc, cnt_c, cum_c, bs, mk, f.L, f.NB, f.sorted_cold, f.eids_cold);
  for (int p = tot_h + tid; p < f.L; p += NT) f.sorted_hot[p] = mk;
  for (int p = tot_c + tid; p < f.L; p += NT) f.sorted_cold[p] = mk;
  for (int blk = tot_h / bs + tid; blk < f.NB; blk += NT) f.eids_hot[blk] = -1;
  for (int blk = tot_c / bs + tid; blk < f.NB; blk += NT) f.eids_cold[blk] = -1;

  // ---- phase 5: stable placement; cnt_* become the running cursors -----------------------
  // (same bucket ownership as fill_side, so each thread overwrites only counts it has read)
  for (int b = lh; b < hh; ++b) cnt_h[b] = cum_h[b];
  for (int b = lc; b < hc; ++b) cnt_c[b] = cum_c[b];
  __syncthreads();
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
        int pos = 0;
        if (key >= 0) {
          cur = key < MAXS ? &cnt_h[key] : &cnt_c[key - MAXS];
          pos = *cur + rank;
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

bool g_attr_done[2] = {false, false};

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
  if (tab)
    lru_manage_kernel<true><<<1, NT, L.total, stream>>>(a);
  else
    lru_manage_kernel<false><<<1, NT, L.total, stream>>>(a);
  return (int)cudaGetLastError();
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
  lru_fused_kernel<<<1, NT, Ls.total, stream>>>(f);
  return (int)cudaGetLastError();
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

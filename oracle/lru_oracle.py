"""numpy restatement of the device-side LRU expert cache -- TEST INFRASTRUCTURE ONLY.

Follows kernels/lru/r4d_lru.hip of davetha/r9700-lru-expert-cache:

* ``manage``  -- ``lru_manage_k`` (r4d_lru.hip:187-269) with ``pickVictims`` /
  ``installVictim`` (r4d_lru.hip:102-185). The serial-argmin and the ranking branches of
  ``pickVictims`` give the same answer (r4d_lru.hip:82-93); this oracle states the answer
  directly: the ``nins`` smallest ``(stamp << 20) | slot`` keys among the slots whose expert
  is not routed this step, installed in ascending key order against the misses in
  ascending expert-id order.
* ``fused``   -- ``lru_fused_k`` (r4d_lru.hip:418-575): the manager, then both
  ``moe_align_block_size`` outputs from the rewritten table (hot side bucketed by slot,
  cold side by expert id, block-padded, sentinel ``mk``, unused expert_ids ``-1``).
  Placement inside a bucket is ascending token index, which is the reference's order for
  ``mk <= 256`` (r4d_lru.hip:542-562) and a valid instance of its atomic order above.
* ``align_sizes`` -- the lengths vLLM's wrapper allocates (r4d_lru.hip:591-595,
  tests/lru/test_fused.py:62-67).
* ``moe_align_block_size`` -- the vLLM op ``lru_fused_k`` replaces, with
  ``ignore_invalid_experts=True`` and an ``expert_map`` (r4d_lru.hip:311-327).

Inputs that the reference leaves undefined (a ``table`` entry >= S, a ``slot_expert``
entry >= E) are treated the way the B200 kernels guard them: the access is skipped.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass, field

import numpy as np

SLOT_BITS = 20           # r4d_lru.hip:29
KEY_MAX = np.iinfo(np.int64).max


@dataclass
class LruState:
    """The eight caller-owned buffers of one MoE layer (kernels/lru/README.md:50-57)."""
    table: np.ndarray                    # int32 [E]  expert -> slot or -1
    map_cold: np.ndarray                 # int32 [E]  expert -> expert when not resident
    slot_expert: np.ndarray              # int32 [S]  slot -> expert or -1
    slot_stamp: np.ndarray               # int64 [S]
    step: int = 0
    routed: np.ndarray = field(default=None)   # uint8 [E] scratch written by the kernel
    miss: np.ndarray = field(default=None)     # int32 [cap, 2]
    n_miss: int = 0

    def __post_init__(self):
        E = self.table.shape[0]
        if self.routed is None:
            self.routed = np.zeros(E, dtype=np.uint8)
        if self.miss is None:
            self.miss = np.full((1, 2), -1, dtype=np.int32)

    @property
    def E(self) -> int:
        return int(self.table.shape[0])

    @property
    def S(self) -> int:
        return int(self.slot_expert.shape[0])

    def copy(self) -> "LruState":
        return LruState(self.table.copy(), self.map_cold.copy(), self.slot_expert.copy(),
                        self.slot_stamp.copy(), int(self.step), self.routed.copy(),
                        self.miss.copy(), int(self.n_miss))


def warm_state(E: int, S: int, hot, stamps=None, step: int = 0, cap: int = 64,
               resident: int | None = None) -> LruState:
    """Warm start: slot i holds hot[i] (tests/lru/test_lru.py:53-66,
    r4d_mxfp4_moe.py.lru.diff L512-533). ``stamps`` defaults to zeros."""
    hot = np.asarray(hot, dtype=np.int64)
    table = np.full(E, -1, dtype=np.int32)
    table[hot] = np.arange(len(hot), dtype=np.int32)
    map_cold = np.arange(E, dtype=np.int32)
    map_cold[hot] = -1
    se = np.full(S, -1, dtype=np.int32)
    se[:len(hot)] = hot
    st = np.zeros(S, dtype=np.int64) if stamps is None else np.asarray(stamps, np.int64).copy()
    return LruState(table, map_cold, se, st, int(step), np.zeros(E, np.uint8),
                    np.full((max(cap, 1), 2), -1, dtype=np.int32), 0)


def manage(s: LruState, topk, max_distinct: int, max_inserts: int) -> int:
    """One ``lru_manage_k`` call (r4d_lru.hip:187-269). Mutates ``s``; returns n_miss."""
    E, S = s.E, s.S
    ids = np.asarray(topk, dtype=np.int64).ravel()
    s.step += 1                                   # :208-211
    s.n_miss = 0
    s.routed[:] = 0                               # :212
    v = ids[(ids >= 0) & (ids < E)]               # :216-219
    s.routed[v] = 1
    if int(s.routed.sum()) > max_distinct:        # :222-226 read-through
        return 0
    st = s.step
    routed_ids = np.nonzero(s.routed)[0]          # ascending expert id (:230-238)
    slots = s.table[routed_ids]
    hit = (slots >= 0)
    hs = slots[hit & (slots < S)]
    s.slot_stamp[hs] = st
    misses = routed_ids[~hit]
    nins = min(len(misses), max_inserts)          # :242
    if nins <= 0:
        return 0
    s.miss.reshape(-1)[0:2 * nins:2] = misses[:nins]    # :244-251
    se = s.slot_expert
    routed_slot = (se >= 0) & (se < E)
    routed_slot[routed_slot] = s.routed[se[routed_slot]] != 0
    keys = (s.slot_stamp << SLOT_BITS) | np.arange(S, dtype=np.int64)   # :128-129
    cand = np.nonzero(~routed_slot)[0]
    order = cand[np.argsort(keys[cand], kind="stable")]
    victims = order[:nins]
    for r, sl in enumerate(victims.tolist()):     # installVictim :102-117
        e = int(misses[r])
        old = int(se[sl])
        if 0 <= old < E:
            s.table[old] = -1
            s.map_cold[old] = old
        se[sl] = e
        s.slot_stamp[sl] = st
        s.table[e] = sl
        s.map_cold[e] = -1
        s.miss.reshape(-1)[2 * r + 1] = sl
    s.n_miss = len(victims)                       # :268
    return s.n_miss


def align_sizes(mk: int, E: int, bs: int = 16) -> tuple[int, int]:
    """(L, NB) vLLM's moe_align_block_size wrapper allocates (r4d_lru.hip:591-595)."""
    L = mk + E * (bs - 1)
    if mk < E:
        L = min(mk * bs, L)
    return L, (L + bs - 1) // bs


def _bucket_align(keys: np.ndarray, nbuckets: int, bs: int, mk: int, L: int, NB: int):
    """Block-padded stable bucket sort of token indices (phases 1-5, r4d_lru.hip:502-575)."""
    sorted_ids = np.full(L, mk, dtype=np.int32)
    eids = np.full(NB, -1, dtype=np.int32)
    cnt = np.bincount(keys[keys >= 0], minlength=nbuckets)[:nbuckets]
    padded = (cnt + bs - 1) // bs * bs
    cum = np.zeros(nbuckets + 1, dtype=np.int64)
    cum[1:] = np.cumsum(padded)
    npad = int(cum[-1])
    for b in np.nonzero(cnt)[0].tolist():
        blocks = np.arange(cum[b] // bs, cum[b + 1] // bs)
        blocks = blocks[blocks < NB]
        eids[blocks] = b
        toks = np.nonzero(keys == b)[0]
        pos = cum[b] + np.arange(len(toks))
        ok = pos < L
        sorted_ids[pos[ok]] = toks[ok]
    return sorted_ids, eids, np.array([npad], dtype=np.int32)


def fused(s: LruState, topk, max_distinct: int, max_inserts: int, bs: int = 16,
          L: int | None = None, NB: int | None = None):
    """One ``lru_fused_k`` call (r4d_lru.hip:418-575).

    Returns (sorted_hot, eids_hot, npad_hot, sorted_cold, eids_cold, npad_cold)."""
    ids = np.asarray(topk, dtype=np.int64).ravel()
    mk = int(ids.size)
    if L is None or NB is None:
        L, NB = align_sizes(mk, s.E, bs)
    manage(s, ids, max_distinct, max_inserts)
    E, S = s.E, s.S
    valid = (ids >= 0) & (ids < E)
    sl = np.full(mk, -1, dtype=np.int64)
    sl[valid] = s.table[ids[valid]]
    hot = valid & (sl >= 0) & (sl < S)            # (unsigned)s < (unsigned)S, :524
    cold = valid & ~hot
    kh = np.where(hot, sl, -1)
    kc = np.where(cold, ids, -1)
    h = _bucket_align(kh, S, bs, mk, L, NB)
    c = _bucket_align(kc, E, bs, mk, L, NB)
    return (*h, *c)


def moe_align_block_size(topk, bs: int, num_experts: int, expert_map):
    """vLLM ``moe_align_block_size(topk, bs, E, expert_map, ignore_invalid_experts=True)``
    with a stable in-bucket order (semantics as stated at r4d_lru.hip:311-327)."""
    ids = np.asarray(topk, dtype=np.int64).ravel()
    mk = int(ids.size)
    L, NB = align_sizes(mk, num_experts, bs)
    emap = np.asarray(expert_map, dtype=np.int64)
    valid = (ids >= 0) & (ids < num_experts)
    mapped = np.full(mk, -1, dtype=np.int64)
    mapped[valid] = emap[ids[valid]]
    return _bucket_align(mapped, num_experts, bs, mk, L, NB)


def gather_expected(dst: list, src: list, slab_bytes: list, miss: np.ndarray, n_miss: int):
    """``lru_gather_k`` (r4d_lru.hip:271-301): slab e of every source -> slot sl of its
    destination for each of the first ``n_miss`` (expert, slot) pairs."""
    pairs = np.asarray(miss).reshape(-1, 2)[:n_miss]
    for d, sv, b in zip(dst, src, slab_bytes):
        for e, sl in pairs.tolist():
            d[sl * b:(sl + 1) * b] = sv[e * b:(e + 1) * b]
    return dst


def residency_audit(slot_expert, dst: list, src: list, slab_bytes: list) -> list[tuple[int, int]]:
    """(slot, buffer) pairs whose bytes differ from the slab of the expert the slot claims:
    the residency audit of tests/lru/test_slots_prod.py (every occupied slot, every buffer)."""
    bad = []
    for sl, e in enumerate(np.asarray(slot_expert).tolist()):
        if e < 0:
            continue
        for i, (d, sv, b) in enumerate(zip(dst, src, slab_bytes)):
            if not np.array_equal(np.asarray(d[sl * b:(sl + 1) * b]), np.asarray(sv[e * b:(e + 1) * b])):
                bad.append((sl, i))
    return bad


def state_digest(s: LruState) -> int:
    """64-bit digest of every field the reference's tests compare after a step
    (tests/lru/test_lru.py:124-137): table, map_cold, slot_expert, slot_stamp, step,
    n_miss and the first n_miss (expert, slot) pairs."""
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(s.table, dtype=np.int32).tobytes())
    h.update(np.ascontiguousarray(s.map_cold, dtype=np.int32).tobytes())
    h.update(np.ascontiguousarray(s.slot_expert, dtype=np.int32).tobytes())
    h.update(np.ascontiguousarray(s.slot_stamp, dtype=np.int64).tobytes())
    h.update(np.int64(s.step).tobytes())
    h.update(np.int32(s.n_miss).tobytes())
    h.update(np.ascontiguousarray(np.asarray(s.miss).reshape(-1, 2)[:s.n_miss],
                                  dtype=np.int32).tobytes())
    return int.from_bytes(h.digest()[:8], "little", signed=True)


def check_invariants(s: LruState) -> list[str]:
    """Complementarity and bijection (tests/lru/test_lru.py:138-145)."""
    bad = []
    t, c, se = s.table, s.map_cold, s.slot_expert
    ar = np.arange(s.E)
    if not (((t >= 0) & (c == -1)) | ((t < 0) & (c == ar))).all():
        bad.append("table/map_cold are not complementary")
    live = se[se >= 0]
    if len(np.unique(live)) != len(live):
        bad.append("duplicate expert in slots")
    if not (t[live] == np.nonzero(se >= 0)[0]).all():
        bad.append("table/slot mismatch")
    return bad


# ---- seeded routing generators (tests/lru/test_lru.py:178-197, test_fused.py:266-277) ----

def zipf_p(E: int, s: float = 1.1) -> np.ndarray:
    p = np.arange(1, E + 1, dtype=float) ** -s
    return p / p.sum()


def zipf_rows(rng, E: int, rows: int, topk: int = 10, s: float = 1.1) -> np.ndarray:
    p = zipf_p(E, s)
    return np.stack([rng.choice(E, size=topk, replace=False, p=p) for _ in range(rows)])


SUITES = {
    # name: (E, S, nsteps, max_distinct, max_inserts)
    "tiny-churn": (32, 8, 200, 8, 8),
    "skewed-512": (512, 257, 300, 128, 64),
    "insert-capped": (128, 32, 150, 128, 4),
    "read-through": (128, 32, 60, 8, 16),
    "padded-rows": (64, 16, 120, 64, 16),
}


def suite_gen(name: str):
    """The per-step routing generator of each policy suite (tests/lru/test_lru.py:178-197)."""
    if name == "tiny-churn":
        return lambda rng, n: rng.choice(32, size=(2, 5), replace=True)
    if name == "skewed-512":
        return lambda rng, n: zipf_rows(rng, 512, 5, 10, 1.1)
    if name == "insert-capped":
        return lambda rng, n: rng.choice(128, size=(8, 10), replace=True)
    if name == "read-through":
        return lambda rng, n: rng.choice(128, size=(16, 10), replace=True)
    if name == "padded-rows":
        def padded(rng, n):
            a = rng.choice(64, size=(4, 10), replace=True)
            a[2:] = -1
            return a
        return padded
    raise KeyError(name)


def suite_start(name: str, seed: int = 0):
    """(rng, state) at the start of a suite: hot set drawn first from the same rng
    (tests/lru/test_lru.py:151-153)."""
    E, S, _, _, maxi = SUITES[name]
    rng = np.random.default_rng(seed)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    return rng, warm_state(E, S, hot, cap=maxi)

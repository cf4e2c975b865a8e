"""GPU parity of the device LRU (librlu.so through its C ABI / the torch custom ops) against
the CPU oracle and the reference's own numpy model (golden digests): every state field is
compared bit-exact after EVERY step, as tests/lru/test_lru.py does; the fused kernel's align
outputs exactly (stable in-bucket order) and against vLLM's moe_align_block_size when that
op loads; graph replay; gather bytes from pinned host memory; a graph of many layers replayed
with changing routing under a residency audit of every slot."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, load_pkg
from oracle import lru_oracle as LO

pytestmark = pytest.mark.gpu
P = load_pkg()
DEV = "cuda"


def to_dev(st: LO.LruState, cap: int):
    miss = np.full((max(cap, 1), 2), -1, dtype=np.int32)
    st.miss = miss.copy()
    t = dict(table=torch.tensor(st.table, device=DEV), map_cold=torch.tensor(st.map_cold, device=DEV),
             slot_expert=torch.tensor(st.slot_expert, device=DEV),
             slot_stamp=torch.tensor(st.slot_stamp, device=DEV),
             routed=torch.tensor(st.routed, device=DEV),
             step=torch.tensor([st.step], dtype=torch.int64, device=DEV),
             miss=torch.tensor(miss, device=DEV), n_miss=torch.zeros(1, dtype=torch.int32, device=DEV))
    return t


ORDER = ["table", "map_cold", "slot_expert", "slot_stamp", "routed", "step", "miss", "n_miss"]


def compare(t, st: LO.LruState, tag: str):
    got = {k: v.cpu().numpy() for k, v in t.items()}
    want = dict(table=st.table, map_cold=st.map_cold, slot_expert=st.slot_expert,
                slot_stamp=st.slot_stamp, routed=st.routed, step=np.array([st.step]),
                miss=st.miss, n_miss=np.array([st.n_miss]))
    for k in ORDER:
        assert np.array_equal(got[k].reshape(-1), np.asarray(want[k]).reshape(-1)), f"{tag}: {k}"


def run_manage(t, ids, md, maxi):
    ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int32), device=DEV)
    torch.ops.vllm.r4d_lru_manage(ids_t, *[t[k] for k in ORDER], md, maxi)


@pytest.mark.parametrize("name", list(LO.SUITES))
def test_manage_suites_every_step(cuda, name):
    g = golden("lru_reference.npz")
    E, S, nsteps, md, maxi = LO.SUITES[name]
    rng, st = LO.suite_start(name, seed=0)
    t = to_dev(st, maxi)
    ids_all = g[f"{name}/ids"]
    for n in range(nsteps):
        ids = ids_all[n]
        LO.manage(st, ids, md, maxi)
        run_manage(t, ids, md, maxi)
        torch.cuda.synchronize()
        compare(t, st, f"{name} step {n}")
        assert LO.state_digest(st) == g[f"{name}/digest"][n]


def _case(g, i):
    k = f"case{i}"
    E, S, mk, maxi, md = (int(v) for v in g[f"{k}/params"])
    st = LO.LruState(g[f"{k}/table"].copy(), g[f"{k}/map_cold"].copy(), g[f"{k}/slot_expert"].copy(),
                     g[f"{k}/slot_stamp"].copy(), int(g[f"{k}/step"][0]))
    return st, g[f"{k}/ids"], md, maxi


@pytest.mark.parametrize("i", range(19))
def test_manage_and_fused_victim_cases(cuda, i):
    """test_victim_equiv.py's 19 cases, both kernels, full state exact."""
    g = golden("lru_reference.npz")
    st, ids, md, maxi = _case(g, i)
    st2 = st.copy()
    t = to_dev(st, maxi)
    run_manage(t, ids, md, maxi)
    LO.manage(st, ids, md, maxi)
    torch.cuda.synchronize()
    compare(t, st, f"manage case {i}")
    assert LO.state_digest(st) == g[f"case{i}/digest"][0]
    # fused from the same pristine state
    t2 = to_dev(st2, maxi)
    ref = LO.fused(st2, ids, md, maxi, 16)
    mk = len(ids)
    Lh, NB = LO.align_sizes(mk, st2.E, 16)
    out = [torch.full((Lh,), -7, dtype=torch.int32, device=DEV), torch.full((NB,), -7, dtype=torch.int32, device=DEV),
           torch.full((1,), -7, dtype=torch.int32, device=DEV), torch.full((Lh,), -7, dtype=torch.int32, device=DEV),
           torch.full((NB,), -7, dtype=torch.int32, device=DEV), torch.full((1,), -7, dtype=torch.int32, device=DEV)]
    torch.ops.vllm.r4d_lru_fused(torch.as_tensor(ids, device=DEV), *[t2[k] for k in ORDER], *out, md, maxi, 16)
    torch.cuda.synchronize()
    compare(t2, st2, f"fused case {i}")
    for j, (o, r) in enumerate(zip(out, ref)):
        assert np.array_equal(o.cpu().numpy(), r), f"case {i} align output {j}"


def test_read_through_inserts_nothing(cuda):
    g = golden("lru_reference.npz")
    st, ids, md, maxi = _case(g, 0)
    t = to_dev(st, maxi)
    run_manage(t, ids, 0, maxi)
    LO.manage(st, ids, 0, maxi)
    torch.cuda.synchronize()
    compare(t, st, "read-through")
    assert int(t["n_miss"].item()) == 0


@pytest.mark.parametrize("rows", [1, 4, 20, 40, 205])
def test_fused_zipf_geometries(cuda, rows):
    """test_fused.py's mk sweep (1..205 rows x top-10): mk above 256 takes the reference's
    atomic-cursor branch; here the order is stable for every mk and must equal the oracle."""
    E, S = 512, 257
    rng = np.random.default_rng(7)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    st = LO.warm_state(E, S, hot, stamps=rng.permutation(S) + 1, step=S, cap=64)
    t = to_dev(st, 64)
    md = max(1, int(S * 0.5))
    for n in range(6):
        ids = LO.zipf_rows(rng, E, rows, 10).ravel().astype(np.int32)
        ref = LO.fused(st, ids, md, 64, 16)
        mk = len(ids)
        Lh, NB = LO.align_sizes(mk, E, 16)
        out = [torch.full((x,), -7, dtype=torch.int32, device=DEV) for x in (Lh, NB, 1, Lh, NB, 1)]
        torch.ops.vllm.r4d_lru_fused(torch.as_tensor(ids, device=DEV), *[t[k] for k in ORDER], *out, md, 64, 16)
        torch.cuda.synchronize()
        compare(t, st, f"rows={rows} step {n}")
        for j, (o, r) in enumerate(zip(out, ref)):
            assert np.array_equal(o.cpu().numpy(), r), f"rows={rows} step {n} output {j}"


def test_fused_matches_vllm_moe_align(cuda):
    """Where vLLM's moe_align_block_size loads on this box, the reference test's own
    comparison (tests/lru/test_fused.py:133-173): npad and expert_ids exact, sorted ids as a
    multiset per expert, padding exactly mk."""
    try:
        from vllm.model_executor.layers.fused_moe.moe_align_block_size import moe_align_block_size
        probe = torch.zeros(10, dtype=torch.int32, device=DEV).view(1, 10)
        moe_align_block_size(probe, 16, 512, torch.zeros(512, dtype=torch.int32, device=DEV),
                             ignore_invalid_experts=True)
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM moe_align_block_size unavailable here: {type(e).__name__}")
    E, S = 512, 257
    rng = np.random.default_rng(3)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    st = LO.warm_state(E, S, hot, stamps=rng.permutation(S) + 1, step=S, cap=64)
    lay = P.lru.LruLayer(**{k: v for k, v in to_dev(st, 64).items()}, max_distinct=128, max_inserts=64)
    for rows in (5, 20, 60):
        ids = torch.as_tensor(LO.zipf_rows(rng, E, rows, 10).astype(np.int32), device=DEV)
        snap = lay.snapshot()
        hot_out, cold_out = lay.fused(ids)
        after = lay.snapshot()
        lay.restore(snap)
        lay.manage(ids)
        ref_hot = moe_align_block_size(ids, 16, E, lay.table, ignore_invalid_experts=True)
        ref_cold = moe_align_block_size(ids, 16, E, lay.map_cold, ignore_invalid_experts=True)
        torch.cuda.synchronize()
        mk = ids.numel()
        for (gs, ge, gn), (rs, re_, rn) in ((hot_out, ref_hot), (cold_out, ref_cold)):
            assert int(gn.item()) == int(rn.item())
            assert torch.equal(ge, re_)
            n = int(gn.item())
            gsn, gen = gs.cpu().numpy(), ge.cpu().numpy()
            rsn, ren = rs.cpu().numpy(), re_.cpu().numpy()

            def by(s_, e_):
                d = {}
                for b in range(n // 16):
                    d.setdefault(int(e_[b]), []).extend(s_[b * 16:(b + 1) * 16].tolist())
                return {k: sorted(v) for k, v in d.items()}
            assert by(gsn, gen) == by(rsn, ren)
            assert (gsn[n:] == mk).all()
        lay.restore(after)


def test_graph_replay_equals_eager(cuda):
    """12 replays of a captured fused step with changing routing == 12 eager calls, state
    and outputs; then the zero-insert (stale output) hazard (tests/lru/test_fused.py:296-364)."""
    E, S, mk = 512, 257, 50
    rng = np.random.default_rng(5)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    stamps = rng.permutation(S) + 1
    routes = [LO.zipf_rows(rng, E, 5, 10).ravel().astype(np.int32) for _ in range(12)]

    def fresh():
        return P.lru.LruLayer(**to_dev(LO.warm_state(E, S, hot, stamps=stamps, step=S, cap=64), 64),
                              max_distinct=128, max_inserts=64)
    lay = fresh()
    ids_static = torch.zeros(mk, dtype=torch.int32, device=DEV)
    out = lay.new_align_outputs(mk)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ids_static.copy_(torch.as_tensor(routes[0], device=DEV))
        lay.fused(ids_static, out)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        lay.fused(ids_static, out)
    torch.cuda.synchronize()
    lay.restore(fresh().snapshot())
    eager = fresh()
    for n, r in enumerate(routes):
        ids_static.copy_(torch.as_tensor(r, device=DEV))
        gr.replay()
        o2 = eager.new_align_outputs(mk)
        eager.fused(torch.as_tensor(r, device=DEV), o2)
        torch.cuda.synchronize()
        for i in range(6):
            assert torch.equal(out[i], o2[i]), f"replay {n} output {i}"
        for k in ORDER:
            assert torch.equal(getattr(lay, k), getattr(eager, k)), f"replay {n} {k}"
    # zero inserts: the same routing again must still rewrite every output
    ids_static.copy_(torch.as_tensor(routes[-1], device=DEV))
    for i in range(6):
        out[i].fill_(-99)
    gr.replay()
    torch.cuda.synchronize()
    assert int(lay.n_miss.item()) == 0
    assert all(int((o == -99).sum()) == 0 for o in out), "stale outputs after a zero-insert step"


def test_gather_bytes_from_pinned_host(cuda):
    """40 driven steps of manage + gather (tests/lru/test_lru.py:211-258): every installed
    slot's six slabs byte-identical to the pinned host source; reduced slab sizes."""
    E, S = 512, 257
    sizes = [8192, 4096, 512, 64, 256, 32]
    g = torch.Generator().manual_seed(1)
    src = [torch.randint(0, 256, (E * b,), dtype=torch.uint8, generator=g).pin_memory() for b in sizes]
    dst = [torch.zeros(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
    rng = np.random.default_rng(3)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    st = LO.warm_state(E, S, hot, cap=64)
    lay = P.lru.LruLayer(**to_dev(st, 64), max_distinct=128, max_inserts=64)
    rng = np.random.default_rng(11)
    dst2 = [d.view(S, b) for d, b in zip(dst, sizes)]
    src2 = [s.view(E, b) for s, b in zip(src, sizes)]
    for n in range(40):
        ids = np.stack([rng.choice(512, size=10, replace=False) for _ in range(5)]).ravel()
        LO.manage(st, ids, 128, 64)
        lay.manage(torch.as_tensor(ids.astype(np.int32), device=DEV))
        lay.gather(dst2, src2, chunks=16, lanes=64)
        torch.cuda.synchronize()
        nm = int(lay.n_miss.item())
        assert nm == st.n_miss
        for e, sl in st.miss[:nm].tolist():
            for i, b in enumerate(sizes):
                assert torch.equal(dst[i][sl * b:(sl + 1) * b].cpu(), src[i][e * b:(e + 1) * b]), (n, e, sl, i)


def test_graph_of_layers_replayed_with_changing_routing(cuda):
    """tests/lru/test_graph_lru.py and test_slots_prod.py together: L layers of (manage +
    gather) captured once and replayed 20 times with fresh Zipf routing written into the
    captured id buffers; after every replay each layer's state equals the oracle's, the
    table / slot invariants hold, the cache has moved, and every occupied slot's six slabs hold
    the bytes of the expert it claims (pinned host sources, UVA gather)."""
    L, E, S = 12, 512, 257
    sizes = [64, 32, 16, 16, 48, 16]
    g = torch.Generator().manual_seed(7)
    rng = np.random.default_rng(17)
    layers, states, srcs, dsts = [], [], [], []
    for _ in range(L):
        src = [torch.randint(0, 256, (E * b,), dtype=torch.uint8, generator=g).pin_memory() for b in sizes]
        hot = sorted(rng.choice(E, S, replace=False).tolist())
        stamps = rng.permutation(S) + 1
        st = LO.warm_state(E, S, hot, stamps=stamps, step=S, cap=64)
        lay = P.lru.LruLayer(**to_dev(st, 64), max_distinct=128, max_inserts=64)
        dst = [torch.empty(S * b, dtype=torch.uint8, device=DEV) for b in sizes]
        for d, sv, b in zip(dst, src, sizes):               # the warm set is resident
            d.view(S, b).copy_(sv.view(E, b)[torch.as_tensor(hot)].to(DEV))
        layers.append(lay), states.append(st), srcs.append(src), dsts.append(dst)
    ids = [torch.zeros(50, dtype=torch.int32, device=DEV) for _ in range(L)]

    def step():
        for lay, i, d, sv in zip(layers, ids, dsts, srcs):
            lay.manage(i)
            lay.gather([x.view(S, b) for x, b in zip(d, sizes)], [x.view(E, b) for x, b in zip(sv, sizes)],
                       chunks=8, lanes=16)
    snaps = [lay.snapshot() for lay in layers]
    dsnap = [[x.clone() for x in d] for d in dsts]          # the warm-up's gathers are undone too
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()                                               # warm-up (then restored)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    for lay, sn, d, ds in zip(layers, snaps, dsts, dsnap):
        lay.restore(sn)
        for x, y in zip(d, ds):
            x.copy_(y)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        step()
    torch.cuda.synchronize()
    for lay, sn in zip(layers, snaps):
        lay.restore(sn)
    first = [st.slot_expert.copy() for st in states]
    for rep in range(20):
        routes = [LO.zipf_rows(rng, E, 5, 10).ravel().astype(np.int32) for _ in range(L)]
        for i, r in zip(ids, routes):
            i.copy_(torch.as_tensor(r, device=DEV))
        gr.replay()
        torch.cuda.synchronize()
        for l in range(L):
            LO.manage(states[l], routes[l], 128, 64)
            compare({k: getattr(layers[l], k) for k in ORDER}, states[l], f"replay {rep} layer {l}")
            assert LO.check_invariants(states[l]) == []
            host = [x.cpu().numpy() for x in dsts[l]]
            assert LO.residency_audit(states[l].slot_expert, host, [x.numpy() for x in srcs[l]], sizes) == [], \
                (rep, l)
    assert any(not np.array_equal(f, st.slot_expert) for f, st in zip(first, states)), "cache never moved"

"""Multi-rank host logic on CPU (gloo, world_size 2), no GPU: the vocab-sharded lm_head combine
of per-shard (max, argmax, logsumexp) equals the unsharded result (ties resolve to the first
global index, mtp.py.diff L223-226); expert-id sharding of the LRU routing; and failure
detection -- a rank that leaves before the collective makes the other rank's combine fail
within the process group's short timeout instead of hanging."""
from __future__ import annotations

import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _combine_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import importlib
    P = importlib.import_module("r9700-lru-expert-cache_b200")
    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(0)
        M, N = 6, 128 * 7
        logits = torch.randn(M, N, generator=g, dtype=torch.float64).float()
        logits[1, 5] = logits[1, 700] = logits[1].max() + 1.0        # tie across shards
        logits[2, 200] = logits[2, 201] = logits[2].max() + 2.0      # tie inside a shard
        r0, r1 = P.sharded.vocab_shards(N, world)[rank]
        loc = logits[:, r0:r1].double()
        mx, a = loc.max(dim=1)
        lse = torch.logsumexp(loc, dim=1)
        gm, ga, gl = P.sharded.combine_row_stats(mx.float(), a + r0, lse.float())
        rm, ra = logits.double().max(dim=1)
        rl = torch.logsumexp(logits.double(), dim=1)
        ok = (torch.equal(ga, ra) and torch.allclose(gm.double(), rm) and
              torch.allclose(gl.double(), rl, atol=1e-5) and int(ga[1]) == 5 and int(ga[2]) == 200)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def _leaver_worker(rank, world, port, q):
    import sys
    sys.path.insert(0, ROOT)
    import importlib
    P = importlib.import_module("r9700-lru-expert-cache_b200")
    _init(rank, world, port, timeout_s=4)
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()                  # the message is out before the process disappears
        os._exit(0)                      # leaves between steps, no collective in flight
    t0 = time.time()
    try:
        P.sharded.combine_row_stats(torch.zeros(3), torch.zeros(3, dtype=torch.int64), torch.zeros(3))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))


def _run(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + timeout
    while len(out) < world and time.time() < deadline:
        try:
            r, v = q.get(timeout=1)
            out[r] = v
        except Exception:  # noqa: BLE001
            if not any(p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    return out


def test_vocab_shards_partition_on_128_row_blocks():
    import importlib
    P = importlib.import_module("r9700-lru-expert-cache_b200")
    for world in (1, 2, 4, 8):
        sh = P.sharded.vocab_shards(151936, world)
        assert sh[0][0] == 0 and sh[-1][1] == 151936
        sizes = [(b - a) // 128 for a, b in sh]
        assert all(a % 128 == 0 for a, _ in sh) and max(sizes) - min(sizes) <= 1
        assert all(sh[i][1] == sh[i + 1][0] for i in range(world - 1))
    assert sorted({(b - a) // 128 for a, b in P.sharded.vocab_shards(151936, 8)}) == [148, 149]


def test_combine_two_ranks_gloo():
    out = _run(_combine_worker)
    assert out == {0: True, 1: True}, out


def test_rank_that_leaves_fails_the_collective_fast():
    out = _run(_leaver_worker, timeout=90)
    assert out.get(1) == "left", out
    assert isinstance(out.get(0), str) and out[0].startswith("error after"), out


def test_expert_id_sharding_matches_per_shard_oracle():
    """Each rank's cache sees routing shifted by -rank*E_local; ids outside [0, E_local) are
    ignored by the manager (r4d_lru.hip:218), so the sharded run equals the oracle run on the
    ids each shard owns."""
    import importlib
    from oracle import lru_oracle as LO
    P = importlib.import_module("r9700-lru-expert-cache_b200")
    E, world = 512, 8
    e_loc = E // world
    rng = np.random.default_rng(4)
    states = [LO.warm_state(e_loc, 32, sorted(rng.choice(e_loc, 32, replace=False).tolist()), cap=16)
              for _ in range(world)]
    ref = [s.copy() for s in states]
    for _ in range(20):
        ids = LO.zipf_rows(rng, E, 5, 10).ravel().astype(np.int32)
        for r in range(world):
            loc = P.sharded.local_expert_ids(torch.as_tensor(ids), r, e_loc).numpy()
            LO.manage(states[r], loc, 16, 16)
            own = ids[(ids >= r * e_loc) & (ids < (r + 1) * e_loc)] - r * e_loc
            LO.manage(ref[r], own, 16, 16)
            assert LO.state_digest(states[r]) == LO.state_digest(ref[r])


def test_combine_poisoned_shard_gives_nan_and_minus_one():
    """A shard whose statistics are poisoned (NaN max, as a head whose bounded wait ran out
    reports them) makes the combined max / logsumexp NaN and the argmax -1, the rule the CUDA
    combines follow; finite shards combine as usual (ties go to the first shard)."""
    import importlib
    import torch
    P = importlib.import_module("r9700-lru-expert-cache_b200")
    a = (torch.tensor([1.0, 2.0]), torch.tensor([3, 4]), torch.tensor([1.5, 2.5]))
    b = (torch.tensor([float("nan"), 2.0]), torch.tensor([-1, 9]), torch.tensor([float("nan"), 2.1]))
    mx, arg, lse = P.sharded.combine_row_stats_local([a, b])
    assert torch.isnan(mx[0]) and torch.isnan(lse[0]) and int(arg[0]) == -1
    assert float(mx[1]) == 2.0 and int(arg[1]) == 4 and torch.isfinite(lse[1])

"""The peer-memory combine kernel (b200_p2p_combine_row_stats) on one GPU, through the C ABI.

world = 1: the kernel stores its rows into its own buffer and reads them back. world = 2, 8
and 12: the other ranks' rows are written into the buffer by the test before the call, as the
tagged words those ranks' stores leave there, so one launch runs the whole combine and no
kernel waits on another. Both match the NCCL path's combine (b200_combine_row_stats over the
float64 triples) bit for bit, over successive calls that alternate the buffer parity and
advance the tag; every token keeps its own call counter. A rank whose rows never arrive, or whose rows carry a stale call's tag, makes the bounded
wait give up after about a second with error word 2, and the context stays usable."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu
P = load_pkg()
L = P._lib
WORDS = 4                      # per token row: max bits, argmax low, argmax high, lse bits


def _stats(M, seed, dev):
    g = torch.Generator().manual_seed(seed)
    mx = torch.randn(M, generator=g) * 4
    lse = mx + torch.rand(M, generator=g) * 3
    arg = torch.randint(0, 151936, (M,), generator=g, dtype=torch.int64)
    arg[::7] += 1 << 33                                   # exercises the argmax high word
    return mx.to(dev), arg.to(dev), lse.to(dev)


def _tagged(mx, arg, lse, tag):
    """The four words one rank stores per token row at the call whose tag is `tag`."""
    t = np.uint64(tag) << np.uint64(32)
    lo = np.uint64(0xFFFFFFFF)
    a = arg.cpu().numpy().view(np.uint64)
    w = np.stack([mx.cpu().numpy().view(np.uint32).astype(np.uint64) | t, (a & lo) | t,
                  (a >> np.uint64(32)) | t, lse.cpu().numpy().view(np.uint32).astype(np.uint64) | t], axis=1)
    return torch.from_numpy(np.ascontiguousarray(w).view(np.int64))


def _outputs(M, dev):
    return (torch.empty(M, device=dev), torch.empty(M, device=dev, dtype=torch.int64),
            torch.empty(M, device=dev))


def _combine_ref(lib, ranks, dev):
    """The NCCL path's combine on the same rows: float64 triples [world][M][3]."""
    gathered = torch.stack([torch.stack([m.double(), a.double(), l.double()], dim=1) for m, a, l in ranks])
    M = gathered.shape[1]
    out = _outputs(M, dev)
    assert lib.b200_combine_row_stats(L.ptr(gathered), len(ranks), M, L.ptr(out[0]), L.ptr(out[1]),
                                      L.ptr(out[2]), L.stream_ptr()) == 0
    return out


def _call(lib, rows, M, M_cap, peers, rank, world, counters, dev):
    out = _outputs(M, dev)
    mx, arg, lse = rows
    rc = lib.b200_p2p_combine_row_stats(L.ptr(mx), L.ptr(arg), L.ptr(lse), M, M_cap, L.ptr(peers), rank, world,
                                        L.ptr(counters), L.ptr(out[0]), L.ptr(out[1]), L.ptr(out[2]),
                                        L.stream_ptr())
    assert rc == 0
    return out


def _same(a, b):
    assert torch.equal(a[0].view(torch.int32), b[0].view(torch.int32))
    assert torch.equal(a[1], b[1])
    assert torch.equal(a[2].view(torch.int32), b[2].view(torch.int32))


def _buffer(lib, world, M_cap, dev):
    nbytes = int(lib.b200_p2p_combine_bytes(world, M_cap))
    assert nbytes == 2 * world * M_cap * WORDS * 8
    buf = torch.zeros(nbytes // 8, device=dev, dtype=torch.int64)
    peers = torch.tensor([buf.data_ptr()] * world, device=dev, dtype=torch.int64)
    return buf, buf.view(2, world, M_cap, WORDS), peers, torch.zeros(M_cap, device=dev, dtype=torch.int64)


@pytest.mark.parametrize("M,M_cap", [(64, 64), (40, 64), (200, 256)])
def test_single_rank_round_trip(cuda, M, M_cap):
    lib = L.lmhead()
    _, _, peers, counter = _buffer(lib, 1, M_cap, cuda)
    for k in range(3):
        rows = _stats(M, 10 + k, cuda)
        got = _call(lib, rows, M, M_cap, peers, 0, 1, counter, cuda)
        _same(got, _combine_ref(lib, [rows], cuda))
    torch.cuda.synchronize()
    assert torch.all(counter[:M] == 3) and torch.all(counter[M:] == 0)     # per-token counters
    assert lib.b200_lmhead_error(1) == 0


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (8, 5), (12, 3), (12, 10)])
def test_several_ranks_in_one_launch(cuda, world, rank):
    """This rank's rows come from its own stores; every other rank's rows were placed by the
    test with this call's tag, in the slot that rank's stores fill. 12 ranks take the kernel's
    second chunk of source ranks."""
    lib = L.lmhead()
    M, M_cap = 64, 64
    _, view, peers, counter = _buffer(lib, world, M_cap, cuda)
    for k in range(4):
        ranks = [_stats(M, 100 * (r + 1) + k, cuda) for r in range(world)]
        if k == 2:
            for r in range(world):
                ranks[r][0][7] = ranks[rank][0][7]        # equal maxima: the lowest rank wins
        for r in range(world):
            if r != rank:
                view[k & 1, r, :M] = _tagged(*ranks[r], k + 1).to(cuda)
        got = _call(lib, ranks[rank], M, M_cap, peers, rank, world, counter, cuda)
        _same(got, _combine_ref(lib, ranks, cuda))
        assert torch.equal(view[k & 1, rank, :M].cpu(), _tagged(*ranks[rank], k + 1))
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 0


def test_missing_or_stale_rows_time_out(cuda):
    """Rank 1's slot holds nothing at the first call and a stale tag at the second: each wait
    ends at its limit with error word 2; a correct call afterwards still succeeds."""
    lib = L.lmhead()
    world, M, M_cap = 2, 8, 8
    _, view, peers, counter = _buffer(lib, world, M_cap, cuda)
    rows = _stats(M, 7, cuda)
    _call(lib, rows, M, M_cap, peers, 0, world, counter, cuda)            # call 0: slot empty
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 2
    view[1, 1, :M] = _tagged(*rows, 1).to(cuda)                            # call 1 wants tag 2
    _call(lib, rows, M, M_cap, peers, 0, world, counter, cuda)
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 2
    view[0, 1, :M] = _tagged(*rows, 3).to(cuda)                            # call 2, tag 3: arrives
    got = _call(lib, rows, M, M_cap, peers, 0, world, counter, cuda)
    _same(got, _combine_ref(lib, [rows, rows], cuda))
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 0 and torch.all(counter == 3)


def test_empty_call_does_not_count(cuda):
    """Calls with M > 0, M == 0, M > 0: the empty call launches nothing and leaves the call
    counter alone, so the third call still uses the parity and tag that every rank expects."""
    lib = L.lmhead()
    world, rank, M, M_cap = 2, 0, 16, 16
    _, view, peers, counter = _buffer(lib, world, M_cap, cuda)
    for k, m in enumerate((M, 0, M)):
        if m == 0:
            rc = lib.b200_p2p_combine_row_stats(None, None, None, 0, M_cap, L.ptr(peers), rank, world,
                                                L.ptr(counter), None, None, None, L.stream_ptr())
            assert rc == 0
            continue
        call = int(counter[0].item())
        ranks = [_stats(M, 300 + 10 * k + r, cuda) for r in range(world)]
        view[call & 1, 1, :M] = _tagged(*ranks[1], call + 1).to(cuda)
        got = _call(lib, ranks[rank], M, M_cap, peers, rank, world, counter, cuda)
        _same(got, _combine_ref(lib, ranks, cuda))
    torch.cuda.synchronize()
    assert torch.all(counter == 2)
    assert lib.b200_lmhead_error(1) == 0

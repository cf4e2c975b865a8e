"""The vocabulary-sharded heads with the peer-memory combine fused into their last kernel
(b200_fp8_lmhead_combined, b200_w4_lmhead_combined), on one GPU through the C ABI.

world = 1: the head stores its rows into its own buffer and reads them back; the result equals
the plain head followed by the standalone combine, bit for bit. world = 2: "rank 1"'s rows are
the plain head's statistics on the other shard, placed in the buffer by the test as the tagged
words that rank's stores leave there, so one launch set runs the whole exchange and no kernel
waits on another. The global (max, argmax, logsumexp) equals the NCCL path's combine of the two
shards' statistics bit for bit, and the unsharded head's within 1e-4 with the argmax exact. Both
the GEMV (M <= 8) and the tcgen05 (9 <= M <= 64) paths, successive calls (buffer parity and
tags advance per token), and the poisoning of the statistics while the device error word is
set: a row that never arrives gives NaN / -1 instead of a plausible value."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu
P = load_pkg()
L = P._lib
F8 = P.fp8_target_lmhead
W4 = P.draft_w4_lmhead
WORDS = 4


def _tagged(mx, arg, lse, tag):
    t = np.uint64(tag) << np.uint64(32)
    lo = np.uint64(0xFFFFFFFF)
    a = arg.cpu().numpy().view(np.uint64)
    w = np.stack([mx.cpu().numpy().view(np.uint32).astype(np.uint64) | t, (a & lo) | t,
                  (a >> np.uint64(32)) | t, lse.cpu().numpy().view(np.uint32).astype(np.uint64) | t], axis=1)
    return torch.from_numpy(np.ascontiguousarray(w).view(np.int64))


def _buffer(lib, world, M_cap, dev):
    nbytes = int(lib.b200_p2p_combine_bytes(world, M_cap))
    buf = torch.zeros(nbytes // 8, device=dev, dtype=torch.int64)
    peers = torch.tensor([buf.data_ptr()] * world, device=dev, dtype=torch.int64)
    return buf.view(2, world, M_cap, WORDS), peers, torch.zeros(M_cap, device=dev, dtype=torch.int64)


def _stats(M, dev):
    return (torch.empty(M, device=dev), torch.empty(M, device=dev, dtype=torch.int64), torch.empty(M, device=dev))


def _fp8_combined(lib, x, wq, ws, off, peers, rank, world, counters, M_cap):
    M, K = x.shape
    out = _stats(M, x.device)
    wsp = P._workspace.workspace(x.device)
    rc = lib.b200_fp8_lmhead_combined(L.ptr(x), M, K, L.ptr(wq), L.ptr(ws), wq.shape[0], off, None, wq.shape[0],
                                      L.ptr(out[0]), L.ptr(out[1]), L.ptr(out[2]), None, None, L.ptr(wsp),
                                      wsp.numel(), L.ptr(peers), rank, world, L.ptr(counters), M_cap,
                                      L.stream_ptr())
    assert rc == 0
    return out


def _nccl_combine(lib, parts, dev):
    gathered = torch.stack([torch.stack([m.double(), a.double(), l.double()], dim=1) for m, a, l in parts])
    M = gathered.shape[1]
    out = _stats(M, dev)
    assert lib.b200_combine_row_stats(L.ptr(gathered), len(parts), M, L.ptr(out[0]), L.ptr(out[1]),
                                      L.ptr(out[2]), L.stream_ptr()) == 0
    return out


def _same(a, b):
    assert torch.equal(a[0].view(torch.int32), b[0].view(torch.int32))
    assert torch.equal(a[1], b[1])
    assert torch.equal(a[2].view(torch.int32), b[2].view(torch.int32))


def _fp8_weight(N, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    return F8.pack_fp8_block((torch.randn(N, 2560, device=dev, generator=g) * 0.02).bfloat16())


@pytest.mark.parametrize("M", [5, 40])
def test_fp8_combined_world1(cuda, M):
    lib = L.lmhead()
    wq, ws = _fp8_weight(128 * 21, 3, cuda)
    view, peers, counters = _buffer(lib, 1, 64, cuda)
    for k in range(3):
        x = torch.randn(M, 2560, device=cuda, dtype=torch.bfloat16)
        got = _fp8_combined(lib, x, wq, ws, 0, peers, 0, 1, counters, 64)
        _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
        _same(got, _nccl_combine(lib, [(mx, arg, lse)], cuda))
    torch.cuda.synchronize()
    assert torch.all(counters[:M] == 3) and lib.b200_lmhead_error(1) == 0


@pytest.mark.parametrize("M", [3, 64])
def test_fp8_combined_world2_placed_peer(cuda, M):
    lib = L.lmhead()
    N = 128 * 37
    wq, ws = _fp8_weight(N, 5, cuda)
    (a0, a1), (b0, b1) = P.sharded.vocab_shards(N, 2)
    view, peers, counters = _buffer(lib, 2, 64, cuda)
    for k in range(2):
        x = torch.randn(M, 2560, device=cuda, dtype=torch.bfloat16)
        s1 = F8.fp8_lmhead(x, wq[b0:b1], ws[b0 // 128:b1 // 128], vocab_offset=b0, want_logits=False)[1:]
        view[k & 1, 1, :M] = _tagged(*s1, k + 1).to(cuda)
        got = _fp8_combined(lib, x, wq[a0:a1], ws[a0 // 128:a1 // 128], a0, peers, 0, 2, counters, 64)
        s0 = F8.fp8_lmhead(x, wq[a0:a1], ws[a0 // 128:a1 // 128], vocab_offset=a0, want_logits=False)[1:]
        _same(got, _nccl_combine(lib, [s0, s1], cuda))
        _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
        assert torch.equal(got[1], arg)
        assert (got[0] - mx).abs().max().item() < 1e-4 and (got[2] - lse).abs().max().item() < 1e-4
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 0


@pytest.mark.parametrize("sym", [False, True])
def test_w4_combined_world2_placed_peer(cuda, sym):
    lib = L.lmhead()
    n, M = 1000, 4
    g = torch.Generator(device=cuda).manual_seed(9)
    w = (torch.randn(n, 2560, device=cuda, generator=g) * 0.02).bfloat16()
    x = torch.randn(M, 2560, device=cuda, generator=g).bfloat16()
    pack = W4.pack_w4a16_sym if sym else W4.pack_w4a16
    half = 512                                                     # shards on 16-row strips
    p0, p1 = pack(w[:half]), pack(w[half:])
    view, peers, counters = _buffer(lib, 2, 16, cuda)
    _, m1, a1, l1 = W4.gemm_w4a16_top(x, p1, vocab_offset=half)
    view[0, 1, :M] = _tagged(m1, a1, l1, 1).to(cuda)
    out = _stats(M, cuda)
    wsp = P._workspace.workspace(cuda)
    rc = lib.b200_w4_lmhead_combined(1 if sym else 0, L.ptr(x), 0, M, 2560, L.ptr(p0.wq), L.ptr(p0.wsz), p0.n_pad,
                                     p0.n, 0, None, p0.n_pad, L.ptr(out[0]), L.ptr(out[1]), L.ptr(out[2]),
                                     L.ptr(wsp), wsp.numel(), L.ptr(peers), 0, 2, L.ptr(counters), 16,
                                     L.stream_ptr())
    assert rc == 0
    _, m0, a0, l0 = W4.gemm_w4a16_top(x, p0)
    _same(out, _nccl_combine(lib, [(m0, a0, l0), (m1, a1, l1)], cuda))
    full = pack(w)
    _, mx, arg, lse = W4.gemm_w4a16_top(x, full)
    assert torch.equal(out[1], arg)
    torch.cuda.synchronize()
    assert lib.b200_lmhead_error(1) == 0


def test_missing_peer_poisons_statistics(cuda):
    """Rank 1's rows never arrive: the combined call's statistics are NaN / -1 (not stale
    words) and the error word reads 2; while it is set, a plain head call's statistics are
    poisoned too; once cleared, the same call is correct again."""
    lib = L.lmhead()
    wq, ws = _fp8_weight(128 * 8, 11, cuda)
    view, peers, counters = _buffer(lib, 2, 8, cuda)
    x = torch.randn(8, 2560, device=cuda, dtype=torch.bfloat16)
    got = _fp8_combined(lib, x, wq, ws, 0, peers, 0, 2, counters, 8)
    torch.cuda.synchronize()
    assert torch.all(torch.isnan(got[0])) and torch.all(got[1] == -1) and torch.all(torch.isnan(got[2]))
    _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
    torch.cuda.synchronize()
    assert torch.all(torch.isnan(mx)) and torch.all(arg == -1)
    assert lib.b200_lmhead_error(1) == 2
    _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
    torch.cuda.synchronize()
    assert torch.all(torch.isfinite(mx)) and torch.all(arg >= 0) and lib.b200_lmhead_error(0) == 0

"""Two ranks on two GPUs (skipped with fewer): the vocabulary-sharded FP8 head combined over
NVLink peer memory (P2PCombiner: the standalone combine kernel, and the head with the combine
fused into its last kernel, at the tcgen05 and the GEMV row counts) matches the unsharded
call (argmax exact; max and logsumexp within 1e-4, since the shards split the fp32 block sums
between CTAs differently), repeatedly and inside a CUDA graph; the NCCL all-gather path
agrees too, and so does the sharded W4 draft head with its fused combine. Ranks are spawned processes on
127.0.0.1 with a short process-group timeout, joined with a time limit."""
from __future__ import annotations

import os

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2


def _rank(rank: int, port: int, q) -> None:
    import datetime
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from conftest import load_pkg
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD))
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))
    try:
        P = load_pkg()
        F8 = P.fp8_target_lmhead
        N, K, M = 128 * 53, 2560, 24
        g = torch.Generator(device=dev).manual_seed(11)          # same weights and tokens on both ranks
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).bfloat16()
        wq, ws = F8.pack_fp8_block(w)
        r0, r1 = P.sharded.vocab_shards(N, WORLD)[rank]
        comb = P.sharded.P2PCombiner(64, dev)
        errs = []
        for it in range(3):
            x = torch.randn(M if it != 1 else 5, K, device=dev, dtype=torch.bfloat16, generator=g)
            _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
            _, m_, a_, l_ = F8.fp8_lmhead(x, wq[r0:r1], ws[r0 // 128:r1 // 128], vocab_offset=r0, want_logits=False)
            cm, ca, cl = comb(m_, a_, l_)
            nm, na, nl = P.sharded.combine_row_stats(m_, a_, l_)
            # the head with the combine fused into its last kernel
            _, fm, fa, fl = comb.fp8_head(x, wq[r0:r1], ws[r0 // 128:r1 // 128], r0, want_logits=False)
            torch.cuda.synchronize(dev)
            errs.append((bool(torch.equal(ca, arg)), float((cm - mx).abs().max()), float((cl - lse).abs().max()),
                         bool(torch.equal(na, ca)), float((nl - cl).abs().max())))
            errs.append((bool(torch.equal(fa, arg)), float((fm - mx).abs().max()), float((fl - lse).abs().max()),
                         bool(torch.equal(fa, ca)), float((fl - cl).abs().max())))
        # the W4 draft head, sharded on 16-row strips, combined inside its last kernel
        W4 = P.draft_w4_lmhead
        wd = (torch.randn(1000, K, device=dev, generator=g) * 0.02).bfloat16()
        xd = torch.randn(4, K, device=dev, generator=g).bfloat16()
        s0, s1 = (0, 512) if rank == 0 else (512, 1000)
        _, dm, da, dl = W4.gemm_w4a16_top(xd, W4.pack_w4a16(wd))
        _, wm, wa, wl = comb.w4_head(xd, W4.pack_w4a16(wd[s0:s1]), s0, want_logits=False)
        torch.cuda.synchronize(dev)
        errs.append((bool(torch.equal(wa, da)), float((wm - dm).abs().max()), float((wl - dl).abs().max()),
                     True, 0.0))
        # the same combine inside a CUDA graph, replayed twice
        x = torch.randn(M, K, device=dev, dtype=torch.bfloat16, generator=g)
        _, mx, arg, lse = F8.fp8_lmhead(x, wq, ws, want_logits=False)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            out = comb(*F8.fp8_lmhead(x, wq[r0:r1], ws[r0 // 128:r1 // 128], vocab_offset=r0, want_logits=False)[1:])
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            out = comb(*F8.fp8_lmhead(x, wq[r0:r1], ws[r0 // 128:r1 // 128], vocab_offset=r0, want_logits=False)[1:])
        for _ in range(2):
            gr.replay()
        torch.cuda.synchronize(dev)
        errs.append((bool(torch.equal(out[1], arg)), float((out[0] - mx).abs().max()),
                     float((out[2] - lse).abs().max()), True, 0.0))
        gr.reset()
        del gr
        q.put((rank, errs, int(P._lib.lmhead().b200_lmhead_error(1))))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
def test_two_rank_peer_memory_combine():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    procs = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(WORLD):
            r, errs, err_word = q.get(timeout=240)
            res[r] = (errs, err_word)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
    assert sorted(res) == list(range(WORLD))
    for r, (errs, err_word) in res.items():
        assert err_word == 0, (r, err_word)
        for ok_arg, dmax, dlse, nccl_arg, dn in errs:
            assert ok_arg and dmax < 1e-4 and dlse < 1e-4 and nccl_arg and dn < 1e-6, (r, errs)

"""Multi-GPU layout of the hot path: one process per GPU, torch.distributed for the plumbing.

lm_head (FP8 target or W4 draft): the vocabulary is split on 128-row block boundaries, so a
shard is a contiguous slice of the packed weight and of its block scales (1187 blocks of the
151936-row head -> 149/148 per GPU at 8). Each rank runs the fused GEMV on its shard with
``vocab_offset`` = its first row and gets (max, argmax, logsumexp) per token row; one
all-gather of those 3 numbers per row (a [M, 3] float64 tensor, exact for the index) and a
local combine give the global result:
    gmax = max_r max_r;   argmax = argmax of the first rank attaining gmax (shards are in
    vocabulary order, so this is the first global index: the reference's tie rule,
    mtp.py.diff L223-226);   lse = gmax + log sum_r exp(lse_r - gmax).

Expert cache: experts are split by id, ``experts_per_rank`` each. A rank's cache sees the
routing shifted by ``-rank * experts_per_rank``; ids outside [0, E_local) are ignored by the
kernel (r4d_lru.hip:218), so the shift is the whole partition. No collective: every rank
updates its own slots.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

BLK = 128


def vocab_shards(n_rows: int, world: int, blk: int = BLK) -> list[tuple[int, int]]:
    """Contiguous [r0, r1) row ranges on `blk`-row boundaries, sizes differing by <= 1 block."""
    assert n_rows % blk == 0, n_rows
    nb = n_rows // blk
    out = []
    for r in range(world):
        b0 = (r * nb) // world
        b1 = ((r + 1) * nb) // world
        out.append((b0 * blk, b1 * blk))
    return out


def combine_row_stats_local(parts):
    """Combine per-shard (max fp32 [M], argmax int64 [M], lse fp32 [M]) tuples, given in
    shard (vocabulary) order."""
    mx = torch.stack([p[0].double() for p in parts])        # [R, M]
    ar = torch.stack([p[1].to(torch.int64) for p in parts])
    ls = torch.stack([p[2].double() for p in parts])
    return _combine(mx, ar, ls)


def _combine(mx: torch.Tensor, ar: torch.Tensor, ls: torch.Tensor):
    gmax, _ = mx.max(dim=0)                  # NaN at any rank -> NaN (a poisoned shard)
    first = (mx == gmax.unsqueeze(0)).to(torch.int8).argmax(dim=0)     # first rank at gmax
    arg = ar.gather(0, first.unsqueeze(0)).squeeze(0)
    arg = torch.where(torch.isnan(gmax), torch.full_like(arg, -1), arg)
    lse = gmax + torch.log(torch.exp(ls - gmax.unsqueeze(0)).sum(dim=0))
    return gmax.float(), arg, lse.float()


def pack_row_stats(mx: torch.Tensor, arg: torch.Tensor, lse: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """(max, argmax, lse) of M rows -> one float64 [M, 3] tensor (argmax exact below 2^53) in a
    single kernel (b200_pack_row_stats): the layout the combine exchanges, and a single
    device-to-host copy for a caller that reads the triples on the host."""
    from . import _lib
    _lib.require_cuda("pack_row_stats", mx, arg, lse, out)
    M = mx.numel()
    arg64 = arg if arg.dtype == torch.int64 else arg.to(torch.int64)
    if out is None:
        out = torch.empty(M, 3, dtype=torch.float64, device=mx.device)
    _lib.check(_lib.lmhead().b200_pack_row_stats(_lib.ptr(mx), _lib.ptr(arg64), _lib.ptr(lse), M,
                                                 _lib.ptr(out), _lib.stream_ptr()), "b200_pack_row_stats")
    return out


def combine_row_stats(mx: torch.Tensor, arg: torch.Tensor, lse: torch.Tensor, group=None):
    """All-gather this rank's per-row (max, argmax, lse) and combine: [M, 3] float64 per
    rank (24 B/row) in one collective; every rank returns the global triple. On CUDA the
    pack and the combine are one small kernel each (b200_pack_row_stats /
    b200_combine_row_stats) around NCCL's all-gather, so the step stays three launches."""
    world = dist.get_world_size(group)
    if mx.is_cuda:
        from . import _lib
        lib = _lib.lmhead()
        M = mx.numel()
        arg64 = arg if arg.dtype == torch.int64 else arg.to(torch.int64)
        local = torch.empty(M, 3, dtype=torch.float64, device=mx.device)
        _lib.check(lib.b200_pack_row_stats(_lib.ptr(mx), _lib.ptr(arg64), _lib.ptr(lse), M, _lib.ptr(local),
                                           _lib.stream_ptr()), "b200_pack_row_stats")
        gathered = torch.empty((world, M, 3), dtype=torch.float64, device=mx.device)
        dist.all_gather_into_tensor(gathered, local, group=group)
        gm = torch.empty(M, dtype=torch.float32, device=mx.device)
        ga = torch.empty(M, dtype=torch.int64, device=mx.device)
        gl = torch.empty(M, dtype=torch.float32, device=mx.device)
        _lib.check(lib.b200_combine_row_stats(_lib.ptr(gathered), world, M, _lib.ptr(gm), _lib.ptr(ga),
                                              _lib.ptr(gl), _lib.stream_ptr()), "b200_combine_row_stats")
        return gm, ga, gl
    local = torch.stack([mx.double(), arg.double(), lse.double()], dim=1).contiguous()
    parts = [torch.empty_like(local) for _ in range(world)]     # gloo (host-side tests)
    dist.all_gather(parts, local, group=group)
    gathered = torch.stack(parts)
    return _combine(gathered[:, :, 0], gathered[:, :, 1].to(torch.int64), gathered[:, :, 2])


class P2PCombiner:
    """combine_row_stats over NVLink peer memory, with no NCCL call and no host involvement, so
    it can sit in a CUDA graph. Each rank stores its (max, argmax, lse) rows straight into every
    rank's buffer (torch symmetric memory) as 8-byte words that carry the call's tag beside 32
    data bits, reads all ranks' rows from its own buffer until their tags are this call's
    (bounded) and combines; every token has its own call counter.

    * ``__call__(mx, arg, lse)``: the combine alone, one kernel (b200_p2p_combine_row_stats).
    * ``fp8_head(x, wq, ws, vocab_offset)`` / ``w4_head(x, packed, vocab_offset)``: this
      rank's head on its vocabulary shard with the combine fused into the head's last kernel
      (b200_fp8_lmhead_combined / b200_w4_lmhead_combined); the statistics returned are
      global.

    Every rank must make the same sequence of calls with the same row count M <= M_cap."""

    def __init__(self, M_cap: int, device: torch.device, group=None):
        import torch.distributed._symmetric_memory as symm_mem
        from . import _lib
        self._lib = _lib
        self.lib = _lib.lmhead()
        group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.M_cap = M_cap
        nbytes = int(self.lib.b200_p2p_combine_bytes(self.world, M_cap))
        self.buf = symm_mem.empty(nbytes, dtype=torch.uint8, device=device)
        self.buf.zero_()
        self.handle = symm_mem.rendezvous(self.buf, group)
        ptrs = [self.handle.get_remote_tensor(q, (nbytes,), torch.uint8).data_ptr() for q in range(self.world)]
        self.peers = torch.tensor(ptrs, dtype=torch.int64, device=device)
        self.counters = torch.zeros(M_cap, dtype=torch.int64, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group)                 # every rank's buffer is zero before any rank stores

    def _stats(self, M, dev, stats_out=None):
        if stats_out is not None:
            return stats_out
        return (torch.empty(M, dtype=torch.float32, device=dev), torch.empty(M, dtype=torch.int64, device=dev),
                torch.empty(M, dtype=torch.float32, device=dev))

    def __call__(self, mx: torch.Tensor, arg: torch.Tensor, lse: torch.Tensor):
        L = self._lib
        M = mx.numel()
        arg64 = arg if arg.dtype == torch.int64 else arg.to(torch.int64)
        gm, ga, gl = self._stats(M, mx.device)
        L.check(self.lib.b200_p2p_combine_row_stats(L.ptr(mx), L.ptr(arg64), L.ptr(lse), M, self.M_cap,
                                                    L.ptr(self.peers), self.rank, self.world,
                                                    L.ptr(self.counters), L.ptr(gm), L.ptr(ga), L.ptr(gl),
                                                    L.stream_ptr()),
                "b200_p2p_combine_row_stats")
        return gm, ga, gl

    def fp8_head(self, x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, vocab_offset: int,
                 want_logits: bool = True, out: torch.Tensor | None = None, stats_out: tuple | None = None):
        """(logits of this shard | None, global max, global argmax, global logsumexp)."""
        from . import fp8_target_lmhead as F8
        from ._workspace import workspace
        L = self._lib
        F8._check(x, wq, ws)
        M, K = x.shape
        N = wq.shape[0]
        y = (out if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=x.device)) \
            if want_logits else None
        mx, arg, lse = self._stats(M, x.device, stats_out)
        wsp = workspace(x.device)
        L.check(self.lib.b200_fp8_lmhead_combined(
            L.ptr(x), M, K, L.ptr(wq), L.ptr(ws), N, int(vocab_offset), L.ptr(y), N if y is None else y.stride(0),
            L.ptr(mx), L.ptr(arg), L.ptr(lse), None, None, L.ptr(wsp), wsp.numel(),
            L.ptr(self.peers), self.rank, self.world, L.ptr(self.counters), self.M_cap, L.stream_ptr()),
            "b200_fp8_lmhead_combined")
        L.debug_check("b200_fp8_lmhead_combined")
        return y, mx, arg, lse

    def w4_head(self, x: torch.Tensor, p, vocab_offset: int, want_logits: bool = True,
                stats_out: tuple | None = None):
        """The W4 draft head (PackedW4, either format) on this rank's shard: (logits of this
        shard sliced to p.n | None, global max, global argmax, global logsumexp)."""
        from ._workspace import workspace
        L = self._lib
        L.require_cuda("w4 head", x, p.wq, p.wsz)
        M, K = x.shape
        if K != p.k or x.dtype not in (torch.bfloat16, torch.float16) or not x.is_contiguous():
            raise ValueError("w4 head: x must be a contiguous bf16/f16 [M, K] tensor matching the pack")
        y = torch.empty(M, p.n_pad, dtype=torch.bfloat16, device=x.device) if want_logits else None
        mx, arg, lse = self._stats(M, x.device, stats_out)
        wsp = workspace(x.device)
        L.check(self.lib.b200_w4_lmhead_combined(
            1 if p.sym else 0, L.ptr(x), 0 if x.dtype == torch.bfloat16 else 1, M, K, L.ptr(p.wq), L.ptr(p.wsz),
            p.n_pad, p.n, int(vocab_offset), L.ptr(y), p.n_pad, L.ptr(mx), L.ptr(arg), L.ptr(lse),
            L.ptr(wsp), wsp.numel(), L.ptr(self.peers), self.rank, self.world, L.ptr(self.counters),
            self.M_cap, L.stream_ptr()), "b200_w4_lmhead_combined")
        L.debug_check("b200_w4_lmhead_combined")
        return (y[:, :p.n] if y is not None else None), mx, arg, lse


def shard_fp8_head(wq: torch.Tensor, ws: torch.Tensor, rank: int, world: int):
    """(wq_shard, ws_shard, vocab_offset) for this rank from a packed FP8 head."""
    r0, r1 = vocab_shards(wq.shape[0], world)[rank]
    return wq[r0:r1], ws[r0 // BLK:r1 // BLK], r0


def local_expert_ids(topk_ids: torch.Tensor, rank: int, experts_per_rank: int) -> torch.Tensor:
    """Routing as seen by the cache of `rank`: ids shifted into [0, experts_per_rank) for the
    experts this rank owns; every other id falls outside the range and is ignored."""
    return (topk_ids.to(torch.int32) - rank * experts_per_rank).contiguous()

"""Device-side LRU expert cache: the host-side mirror of the reference's custom ops.

Same op names, argument meaning and error behaviour as the patch that binds librlu
(patches/.../r4d_mxfp4_moe.py.lru.diff L179-354): ``torch.ops.vllm.r4d_lru_manage``,
``torch.ops.vllm.r4d_lru_gather`` and ``torch.ops.vllm.r4d_lru_fused``, each mutating its
state tensors in place and raising ``RuntimeError`` on a non-zero return code. The kernels
are this package's librlu.so (csrc/lru.cu); nothing here computes on the host.

``LruLayer`` holds one MoE layer's eight state buffers with the reference's warm start
(_build_lru, L502-541): slot i holds hot expert i, stamps seeded by profile rank in [1, S]
(or zero), ``step = S``, read-through above ``max(1, int(S * thresh))`` distinct experts.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

BLOCK = 16


def _align_sizes(mk: int, num_experts: int, block_size: int = BLOCK) -> tuple[int, int]:
    """(L, NB) that vLLM's moe_align_block_size allocates for `mk` (token, k) slots
    (r4d_mxfp4_moe.py.lru.diff L278-284)."""
    n = mk + num_experts * (block_size - 1)
    if mk < num_experts:
        n = min(mk * block_size, n)
    return n, (n + block_size - 1) // block_size


def _per_expert_bytes(t: torch.Tensor) -> int:
    return t[0].numel() * t.element_size()


def _device_ptr(t: torch.Tensor) -> int:
    """Device-usable address of `t`: CUDA memory as is, pinned host memory through
    cudaHostGetDevicePointer (the UVA source of the gather)."""
    if t.is_cuda:
        return t.data_ptr()
    if not t.is_pinned():
        raise ValueError("lru gather: a host source must be pinned (UVA)")
    dev = ctypes.c_void_p()
    rc = _lib.rlu().r4d_lru_host_device_pointer(ctypes.c_void_p(t.data_ptr()), ctypes.byref(dev))
    if rc != 0:
        raise RuntimeError(f"cudaHostGetDevicePointer failed rc={rc}")
    return dev.value


def _i32(t: torch.Tensor, name: str) -> None:
    if t.dtype != torch.int32 or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 tensor")


def lru_manage(topk_ids: torch.Tensor, table: torch.Tensor, map_cold: torch.Tensor,
               slot_expert: torch.Tensor, slot_stamp: torch.Tensor, routed: torch.Tensor,
               step: torch.Tensor, miss: torch.Tensor, n_miss: torch.Tensor,
               max_distinct: int, max_inserts: int) -> None:
    """One launch of the manager (r4d_mxfp4_moe.py.lru.diff L226-254)."""
    _i32(topk_ids, "topk_ids")
    _lib.require_cuda("r4d_lru_manage", topk_ids, table, map_cold, slot_expert, slot_stamp,
                      routed, step, miss, n_miss)
    rc = _lib.rlu().r4d_lru_manage(
        _lib.ptr(topk_ids), topk_ids.numel(), table.numel(), slot_expert.numel(),
        max_distinct, max_inserts, _lib.ptr(table), _lib.ptr(map_cold), _lib.ptr(slot_expert),
        _lib.ptr(slot_stamp), _lib.ptr(routed), _lib.ptr(step), _lib.ptr(miss),
        _lib.ptr(n_miss), _lib.stream_ptr())
    if rc != 0:
        raise RuntimeError(f"r4d_lru_manage failed rc={rc}")


def lru_gather(dsts: list[torch.Tensor], srcs: list[torch.Tensor], miss: torch.Tensor,
               n_miss: torch.Tensor, chunks: int, lanes: int) -> None:
    """Copy the six per-expert slabs of every miss into its slot (L265-293)."""
    if len(dsts) != 6 or len(srcs) != 6:
        raise ValueError("lru gather takes exactly six (dst, src) buffer pairs")
    _lib.require_cuda("r4d_lru_gather", *dsts, miss, n_miss)
    args = []
    for d, s in zip(dsts, srcs):
        nb = _per_expert_bytes(s)
        if nb != _per_expert_bytes(d):
            raise ValueError(f"lru gather: slab size mismatch {nb} vs {_per_expert_bytes(d)}")
        args += [ctypes.c_void_p(d.data_ptr()), ctypes.c_void_p(_device_ptr(s)), ctypes.c_long(nb)]
    rc = _lib.rlu().r4d_lru_gather(*args, _lib.ptr(miss), _lib.ptr(n_miss), chunks, lanes,
                                   _lib.stream_ptr())
    if rc != 0:
        raise RuntimeError(f"r4d_lru_gather failed rc={rc} (slab sizes must be 16B multiples)")


def lru_fused(topk_ids: torch.Tensor, table: torch.Tensor, map_cold: torch.Tensor,
              slot_expert: torch.Tensor, slot_stamp: torch.Tensor, routed: torch.Tensor,
              step: torch.Tensor, miss: torch.Tensor, n_miss: torch.Tensor,
              sorted_hot: torch.Tensor, eids_hot: torch.Tensor, npad_hot: torch.Tensor,
              sorted_cold: torch.Tensor, eids_cold: torch.Tensor, npad_cold: torch.Tensor,
              max_distinct: int, max_inserts: int, block_size: int) -> None:
    """Manager + both moe_align_block_size outputs in one launch (L296-337). Every element
    of all six outputs is written on every call (single exit)."""
    _i32(topk_ids, "topk_ids")
    _lib.require_cuda("r4d_lru_fused", topk_ids, table, map_cold, slot_expert, slot_stamp,
                      routed, step, miss, n_miss, sorted_hot, eids_hot, npad_hot, sorted_cold,
                      eids_cold, npad_cold)
    rc = _lib.rlu().r4d_lru_fused(
        _lib.ptr(topk_ids), topk_ids.numel(), table.numel(), slot_expert.numel(),
        max_distinct, max_inserts, _lib.ptr(table), _lib.ptr(map_cold), _lib.ptr(slot_expert),
        _lib.ptr(slot_stamp), _lib.ptr(routed), _lib.ptr(step), _lib.ptr(miss),
        _lib.ptr(n_miss), block_size, sorted_hot.numel(), eids_hot.numel(),
        _lib.ptr(sorted_hot), _lib.ptr(eids_hot), _lib.ptr(npad_hot), _lib.ptr(sorted_cold),
        _lib.ptr(eids_cold), _lib.ptr(npad_cold), _lib.stream_ptr())
    if rc != 0:
        raise RuntimeError(f"r4d_lru_fused failed rc={rc} (E and slots must be <= 1024)")


# ---- torch custom ops under the reference's names --------------------------------------------

_MANAGE_MUT = ["table", "map_cold", "slot_expert", "slot_stamp", "routed", "step", "miss", "n_miss"]


def _register_ops() -> None:
    lib = torch.library
    if hasattr(torch.ops.vllm, "r4d_lru_manage"):      # registered by an earlier import
        return

    @lib.custom_op("vllm::r4d_lru_manage", mutates_args=_MANAGE_MUT)
    def _manage(topk_ids: torch.Tensor, table: torch.Tensor, map_cold: torch.Tensor,
                slot_expert: torch.Tensor, slot_stamp: torch.Tensor, routed: torch.Tensor,
                step: torch.Tensor, miss: torch.Tensor, n_miss: torch.Tensor,
                max_distinct: int, max_inserts: int) -> None:
        lru_manage(topk_ids, table, map_cold, slot_expert, slot_stamp, routed, step, miss,
                   n_miss, max_distinct, max_inserts)

    @lib.custom_op("vllm::r4d_lru_gather", mutates_args=["dsts"])
    def _gather(dsts: list[torch.Tensor], srcs: list[torch.Tensor], miss: torch.Tensor,
                n_miss: torch.Tensor, chunks: int, lanes: int) -> None:
        lru_gather(dsts, srcs, miss, n_miss, chunks, lanes)

    @lib.custom_op("vllm::r4d_lru_fused",
                   mutates_args=_MANAGE_MUT + ["sorted_hot", "eids_hot", "npad_hot",
                                               "sorted_cold", "eids_cold", "npad_cold"])
    def _fused(topk_ids: torch.Tensor, table: torch.Tensor, map_cold: torch.Tensor,
               slot_expert: torch.Tensor, slot_stamp: torch.Tensor, routed: torch.Tensor,
               step: torch.Tensor, miss: torch.Tensor, n_miss: torch.Tensor,
               sorted_hot: torch.Tensor, eids_hot: torch.Tensor, npad_hot: torch.Tensor,
               sorted_cold: torch.Tensor, eids_cold: torch.Tensor, npad_cold: torch.Tensor,
               max_distinct: int, max_inserts: int, block_size: int) -> None:
        lru_fused(topk_ids, table, map_cold, slot_expert, slot_stamp, routed, step, miss,
                  n_miss, sorted_hot, eids_hot, npad_hot, sorted_cold, eids_cold, npad_cold,
                  max_distinct, max_inserts, block_size)


_register_ops()


@dataclass
class LruLayer:
    """One layer's cache state (kernels/lru/README.md:50-57), all on one CUDA device."""
    table: torch.Tensor        # int32 [E]
    map_cold: torch.Tensor     # int32 [E]
    slot_expert: torch.Tensor  # int32 [S]
    slot_stamp: torch.Tensor   # int64 [S]
    routed: torch.Tensor       # uint8 [E]
    step: torch.Tensor         # int64 [1]
    miss: torch.Tensor         # int32 [cap, 2]
    n_miss: torch.Tensor       # int32 [1]
    max_distinct: int
    max_inserts: int

    NAMES = ("table", "map_cold", "slot_expert", "slot_stamp", "routed", "step", "miss", "n_miss")

    @property
    def E(self) -> int:
        return self.table.numel()

    @property
    def S(self) -> int:
        return self.slot_expert.numel()

    @classmethod
    def warm(cls, hot: list[int] | torch.Tensor, num_experts: int, device,
             profile_rank: dict[int, int] | None = None, thresh: float = 0.5,
             max_inserts: int = 64, stamps: torch.Tensor | None = None,
             step: int | None = None) -> "LruLayer":
        """Warm start from a hot set (r4d_mxfp4_moe.py.lru.diff L502-533)."""
        hot_t = torch.as_tensor(hot, dtype=torch.int64, device=device)
        S = hot_t.numel()
        table = torch.full((num_experts,), -1, dtype=torch.int32, device=device)
        table[hot_t] = torch.arange(S, dtype=torch.int32, device=device)
        map_cold = torch.arange(num_experts, dtype=torch.int32, device=device)
        map_cold[hot_t] = -1
        slot_expert = hot_t.to(torch.int32).clone()
        if stamps is not None:
            slot_stamp = stamps.to(device=device, dtype=torch.int64).clone()
        elif profile_rank is not None:
            r = torch.tensor([profile_rank.get(int(e), len(profile_rank)) for e in hot_t.tolist()],
                             dtype=torch.int64, device=device)
            slot_stamp = S - torch.argsort(torch.argsort(r))      # hottest -> S, coldest -> 1
        else:
            slot_stamp = torch.zeros(S, dtype=torch.int64, device=device)
        cap = min(max_inserts, S)
        return cls(table, map_cold, slot_expert, slot_stamp.contiguous(),
                   torch.zeros(num_experts, dtype=torch.uint8, device=device),
                   torch.full((1,), S if step is None else step, dtype=torch.int64, device=device),
                   torch.full((max(cap, 1), 2), -1, dtype=torch.int32, device=device),
                   torch.zeros(1, dtype=torch.int32, device=device),
                   max(1, int(S * thresh)), cap)

    def snapshot(self) -> dict[str, torch.Tensor]:
        return {n: getattr(self, n).clone() for n in self.NAMES}

    def restore(self, snap: dict[str, torch.Tensor]) -> None:
        for n in self.NAMES:
            getattr(self, n).copy_(snap[n])

    def state_args(self) -> list[torch.Tensor]:
        return [getattr(self, n) for n in self.NAMES]

    def manage(self, topk_ids: torch.Tensor) -> None:
        torch.ops.vllm.r4d_lru_manage(topk_ids.reshape(-1).to(torch.int32), *self.state_args(),
                                      self.max_distinct, self.max_inserts)

    def new_align_outputs(self, mk: int, block_size: int = BLOCK) -> list[torch.Tensor]:
        n, nb = _align_sizes(mk, self.E, block_size)
        dev = self.table.device
        return [torch.empty(n, dtype=torch.int32, device=dev),
                torch.empty(nb, dtype=torch.int32, device=dev),
                torch.empty(1, dtype=torch.int32, device=dev),
                torch.empty(n, dtype=torch.int32, device=dev),
                torch.empty(nb, dtype=torch.int32, device=dev),
                torch.empty(1, dtype=torch.int32, device=dev)]

    def fused(self, topk_ids: torch.Tensor, out: list[torch.Tensor] | None = None,
              block_size: int = BLOCK):
        """The fused step; returns ((sorted, eids, npad) hot, (sorted, eids, npad) cold)."""
        ids = topk_ids.reshape(-1).to(torch.int32)
        if out is None:
            out = self.new_align_outputs(ids.numel(), block_size)
        torch.ops.vllm.r4d_lru_fused(ids, *self.state_args(), *out, self.max_distinct,
                                     self.max_inserts, block_size)
        return tuple(out[0:3]), tuple(out[3:6])

    def gather(self, dsts: list[torch.Tensor], srcs: list[torch.Tensor], chunks: int = 8,
               lanes: int = 16) -> None:
        torch.ops.vllm.r4d_lru_gather(dsts, srcs, self.miss, self.n_miss, chunks, lanes)

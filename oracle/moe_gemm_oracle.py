"""CPU/torch oracle of the grouped MXFP4 x FP8 MoE GEMM -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this module, as the
checker; the product path (r9700-lru-expert-cache_b200/moe_ops.py -> csrc/moe_gemm.cu) never
imports it.

The kernel it checks replaces the closed r4d_gemm_moe_mxfp4a8_nt_b16 (no source in the
reference). Its semantics are the reference's own harness's pure-torch reference
(tests/k1/moe_ref_harness.py), restated here:
  * dequant_expert: e2m1 codes (low nibble = even k) times 2^(E8M0 - 127) per 32-K group
    (moe_ref_harness.py:86-98);
  * moe_align_block_size: per-expert runs of flat (token * top_k + k) ids in a stable order,
    each padded to a multiple of the block with the sentinel numel, expert_ids per block, the
    padded length (moe_ref_harness.py:109-146), plus vLLM's expert_map / ignore_invalid_experts
    form the hot / cold calls use (an id mapped to -1 is dropped);
  * build_case: E8M0 scales ref - drop with ref in [120, 136) and drop in [0, 8], so every
    scaled weight is exact (moe_ref_harness.py:168-210);
  * gemm_ref: row i of the output reads activation row i // top_k, the weights of its block's
    expert, fp32 (the harness's `a_f32 @ wd.T`), times the routed weight when given.
Parity is by tolerance (the reference accepts fp32 accumulation order and the bf16 output
rounding as the only slack, moe_ref_harness.py:342-344); rows the blocks do not name stay NaN
in the reference output so that a test can check the kernel leaves them untouched.
"""
from __future__ import annotations

import torch

GROUP = 32
BLOCK = 16
FP8_MAX = 448.0
E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def dequant_expert(w: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """One expert in checkpoint order: uint8 [N, K/2] codes + uint8 [N, K/32] E8M0 -> fp32 [N, K]."""
    N, K2 = w.shape
    codes = torch.empty(N, 2 * K2, dtype=torch.uint8, device=w.device)
    codes[:, 0::2] = w & 0x0F
    codes[:, 1::2] = w >> 4
    mag = torch.tensor(E2M1, device=w.device)[(codes & 0x7).long()]
    mag = torch.where((codes & 0x8) > 0, -mag, mag)
    return mag * torch.exp2(s.float() - 127.0).repeat_interleave(GROUP, dim=1)


def quant_fp8_per_token(x: torch.Tensor):
    """The harness's per-token FP8 quant (moe_ref_harness.py:101-106): (e4m3 [M, K], fp32 [M])."""
    amax = x.abs().amax(dim=1).float().clamp(min=1e-12)
    scale = (amax / FP8_MAX).contiguous()
    q = (x.float() / scale.unsqueeze(1)).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    return q, scale


def align_sizes(mtk: int, num_experts: int, block: int = BLOCK) -> int:
    """Capacity of sorted_ids as vLLM allocates it (moe_ref_harness.py:117-120)."""
    cap = mtk + num_experts * (block - 1)
    if mtk < num_experts:
        cap = min(mtk * block, cap)
    return cap


def moe_align_block_size(topk_ids: torch.Tensor, block: int, num_experts: int,
                         expert_map: torch.Tensor | None = None):
    """(sorted_ids, expert_ids, num_post_pad), int32, stable within each expert. With
    expert_map, an id e becomes expert_map[e] and ids mapped to -1 are dropped (vLLM's
    ignore_invalid_experts=True, the hot / cold calls)."""
    mtk = topk_ids.numel()
    cap = align_sizes(mtk, num_experts, block)
    flat = topk_ids.reshape(-1).long()
    if expert_map is not None:
        flat = expert_map.long()[flat]
    keep = flat >= 0
    order = torch.argsort(torch.where(keep, flat, num_experts), stable=True)
    counts = torch.bincount(flat[keep], minlength=num_experts)
    sorted_ids = torch.full((cap,), mtk, dtype=torch.int32, device=topk_ids.device)
    expert_ids = torch.zeros((cap + block - 1) // block, dtype=torch.int32, device=topk_ids.device)
    src = dst = 0
    for e, c in enumerate(counts.tolist()):
        if c == 0:
            continue
        nb = (c + block - 1) // block
        sorted_ids[dst:dst + c] = order[src:src + c].to(torch.int32)
        expert_ids[dst // block: dst // block + nb] = e
        src += c
        dst += nb * block
    return sorted_ids, expert_ids, torch.tensor([dst], dtype=torch.int32, device=topk_ids.device)


def build_case(E: int, N: int, K: int, M: int, top_k: int, seed: int, device):
    """Random weights / scales / routing in checkpoint order (moe_ref_harness.py:168-210):
    w uint8 [E, N, K/2], s uint8 [E, N, K/32], x fp32 [M, K] * 0.4, topk_ids int32 [M, top_k],
    routed weights fp32 [M * top_k]."""
    g = torch.Generator(device=device).manual_seed(seed)
    nb = K // GROUP
    ref = torch.randint(120, 136, (E, N, 1), generator=g, dtype=torch.int32, device=device)
    drop = torch.randint(0, 9, (E, N, nb), generator=g, dtype=torch.int32, device=device)
    s = (ref - drop).clamp(0, 254).to(torch.uint8)
    w = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.uint8, device=device)
    topk_ids = torch.randint(0, E, (M, top_k), generator=g, dtype=torch.int32, device=device)
    x = torch.randn(M, K, generator=g, device=device, dtype=torch.float32) * 0.4
    tw = torch.rand(M * top_k, generator=g, device=device, dtype=torch.float32)
    return w, s, x, topk_ids, tw


def gemm_ref(qx: torch.Tensor, xs: torch.Tensor, w: torch.Tensor, s: torch.Tensor,
             sorted_ids: torch.Tensor, expert_ids: torch.Tensor, num_post_pad: torch.Tensor,
             tw: torch.Tensor | None, mtk: int, top_k: int, expert_index: torch.Tensor | None = None):
    """fp32 [mtk, N]: the rows the live blocks name, NaN elsewhere. expert_index maps a block's
    expert id to the row of w / s holding that expert (the hot call's slot -> expert)."""
    N = w.shape[1]
    out = torch.full((mtk, N), float("nan"), dtype=torch.float32, device=qx.device)
    a = qx.float() * xs.reshape(-1, 1).float()
    npad = int(num_post_pad.reshape(-1)[0])
    for b in range(npad // BLOCK):
        e = int(expert_ids[b])
        if e < 0:
            continue
        ids = [int(i) for i in sorted_ids[b * BLOCK:(b + 1) * BLOCK].tolist() if 0 <= int(i) < mtk]
        if not ids:
            continue
        we = int(expert_index[e]) if expert_index is not None else e
        wd = dequant_expert(w[we], s[we])
        rows = torch.tensor(ids, device=qx.device)
        val = a[rows // top_k] @ wd.T
        if tw is not None:
            val = val * tw.reshape(-1)[rows].unsqueeze(1)
        out[rows] = val
    return out

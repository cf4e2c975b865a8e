"""``moe_sum``: the routed experts' outputs of each token summed over top_k, the last step of
the MoE block (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff
L638, L696: ``ops.moe_sum(ic3.view(M, top_k, H), output)``), with vLLM's signature and
rounding, backed by the sm_100a kernel ``b200_moe_sum`` in csrc/moe_sum.cu.

Rounding: for top_k in {2, 3, 4} the running sum is rounded to the storage dtype after every
add (vLLM's kernel keeps it in that type); for any other top_k vLLM falls back to torch.sum
over the top_k axis, whose CUDA reduction keeps four interleaved fp32 accumulators
(k = i mod 4) combined as ((a0 + a1) + a2) + a3 and rounds once; the kernel sums in that order.
For H = 1 torch splits the top_k axis across threads instead, an order this kernel does not
follow.
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def moe_sum(input: torch.Tensor, output: torch.Tensor) -> None:  # noqa: A002 (vLLM's name)
    """output[t, :] = sum_k input[t, k, :]; input [T, top_k, H] contiguous, output [T, H]
    (unit column stride), same dtype. Writes `output` in place."""
    _lib.require_cuda("moe_sum", input, output)
    if input.ndim != 3 or not input.is_contiguous():
        raise ValueError("moe_sum: input must be a contiguous [tokens, top_k, H] tensor")
    t, topk, h = input.shape
    if output.shape != (t, h) or output.dtype != input.dtype or output.stride(1) != 1:
        raise ValueError("moe_sum: output must be [tokens, H] of input's dtype, unit column stride")
    if input.dtype not in _DTYPES:
        raise ValueError(f"moe_sum: unsupported dtype {input.dtype}")
    rc = _lib.lmhead().b200_moe_sum(_lib.ptr(input), _lib.ptr(output), t, topk, h,
                                    output.stride(0), _DTYPES[input.dtype], _lib.stream_ptr())
    _lib.check(rc, "b200_moe_sum")


# ---- grouped MXFP4 x FP8 MoE GEMM (the consumer of r4d_lru_fused's align outputs) ------------
#
# The reference's R4dMxfp4MoEExperts runs the closed r4d_gemm_moe_mxfp4a8_nt_b16 twice per
# projection, over the resident (hot) experts from their compact VRAM copies and over the rest
# (cold) from the full tensors, into one output (r4d_mxfp4_moe.py.lru.diff L584-606,
# _r4d_mxfp4_moe_gemm_into at L454-500). Here the same op runs the sm_100a kernel of
# csrc/moe_gemm.cu on the B200 packing of the same checkpoint codes and scales.

MOE_BLOCK = 16       # rows per aligned block (r4d_gemm_moe_mxfp4a8_nt_b16_block)
MOE_GROUP = 32       # K per E8M0 exponent (r4d_gemm_moe_mxfp4a8_nt_b16_group)


def _pack_index(device):
    """For lane l = 4 g + t of a 32-K group, k-half h, A register p and element j (0: low
    nibble, 1: high): the (row in the 16-row strip, k in the group) the code comes from, and its
    bit position in the lane's 8 bytes (byte 4 h + p, element j in nibble j)."""
    lane = torch.arange(32, device=device).view(32, 1, 1, 1)
    h = torch.arange(2, device=device).view(1, 2, 1, 1)
    p = torch.arange(4, device=device).view(1, 1, 4, 1)
    j = torch.arange(2, device=device).view(1, 1, 1, 2)
    g, t = lane >> 2, lane & 3
    row = (g + 8 * (p & 1)).expand(32, 2, 4, 2)
    k = (16 * h + 2 * t + 8 * (p >> 1) + j).expand(32, 2, 4, 2)
    shift = (32 * h + 8 * p + 4 * j).expand(32, 2, 4, 2)
    return row, k, shift


@torch.no_grad()
def pack_mxfp4_moe(w: torch.Tensor, scales: torch.Tensor):
    """Checkpoint MXFP4 expert weights -> the B200 packing.

    w uint8 [E, N, K/2]: byte j of a row holds the e2m1 code of k = 2 j in its low nibble and of
    k = 2 j + 1 in its high nibble (the checkpoint order the reference permutes,
    r4d_mxfp4_moe.py.lru.diff _permute_moe_inplace); scales uint8 [E, N, K/32] E8M0.
    Returns (wq uint8 [E, N/16, 272 K/32], ws, wref): wq holds one record per 16-row strip --
    the codes in mma.sync fragment order [K/32][32 lanes][8 B], then the strip's exponents
    [16 rows][K/32] -- so that a run of strips is one contiguous copy; ws (the scales viewed by
    strip, [E, N/16, 16, K/32]) and wref (each row's largest exponent, the reference's
    w*_wref = s.max(dim=2)) complete the reference's argument list and are not read by the
    kernel."""
    E, N, K2 = w.shape
    K = 2 * K2
    if w.dtype != torch.uint8 or scales.dtype != torch.uint8 or scales.shape != (E, N, K // MOE_GROUP):
        raise ValueError("pack_mxfp4_moe: w uint8 [E, N, K/2] and scales uint8 [E, N, K/32] expected")
    if N % 16 or K % MOE_GROUP:
        raise ValueError("pack_mxfp4_moe: N % 16 == 0 and K % 32 == 0 are required")
    NS, G = N // 16, K // MOE_GROUP
    row, k, shift = _pack_index(w.device)
    wq = torch.empty(E, NS, G * 272, dtype=torch.uint8, device=w.device)
    for e in range(E):                       # one expert at a time bounds the temporaries
        codes = torch.stack((w[e] & 0xF, w[e] >> 4), dim=-1).reshape(NS, 16, G, MOE_GROUP)
        codes = codes.permute(0, 2, 1, 3)                                   # [NS, G, 16, 32]
        picked = codes[:, :, row, k].to(torch.int64)                        # [NS, G, 32, 2, 4, 2]
        word64 = (picked << shift).sum(dim=(-1, -2, -3))                    # [NS, G, 32]
        b = torch.stack([(word64 >> (8 * i)) & 0xFF for i in range(8)], dim=-1)
        wq[e, :, :G * 256] = b.to(torch.uint8).reshape(NS, G * 256)
    ws = scales.reshape(E, NS, 16, G).contiguous()
    wq[:, :, G * 256:] = ws.reshape(E, NS, 16 * G)
    wref = scales.max(dim=2).values.contiguous()
    return wq, ws, wref


@torch.no_grad()
def unpack_mxfp4_moe(wq: torch.Tensor):
    """The inverse of pack_mxfp4_moe's records: (w [E, N, K/2], scales [E, N, K/32]) in
    checkpoint order."""
    E, NS, R = wq.shape
    G = R // 272
    row, k, shift = _pack_index(wq.device)
    b = wq[:, :, :G * 256].reshape(E, NS, G, 32, 8).to(torch.int64)
    word64 = sum(b[..., i] << (8 * i) for i in range(8))                    # [E, NS, G, 32]
    codes = torch.empty(E, NS, G, 16, MOE_GROUP, dtype=torch.uint8, device=wq.device)
    vals = ((word64.view(E, NS, G, 32, 1, 1, 1) >> shift) & 0xF).to(torch.uint8)
    codes[:, :, :, row, k] = vals
    codes = codes.permute(0, 1, 3, 2, 4).reshape(E, NS * 16, G * MOE_GROUP)
    w = (codes[..., 0::2] | (codes[..., 1::2] << 4)).contiguous()
    scales = wq[:, :, G * 256:].reshape(E, NS * 16, G).contiguous()
    return w, scales


def _check_cfg(em: int, N: int, K: int, wv: int, sk: int, npw: int) -> None:
    """The reference op's preconditions on its launch knobs (r4d_mxfp4_moe.py.lru.diff
    L484-488), kept so that a caller's configuration is validated the same way."""
    if not (em >= 1 and N % 16 == 0 and K % (sk * MOE_GROUP) == 0 and wv * sk * 32 <= 1024
            and npw in (1, 2, 4, 8) and wv * npw * sk * 1024 <= 64 * 1024):
        raise ValueError(f"r4d_mxfp4_moe_gemm: invalid shape/config em={em} N={N} K={K} cfg={(wv, sk, npw)}")


def _moe_check(y, qx, x_scale, wq, sorted_ids, expert_ids, num_post_pad, topk_weights, mtk):
    """The op's argument checks; returns (K, N, em, x_scale flat, topk_weights flat or None)."""
    K = qx.shape[1]
    E, NS, R = wq.shape
    G = R // 272
    N = NS * 16
    if y.shape != (mtk, N) or y.dtype != torch.bfloat16 or not y.is_contiguous():
        raise ValueError(f"r4d_mxfp4_moe_gemm: y must be contiguous bf16 [{mtk}, {N}]")
    if G * MOE_GROUP != K or qx.dtype != torch.float8_e4m3fn or not qx.is_contiguous():
        raise ValueError("r4d_mxfp4_moe_gemm: qx must be contiguous e4m3 [tokens, K] matching the pack")
    if R % 272 or wq.dtype != torch.uint8 or not wq.is_contiguous():
        raise ValueError("r4d_mxfp4_moe_gemm: wq must be a contiguous uint8 [E, N/16, 272 K/32] pack")
    for t, name in ((sorted_ids, "sorted_ids"), (expert_ids, "expert_ids"), (num_post_pad, "num_post_pad")):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise ValueError(f"r4d_mxfp4_moe_gemm: {name} must be contiguous int32")
    xs = x_scale.reshape(-1)
    if xs.dtype != torch.float32 or not xs.is_contiguous():
        raise ValueError("r4d_mxfp4_moe_gemm: x_scale must be contiguous fp32")
    tw = None
    if topk_weights is not None:
        tw = topk_weights.reshape(-1)
        if tw.dtype != torch.float32 or tw.numel() < mtk or not tw.is_contiguous():
            raise ValueError("r4d_mxfp4_moe_gemm: topk_weights must be contiguous fp32 [mtk]")
    return K, N, sorted_ids.numel(), xs, tw


def mxfp4_moe_gemm_into(y: torch.Tensor, qx: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor,
                        ws: torch.Tensor, wref: torch.Tensor, sorted_ids: torch.Tensor,
                        expert_ids: torch.Tensor, num_post_pad: torch.Tensor,
                        topk_weights: torch.Tensor | None, mtk: int, top_k: int,
                        wv: int = 1, sk: int = 1, npw: int = 1) -> None:
    """y[i, :] for every row i the aligned blocks name (the rows of a block share its expert):
    bf16(topk_weights[i] * x_scale[i // top_k] * qx[i // top_k] . W_e); other rows untouched.
    qx e4m3 [tokens, K], x_scale fp32 [tokens] (or [tokens, 1]); wq from pack_mxfp4_moe (or the
    hot experts' compact copies indexed by slot); ws / wref are the reference's remaining
    arguments (any CUDA tensors: the kernel reads codes and exponents from wq); y bf16
    [mtk, N]."""
    _lib.require_cuda("r4d_mxfp4_moe_gemm", y, qx, x_scale, wq, ws, wref, sorted_ids, expert_ids,
                      num_post_pad, topk_weights)
    K, N, em, xs, tw = _moe_check(y, qx, x_scale, wq, sorted_ids, expert_ids, num_post_pad, topk_weights, mtk)
    _check_cfg(em, N, K, wv, sk, npw)
    lib = _lib.lmhead()
    lib.r4d_gemm_moe_mxfp4a8_nt_b16(qx.data_ptr(), xs.data_ptr(), wq.data_ptr(), ws.data_ptr(),
                                    wref.data_ptr(), y.data_ptr(), sorted_ids.data_ptr(),
                                    expert_ids.data_ptr(), num_post_pad.data_ptr(),
                                    0 if tw is None else tw.data_ptr(), em, mtk, top_k, K, N, wv, sk, npw,
                                    torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.r4d_gemm_moe_mxfp4a8_nt_b16_last_error(), "r4d_gemm_moe_mxfp4a8_nt_b16")


def mxfp4_moe_gemm(qx: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor,
                   wref: torch.Tensor, sorted_ids: torch.Tensor, expert_ids: torch.Tensor,
                   num_post_pad: torch.Tensor, topk_weights: torch.Tensor | None, mtk: int, top_k: int,
                   wv: int = 1, sk: int = 1, npw: int = 1) -> torch.Tensor:
    """The allocating form (the reference's r4d_mxfp4_moe_gemm): a fresh bf16 [mtk, N]."""
    y = torch.empty(mtk, wq.shape[1] * 16, dtype=torch.bfloat16, device=qx.device)
    mxfp4_moe_gemm_into(y, qx, x_scale, wq, ws, wref, sorted_ids, expert_ids, num_post_pad, topk_weights,
                        mtk, top_k, wv, sk, npw)
    return y


def gemm_split(y: torch.Tensor, qx: torch.Tensor, xs: torch.Tensor, full: tuple, hot: tuple,
               align_hot: tuple, align_cold: tuple, tw: torch.Tensor | None, mtk: int, top_k: int,
               skip_cold: bool = False, cfg: tuple = (1, 1, 1)) -> None:
    """_gemm_split (r4d_mxfp4_moe.py.lru.diff L584-606): the hot call over the resident slots'
    copies (`hot` = (wq, ws, wref) indexed by slot, align_hot from r4d_lru_fused) and the cold
    call over the full tensors (`full`, indexed by expert id, align_cold), filling disjoint rows
    of y -- here in ONE launch (b200_moe_gemm_hot_cold), which is the two calls' result without
    the second launch. skip_cold runs the hot call alone."""
    if skip_cold:
        mxfp4_moe_gemm_into(y, qx, xs, *hot, *align_hot, tw, mtk, top_k, *cfg)
        return
    _lib.require_cuda("r4d_mxfp4_moe_gemm", y, qx, xs, hot[0], full[0], *align_hot, *align_cold, tw)
    K, N, em_h, xsf, twf = _moe_check(y, qx, xs, hot[0], *align_hot, tw, mtk)
    K2, N2, em_c, _, _ = _moe_check(y, qx, xs, full[0], *align_cold, tw, mtk)
    _check_cfg(em_h, N, K, *cfg)
    _check_cfg(em_c, N, K, *cfg)
    rc = _lib.lmhead().b200_moe_gemm_hot_cold(
        qx.data_ptr(), xsf.data_ptr(), hot[0].data_ptr(), full[0].data_ptr(), y.data_ptr(),
        align_hot[0].data_ptr(), align_hot[1].data_ptr(), align_hot[2].data_ptr(), em_h,
        align_cold[0].data_ptr(), align_cold[1].data_ptr(), align_cold[2].data_ptr(), em_c,
        0 if twf is None else twf.data_ptr(), mtk, top_k, K, N, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "b200_moe_gemm_hot_cold")


def _register_moe_ops() -> None:
    if hasattr(torch.ops.vllm, "r4d_mxfp4_moe_gemm_into"):
        return

    @torch.library.custom_op("vllm::r4d_mxfp4_moe_gemm_into", mutates_args=["y"])
    def _gemm_into(y: torch.Tensor, qx: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor,
                   ws: torch.Tensor, wref: torch.Tensor, sorted_ids: torch.Tensor, expert_ids: torch.Tensor,
                   num_post_pad: torch.Tensor, topk_weights: torch.Tensor | None, mtk: int, top_k: int,
                   wv: int, sk: int, npw: int) -> None:
        mxfp4_moe_gemm_into(y, qx, x_scale, wq, ws, wref, sorted_ids, expert_ids, num_post_pad,
                            topk_weights, mtk, top_k, wv, sk, npw)

    @torch.library.custom_op("vllm::r4d_mxfp4_moe_gemm", mutates_args=())
    def _gemm(qx: torch.Tensor, x_scale: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, wref: torch.Tensor,
              sorted_ids: torch.Tensor, expert_ids: torch.Tensor, num_post_pad: torch.Tensor,
              topk_weights: torch.Tensor | None, mtk: int, top_k: int, wv: int, sk: int,
              npw: int) -> torch.Tensor:
        return mxfp4_moe_gemm(qx, x_scale, wq, ws, wref, sorted_ids, expert_ids, num_post_pad, topk_weights,
                              mtk, top_k, wv, sk, npw)

    @_gemm.register_fake
    def _gemm_fake(qx, x_scale, wq, ws, wref, sorted_ids, expert_ids, num_post_pad, topk_weights, mtk, top_k,
                   wv, sk, npw):
        return qx.new_empty((mtk, wq.shape[1] * 16), dtype=torch.bfloat16)


_register_moe_ops()

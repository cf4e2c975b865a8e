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

"""Per-token FP8 quant of the MoE hidden states: the host-side mirror of ``fp8_quant_shared``
(patches/model_executor/kernels/linear/mxfp4/r4dhip.py.diff L19-34) and of the vLLM op it
calls, ``ops.scaled_fp8_quant(x, use_per_token_if_dynamic=True)``, backed by the sm_100a
kernel ``b200_per_token_quant_fp8`` in csrc/quant.cu.

The quant is the second half of fused_silu_mul_quant without the SiLU: per row amax (capped
by ``scale_ub`` when given), ``scale = max(amax / 448, 1 / (448 * 512))``, and
``q = e4m3(clamp(x / scale, +-448))`` with a true division.

``fp8_quant_shared`` keeps the reference's single-slot handoff: the shared expert and the
routed experts quantize the same hidden-state tensor back to back, so with
``VLLM_R4D_SHARE_A8=1`` the second call reuses the first's result. The slot is keyed on
Python object identity (inference tensors carry no version counter, and a bare data_ptr can
be reused by an unrelated tensor), holds a strong reference so the key cannot be freed and
aliased while cached, and is cleared by the hit so a result is served at most once. It
still assumes nobody writes into that tensor in place between the two calls (off by
default, as in the reference).
"""
from __future__ import annotations

import os

import torch

from . import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1}
_A8_SHARE = os.environ.get("VLLM_R4D_SHARE_A8", "0") == "1"
_a8_slot: tuple | None = None


def scaled_fp8_quant(x: torch.Tensor, scale: torch.Tensor | None = None,
                     use_per_token_if_dynamic: bool = False,
                     scale_ub: torch.Tensor | None = None,
                     fp8_dtype: torch.dtype = torch.float8_e4m3fn
                     ) -> tuple[torch.Tensor, torch.Tensor]:
    """Dynamic per-token FP8 quant: (q e4m3 [rows, K], scale fp32 [rows, 1]).

    Only the form the hot path calls is built (dynamic, per token): a static ``scale`` or
    ``use_per_token_if_dynamic=False`` (one scale for the whole tensor) raise."""
    if scale is not None or not use_per_token_if_dynamic:
        raise NotImplementedError("scaled_fp8_quant: only the dynamic per-token form is built")
    if fp8_dtype != torch.float8_e4m3fn:
        raise ValueError(f"scaled_fp8_quant: only torch.float8_e4m3fn is supported, got {fp8_dtype}")
    _lib.require_cuda("scaled_fp8_quant", x, scale_ub)
    if x.ndim != 2 or x.stride(1) != 1 or x.dtype not in _DTYPES:
        raise ValueError("scaled_fp8_quant: x must be 2-D bf16/f16 with unit last stride")
    if scale_ub is not None and (scale_ub.numel() != 1 or scale_ub.dtype != torch.float32):
        raise ValueError("scaled_fp8_quant: scale_ub must be one fp32 value")
    rows, k = x.shape
    q = torch.empty((rows, k), dtype=fp8_dtype, device=x.device)
    s = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    if rows:
        rc = _lib.lmhead().b200_per_token_quant_fp8(
            _lib.ptr(x), rows, k, x.stride(0), _DTYPES[x.dtype], _lib.ptr(scale_ub),
            _lib.ptr(q), _lib.ptr(s), _lib.stream_ptr())
        _lib.check(rc, "b200_per_token_quant_fp8")
    return q, s


def fp8_quant_shared(x: torch.Tensor, quant=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token fp8 quantization of `x`, reusing the immediately preceding result for the
    same tensor object when VLLM_R4D_SHARE_A8=1. ``quant`` replaces the quant call (the
    tests pass a host-side one)."""
    global _a8_slot
    q_fn = quant or (lambda t: scaled_fp8_quant(t, use_per_token_if_dynamic=True))
    if not _A8_SHARE:
        return q_fn(x)
    slot = _a8_slot
    if slot is not None and slot[0] is x:
        _a8_slot = None                          # single use: a hit is served once
        return slot[1], slot[2]
    qx, xs = q_fn(x)
    _a8_slot = (x, qx, xs)
    return qx, xs


def set_share(enabled: bool) -> None:
    """Switch the handoff at run time (VLLM_R4D_SHARE_A8 sets the default) and drop the slot."""
    global _A8_SHARE, _a8_slot
    _A8_SHARE = bool(enabled)
    _a8_slot = None

"""Fused ``silu_and_mul`` + FP8 activation quant: the host-side mirror of
kernels/fused_silu_mul_quant.py (``supported``, ``silu_mul_quant``), backed by the sm_100a
kernel in csrc/quant.cu (``b200_silu_mul_quant``).

Bit-identical to vLLM's ``silu_and_mul`` followed by ``scaled_fp8_quant(...,
use_per_token_if_dynamic=True)``: silu rounded to the storage dtype before the multiply, the
product rounded on store, the row absmax of that stored value, the scale floored at
1/(448*512), and a true division by the scale (fused_silu_mul_quant.py:9-14).

``silu_mul_quant_group`` is the per-token group-128 variant (scales [rows, d/128], the
per_token_group_quant_fp8 formula) that feeds block-scaled FP8 GEMMs.
"""
from __future__ import annotations

import torch

from . import _lib

_MIN_SCALE_DIV = 512.0
_MAX_BLOCK = 8192
_DTYPES = {torch.bfloat16: 0, torch.float16: 1}


def _next_pow2(n: int) -> int:
    return 1 if n <= 1 else 1 << (n - 1).bit_length()


def supported(x: torch.Tensor) -> bool:
    """Whether `x` is a [rows, 2*d] gated-activation input this kernel handles
    (fused_silu_mul_quant.py:60-72: 2-D bf16/f16, even width, unit last stride, and a
    half-row of at most 8192)."""
    return (
        x.is_cuda
        and x.ndim == 2
        and x.dtype in _DTYPES
        and x.shape[1] % 2 == 0
        and x.stride(1) == 1
        and _next_pow2(x.shape[1] // 2) <= _MAX_BLOCK
    )


def _check_fp8(fp8_dtype: torch.dtype) -> None:
    if fp8_dtype != torch.float8_e4m3fn:
        raise ValueError(f"silu_mul_quant: only torch.float8_e4m3fn is supported, got {fp8_dtype}")


def silu_mul_quant(x: torch.Tensor, fp8_dtype: torch.dtype, write_act: bool = False
                   ) -> tuple[torch.Tensor | None, torch.Tensor, torch.Tensor]:
    """``silu_and_mul(x)`` and its per-token fp8 quant in one launch.

    Returns (act, q, scale): act is the activation in x's dtype and None unless
    `write_act`; q e4m3 [rows, d]; scale fp32 [rows, 1]. Caller checks supported() first.
    """
    _check_fp8(fp8_dtype)
    _lib.require_cuda("silu_mul_quant", x)
    rows, d = x.shape[0], x.shape[1] // 2
    q = torch.empty((rows, d), dtype=fp8_dtype, device=x.device)
    scale = torch.empty((rows, 1), dtype=torch.float32, device=x.device)
    act = torch.empty((rows, d), dtype=x.dtype, device=x.device) if write_act else None
    if rows:
        rc = _lib.lmhead().b200_silu_mul_quant(
            _lib.ptr(x), rows, d, x.stride(0), _DTYPES[x.dtype], _lib.ptr(q), _lib.ptr(scale),
            _lib.ptr(act), 0, _lib.stream_ptr())
        _lib.check(rc, "b200_silu_mul_quant")
    return act, q, scale


def silu_mul_quant_group(x: torch.Tensor, fp8_dtype: torch.dtype = torch.float8_e4m3fn,
                         group: int = 128, write_act: bool = False
                         ) -> tuple[torch.Tensor | None, torch.Tensor, torch.Tensor]:
    """SiLU*mul with per-token group-128 scales: (act | None, q e4m3 [rows, d],
    scale fp32 [rows, d/128]). Needs d % 128 == 0 and 16-byte aligned rows."""
    _check_fp8(fp8_dtype)
    _lib.require_cuda("silu_mul_quant_group", x)
    if group != 128:
        raise ValueError("silu_mul_quant_group: group must be 128")
    rows, d = x.shape[0], x.shape[1] // 2
    if d % group:
        raise ValueError(f"silu_mul_quant_group: d={d} must be a multiple of {group}")
    q = torch.empty((rows, d), dtype=fp8_dtype, device=x.device)
    scale = torch.empty((rows, d // group), dtype=torch.float32, device=x.device)
    act = torch.empty((rows, d), dtype=x.dtype, device=x.device) if write_act else None
    if rows:
        rc = _lib.lmhead().b200_silu_mul_quant(
            _lib.ptr(x), rows, d, x.stride(0), _DTYPES[x.dtype], _lib.ptr(q), _lib.ptr(scale),
            _lib.ptr(act), group, _lib.stream_ptr())
        _lib.check(rc, "b200_silu_mul_quant(group=128)")
    return act, q, scale


def per_token_group_quant_fp8(x: torch.Tensor, group_size: int = 128,
                              dtype: torch.dtype = torch.float8_e4m3fn
                              ) -> tuple[torch.Tensor, torch.Tensor]:
    """vLLM's per_token_group_quant_fp8(x, group) as called by the FP8 target head
    (kernels/fp8_target_lmhead.py:73): q e4m3 [M, K], row-major fp32 scales [M, K/group]."""
    _check_fp8(dtype)
    _lib.require_cuda("per_token_group_quant_fp8", x)
    if x.ndim != 2 or x.stride(1) != 1 or x.dtype not in _DTYPES:
        raise ValueError("per_token_group_quant_fp8: x must be 2-D bf16/f16 with unit last stride")
    M, K = x.shape
    q = torch.empty((M, K), dtype=dtype, device=x.device)
    s = torch.empty((M, K // group_size), dtype=torch.float32, device=x.device)
    rc = _lib.lmhead().b200_per_token_group_quant_fp8(
        _lib.ptr(x), M, K, x.stride(0), _DTYPES[x.dtype], group_size, _lib.ptr(q), _lib.ptr(s),
        _lib.stream_ptr())
    _lib.check(rc, "b200_per_token_group_quant_fp8")
    return q, s

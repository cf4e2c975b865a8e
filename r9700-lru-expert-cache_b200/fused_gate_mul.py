"""The MoE shared expert's ``sigmoid(gate) * out`` in one launch: the host-side mirror of
kernels/fused_gate_mul.py (``supported``, ``sigmoid_gate_mul``, ``supported_gemv``,
``gemv_sigmoid_gate_mul``), backed by the sm_100a kernels in csrc/gate.cu.

``sigmoid_gate_mul`` is bit-identical to ``F.sigmoid(gate) * out``: the sigmoid is computed
in fp32 and rounded to the gate's dtype before the multiply, as aten's opmath does
(fused_gate_mul.py:7-10). ``gemv_sigmoid_gate_mul`` also folds the [1, K]
``shared_expert_gate`` GEMV in; only the last bit of the gate scalar can differ from the stock
path, everything after the dot rounds the same way (fused_gate_mul.py:84-88).

Both write a fresh tensor rather than mutate ``out``, which may be an all-reduce output
buffer (fused_gate_mul.py:59-62).
"""
from __future__ import annotations

import torch

from . import _lib

_DTYPES = {torch.bfloat16: 0, torch.float16: 1, torch.float32: 2}


def supported(gate: torch.Tensor, out: torch.Tensor) -> bool:
    """Whether this pair is the [T, 1] x [T, H] shared-expert-gate shape
    (fused_gate_mul.py:41-53)."""
    return (
        gate.is_cuda
        and out.is_cuda
        and gate.dtype == out.dtype
        and gate.dtype in _DTYPES
        and gate.ndim == 2
        and out.ndim == 2
        and gate.shape[1] == 1
        and gate.shape[0] == out.shape[0]
        and gate.stride(0) == 1
        and out.stride(1) == 1
    )


def sigmoid_gate_mul(gate: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """``sigmoid(gate) * out`` in one launch. Caller checks supported() first."""
    _lib.require_cuda("sigmoid_gate_mul", gate, out)
    n_rows, n_cols = out.shape
    y = torch.empty((n_rows, n_cols), dtype=out.dtype, device=out.device)
    if n_rows and n_cols:
        rc = _lib.lmhead().b200_sigmoid_gate_mul(
            _lib.ptr(y), _lib.ptr(out), _lib.ptr(gate), n_rows, n_cols, out.stride(0),
            _DTYPES[out.dtype], _lib.stream_ptr())
        _lib.check(rc, "b200_sigmoid_gate_mul")
    return y


def supported_gemv(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor,
                   max_rows: int) -> bool:
    """Whether this is the [T, K] x [1, K] -> [T, 1] shared-expert-gate GEMV with
    0 < T <= max_rows (fused_gate_mul.py:124-147): decode-sized row counts only, prefill
    stays on the library GEMM."""
    return (
        x.is_cuda
        and weight.is_cuda
        and out.is_cuda
        and x.dtype == weight.dtype == out.dtype
        and x.dtype in _DTYPES
        and x.ndim == 2
        and weight.ndim == 2
        and out.ndim == 2
        and weight.shape[0] == 1
        and weight.shape[1] == x.shape[1]
        and weight.stride(1) == 1
        and x.shape[0] == out.shape[0]
        and x.stride(1) == 1
        and out.stride(1) == 1
        and 0 < x.shape[0] <= max_rows
    )


def gemv_sigmoid_gate_mul(x: torch.Tensor, weight: torch.Tensor,
                          out: torch.Tensor) -> torch.Tensor:
    """``sigmoid(x @ weight.T) * out`` in one launch. Caller checks supported_gemv()."""
    _lib.require_cuda("gemv_sigmoid_gate_mul", x, weight, out)
    n_rows, k = x.shape
    n_cols = out.shape[1]
    y = torch.empty((n_rows, n_cols), dtype=out.dtype, device=out.device)
    rc = _lib.lmhead().b200_gemv_sigmoid_gate_mul(
        _lib.ptr(y), _lib.ptr(out), _lib.ptr(x), _lib.ptr(weight), n_rows, k, n_cols,
        x.stride(0), out.stride(0), _DTYPES[x.dtype], _lib.stream_ptr())
    _lib.check(rc, "b200_gemv_sigmoid_gate_mul")
    return y

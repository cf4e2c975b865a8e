"""Caller-owned scratch for the fused lm_head entries (activation tiles and rows, per-CTA row
statistics, partial accumulators). One buffer per (device, stream), reused by every call on
that stream; it needs no initialisation. Calls that share a buffer must not overlap."""
from __future__ import annotations

import torch

from . import _lib

_WS: dict[tuple[int, int], torch.Tensor] = {}


def workspace(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    ws = _WS.get(key)
    if ws is None:
        nbytes = int(_lib.lmhead().b200_lmhead_workspace_bytes())
        ws = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _WS[key] = ws
    return ws

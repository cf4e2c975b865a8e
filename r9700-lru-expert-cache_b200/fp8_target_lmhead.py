"""FP8-e4m3 target lm_head with 128x128 fp32 block scales: the host-side mirror of
kernels/fp8_target_lmhead.py (``available``, ``pack_fp8_block``, ``gemm_fp8_block``,
``Fp8TargetHead``, ``_MAX_M``), backed by the sm_100a kernels of csrc/lmhead.cu.

Quantization (unchanged from the reference, fp8_target_lmhead.py:14-18, 56-65): per
128(N) x 128(K) block scale = max(amax, 1e-12)/448 and w_q = e4m3(clamp(w/scale)); the
activation is quantized per token in groups of 128 (per_token_group_quant_fp8), here fused
into the GEMV prologue.

Layout: the reference stores the weight in gfx1201 WMMA fragment order. The B200 pack stores
it as 16-row strips, ``[N/16][K/128][16 rows][128 B]`` with the 16-byte chunk c of row r at
chunk ``c ^ (r & 7)`` -- one bulk copy per strip run for the GEMV, and the 128-byte-swizzled
K-major tile a tensor-core operand expects. ``unpack_fp8_block`` restores row-major order.

``fp8_lmhead`` is the fused entry: logits plus per-row max, argmax and
logsumexp in the same pass over the weight.
"""
from __future__ import annotations

import os

import torch

from . import _lib
from ._workspace import workspace

_BLK = 128
_MAX_M = int(os.environ.get("VLLM_TARGET_FP8_LMHEAD_MAX_M", "64"))
FP8 = torch.float8_e4m3fn


def available() -> bool:
    """True when the kernels can run here: a CUDA sm_100 device and the library loads."""
    try:
        if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
            return False
        _lib.lmhead()
    except Exception:  # noqa: BLE001
        return False
    return True


def _strip_swizzle(wq_rows: torch.Tensor) -> torch.Tensor:
    """Row-major e4m3 [R, K] (R % 16 == 0) -> strip layout bytes, viewed [R, K]."""
    R, K = wq_rows.shape
    b = wq_rows.view(torch.uint8).reshape(R // 16, 16, K // 128, 8, 16)     # st, r, kb, c, byte
    r = torch.arange(16, device=b.device).view(1, 16, 1, 1, 1)
    c = torch.arange(8, device=b.device).view(1, 1, 1, 8, 1)
    src = (c ^ (r & 7)).expand(R // 16, 16, K // 128, 8, 16)
    out = torch.gather(b, 3, src)            # out chunk c' = in chunk c' ^ (r & 7)
    return out.permute(0, 2, 1, 3, 4).contiguous().view(FP8).view(R, K)


def unpack_fp8_block(wq: torch.Tensor) -> torch.Tensor:
    """Strip layout -> row-major e4m3 [N, K] (the inverse of the pack's permutation)."""
    N, K = wq.shape
    b = wq.contiguous().view(torch.uint8).reshape(N // 16, K // 128, 16, 8, 16).permute(0, 2, 1, 3, 4)
    r = torch.arange(16, device=b.device).view(1, 16, 1, 1, 1)
    c = torch.arange(8, device=b.device).view(1, 1, 1, 8, 1)
    src = (c ^ (r & 7)).expand(N // 16, 16, K // 128, 8, 16)
    return torch.gather(b, 3, src).reshape(N, K).view(FP8)


@torch.no_grad()
def pack_fp8_block(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [N, K] -> (strip-packed e4m3 [N, K], fp32 block scales [N/128, K/128]).

    Row-chunked (4096 rows) so the fp32 temporaries stay small, as in the reference."""
    N, K = w.shape
    assert N % _BLK == 0 and K % _BLK == 0, (N, K)
    out = torch.empty(N, K, dtype=FP8, device=w.device)
    ws = torch.empty(N // _BLK, K // _BLK, dtype=torch.float32, device=w.device)
    rows = 4096
    for r0 in range(0, N, rows):
        r1 = min(N, r0 + rows)
        wf = w[r0:r1].float().view((r1 - r0) // _BLK, _BLK, K // _BLK, _BLK)
        amax = wf.abs().amax(dim=(1, 3), keepdim=True).clamp(min=1e-12)
        scale = amax / 448.0
        wq = (wf / scale).clamp(-448.0, 448.0).to(FP8).view(r1 - r0, K)
        out[r0:r1] = _strip_swizzle(wq)
        ws[r0 // _BLK:r1 // _BLK] = scale.view((r1 - r0) // _BLK, K // _BLK)
        del wf, amax, scale, wq
    return out, ws


def _check(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor) -> None:
    _lib.require_cuda("fp8 lm_head", x, wq, ws)
    if x.dtype != torch.bfloat16 or x.ndim != 2 or not x.is_contiguous():
        raise ValueError("fp8 lm_head: x must be a contiguous bf16 [M, K] tensor")
    if wq.dtype != FP8 or wq.shape[1] != x.shape[1] or not wq.is_contiguous():
        raise ValueError(f"fp8 lm_head: weight {tuple(wq.shape)} {wq.dtype} does not match x {tuple(x.shape)}")
    if ws.dtype != torch.float32 or ws.shape != (wq.shape[0] // _BLK, wq.shape[1] // _BLK):
        raise ValueError("fp8 lm_head: ws must be fp32 [N/128, K/128]")


def fp8_lmhead(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, vocab_offset: int = 0,
               want_logits: bool = True, out: torch.Tensor | None = None,
               debug_quant: bool = False, stats_out: tuple | None = None):
    """Fused quant + GEMV + row statistics.

    Returns (logits bf16 [M, N] | None, row_max fp32 [M], argmax int64 [M] (+ vocab_offset),
    logsumexp fp32 [M]) and, with ``debug_quant``, the quantized activation (q, scales).
    ``out`` / ``stats_out`` = (row_max, argmax, logsumexp) take caller-owned outputs (no
    allocation per call, e.g. inside a decode loop or a CUDA graph)."""
    _check(x, wq, ws)
    M, K = x.shape
    N = wq.shape[0]
    dev = x.device
    y = None
    if want_logits:
        y = out if out is not None else torch.empty(M, N, dtype=torch.bfloat16, device=dev)
    if stats_out is not None:
        mx, arg, lse = stats_out
        if (mx.dtype, arg.dtype, lse.dtype) != (torch.float32, torch.int64, torch.float32) or \
                min(mx.numel(), arg.numel(), lse.numel()) < M:
            raise ValueError("fp8 lm_head: stats_out must be (fp32 [M], int64 [M], fp32 [M])")
        _lib.require_cuda("fp8 lm_head", mx, arg, lse)
    else:
        mx = torch.empty(M, dtype=torch.float32, device=dev)
        arg = torch.empty(M, dtype=torch.int64, device=dev)
        lse = torch.empty(M, dtype=torch.float32, device=dev)
    qx = torch.empty(M, K, dtype=FP8, device=dev) if debug_quant else None
    xs = torch.empty(M, K // _BLK, dtype=torch.float32, device=dev) if debug_quant else None
    wsp = workspace(dev)
    rc = _lib.lmhead().b200_fp8_lmhead(
        _lib.ptr(x), M, K, _lib.ptr(wq), _lib.ptr(ws), N, int(vocab_offset), _lib.ptr(y),
        N if y is None else y.stride(0), _lib.ptr(mx), _lib.ptr(arg), _lib.ptr(lse),
        _lib.ptr(qx), _lib.ptr(xs), _lib.ptr(wsp), wsp.numel(), _lib.stream_ptr())
    _lib.check(rc, "b200_fp8_lmhead")
    _lib.debug_check("b200_fp8_lmhead")
    res = (y, mx, arg, lse)
    return res + (qx, xs) if debug_quant else res


class Fp8LmheadStep:
    """A prepared fp8_lmhead call for a decode loop that reuses its buffers: the activation x,
    the logits ``out`` (or none), the statistics triple ``stats_out`` and, optionally, the
    packed float64 [M, 3] triple ``packed_out`` (pack_row_stats' layout, for one device-to-host
    copy) are checked once, together with the launch stream (the current one at construction)
    and its workspace; each call then passes only the weight -- which may rotate between
    same-shaped copies -- to one C call (two with ``packed_out``), with no allocation and no
    per-tensor checks. With a ``combiner`` (sharded.P2PCombiner) the statistics are the
    ranks' combined ones, as in P2PCombiner.fp8_head."""

    def __init__(self, x: torch.Tensor, n_rows: int, vocab_offset: int = 0, out: torch.Tensor | None = None,
                 stats_out: tuple | None = None, packed_out: torch.Tensor | None = None, combiner=None):
        from ._workspace import workspace
        _lib.require_cuda("fp8 lm_head step", x, out, packed_out, *(stats_out or ()))
        if x.dtype != torch.bfloat16 or x.ndim != 2 or not x.is_contiguous():
            raise ValueError("fp8 lm_head step: x must be a contiguous bf16 [M, K] tensor")
        M, K = x.shape
        if K % _BLK:
            raise ValueError("fp8 lm_head step: K must be a multiple of 128")
        if out is not None and (out.dtype != torch.bfloat16 or out.shape[0] < M or out.shape[1] < n_rows
                                or out.stride(1) != 1):
            raise ValueError("fp8 lm_head step: out must be bf16 [>= M, >= N] with unit column stride")
        if stats_out is None:
            stats_out = (torch.empty(M, dtype=torch.float32, device=x.device),
                         torch.empty(M, dtype=torch.int64, device=x.device),
                         torch.empty(M, dtype=torch.float32, device=x.device))
        mx, arg, lse = stats_out
        if (mx.dtype, arg.dtype, lse.dtype) != (torch.float32, torch.int64, torch.float32) or \
                min(mx.numel(), arg.numel(), lse.numel()) < M:
            raise ValueError("fp8 lm_head step: stats_out must be (fp32 [M], int64 [M], fp32 [M])")
        if packed_out is not None and (packed_out.dtype != torch.float64 or packed_out.numel() < 3 * M
                                       or not packed_out.is_contiguous()):
            raise ValueError("fp8 lm_head step: packed_out must be a contiguous float64 [M, 3]")
        self.x, self.out, self.stats, self.packed = x, out, stats_out, packed_out
        self._wshape, self._sshape = (n_rows, K), (n_rows // _BLK, K // _BLK)
        lib = _lib.lmhead()
        wsp = workspace(x.device)
        self._wsp = wsp
        stream = torch.cuda.current_stream(x.device).cuda_stream
        y_ptr = out.data_ptr() if out is not None else 0
        ldy = out.stride(0) if out is not None else n_rows
        self._head = (x.data_ptr(), M, K)
        if combiner is None:
            self._fn = lib.b200_fp8_lmhead
            self._tail = (n_rows, int(vocab_offset), y_ptr, ldy, mx.data_ptr(), arg.data_ptr(), lse.data_ptr(),
                          None, None, wsp.data_ptr(), wsp.numel(), stream)
        else:
            self._fn = lib.b200_fp8_lmhead_combined
            self._tail = (n_rows, int(vocab_offset), y_ptr, ldy, mx.data_ptr(), arg.data_ptr(), lse.data_ptr(),
                          None, None, wsp.data_ptr(), wsp.numel(), combiner.peers.data_ptr(), combiner.rank,
                          combiner.world, combiner.counters.data_ptr(), combiner.M_cap, stream)
        self._pack = None
        if packed_out is not None:
            self._pack = (lib.b200_pack_row_stats,
                          (mx.data_ptr(), arg.data_ptr(), lse.data_ptr(), M, packed_out.data_ptr(), stream))

    def __call__(self, wq: torch.Tensor, ws: torch.Tensor) -> None:
        if wq.shape != self._wshape or ws.shape != self._sshape:
            raise ValueError("fp8 lm_head step: the weight's shape differs from the prepared one")
        rc = self._fn(*self._head, wq.data_ptr(), ws.data_ptr(), *self._tail)
        if rc != 0:
            raise RuntimeError(f"b200_fp8_lmhead failed rc={rc}")
        if self._pack is not None:
            fn, args = self._pack
            rc = fn(*args)
            if rc != 0:
                raise RuntimeError(f"b200_pack_row_stats failed rc={rc}")
        _lib.debug_check("b200_fp8_lmhead")


def gemm_fp8_block(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor) -> torch.Tensor:
    """bf16 [M, K] @ dequant(W)^T -> bf16 [M, N]; the caller guarantees M <= _MAX_M
    (fp8_target_lmhead.py:70-74). The activation quant runs inside the kernel."""
    _check(x, wq, ws)
    M, K = x.shape
    y = torch.empty(M, wq.shape[0], dtype=torch.bfloat16, device=x.device)
    wsp = workspace(x.device)
    rc = _lib.lmhead().b200_fp8_lmhead(
        _lib.ptr(x), M, K, _lib.ptr(wq), _lib.ptr(ws), wq.shape[0], 0, _lib.ptr(y), y.stride(0),
        None, None, None, None, None, _lib.ptr(wsp), wsp.numel(), _lib.stream_ptr())
    _lib.check(rc, "b200_fp8_lmhead")
    return y


def fp8_block_scaled_mm(qx: torch.Tensor, wq: torch.Tensor, xs: torch.Tensor,
                        ws: torch.Tensor) -> torch.Tensor:
    """Pre-quantized operands through fp8hip_gemm_w8a8_launch's ABI -> bf16 [M, N]."""
    _lib.require_cuda("fp8_block_scaled_mm", qx, wq, xs, ws)
    M, K = qx.shape
    N = wq.shape[0]
    y = torch.empty(M, N, dtype=torch.bfloat16, device=qx.device)
    rc = _lib.lmhead().fp8hip_gemm_w8a8_launch(_lib.ptr(qx), _lib.ptr(wq), _lib.ptr(xs),
                                               _lib.ptr(ws), _lib.ptr(y), M, N, K, _lib.stream_ptr())
    _lib.check(rc, "fp8hip_gemm_w8a8_launch")
    return y


class Fp8TargetHead:
    """Drop-in replacement for the lm_head's quant_method.apply at decode M
    (fp8_target_lmhead.py:77-93)."""

    def __init__(self, orig_method, weight: torch.Tensor, pack_path: str | None = None):
        self.orig = orig_method
        if pack_path is None:
            self.wq, self.ws = pack_fp8_block(weight)
        else:                                   # persisted pack of this weight, else pack + save
            from .packs import cached_fp8
            self.wq, self.ws = cached_fp8(weight, pack_path)
        self.n_fp8 = 0

    def apply(self, layer, x: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
        flat = x.reshape(-1, x.shape[-1])
        if flat.shape[0] > _MAX_M or bias is not None or x.dtype != torch.bfloat16:
            return self.orig.apply(layer, x, bias=bias)
        y = gemm_fp8_block(flat.contiguous(), self.wq, self.ws)
        self.n_fp8 += 1
        return y.reshape(*x.shape[:-1], y.shape[-1])

    def __getattr__(self, name):        # everything else passes through to the original
        return getattr(self.orig, name)

"""CPU restatements of the quantization and lm_head math -- TEST INFRASTRUCTURE ONLY.

Every function is device-agnostic torch code: called on CPU tensors it is the CPU oracle,
called on CUDA tensors (in the GPU tests) it is the "torch-GPU eager restatement" whose
``expf`` and IEEE division are the same device functions the B200 kernels call.

Sources followed (davetha/r9700-lru-expert-cache):
* ``silu_mul_quant``  -- kernels/fused_silu_mul_quant.py:43-57 (rounding spelled out :9-14)
* ``per_token_quant_fp8`` -- vLLM ``scaled_fp8_quant(use_per_token_if_dynamic=True)`` as called by
  ``fp8_quant_shared`` (patches/model_executor/kernels/linear/mxfp4/r4dhip.py.diff L19-34);
  the same scale and division as fused_silu_mul_quant.py:51-57 without the SiLU
* ``group_quant_fp8`` -- vLLM ``per_token_group_quant_fp8`` as called at
  kernels/fp8_target_lmhead.py:73; vLLM 0.22 fp8_utils.py ``_per_token_group_quant_fp8``
  (amax floored at eps, scale = amax * fp32(1/448), q = e4m3(clamp(x / scale)))
* ``pack_fp8_block`` -- kernels/fp8_target_lmhead.py:44-67 (without the gfx1201 shuffle)
* ``fp8_block_gemm_ref`` -- tests/k3/test_fp8sk.py:69,77 (fp32 oracle on the unshuffled W)
* ``quantize_w4`` / ``unpack_w4`` -- kernels/draft_w4_lmhead.py:154-198, 262-285
* ``w4_gemm_ref`` -- tests/k3/w4_verify.py:50 (F.linear of f16-rounded x on the dequant W)

and the B200 packed layouts the kernels read (their own format; the codes, scales and zeros
inside are the reference's):
* FP8: ``[N/16 strips][K/128][16 rows][128 B]``, 16-byte chunk c of row r stored at chunk
  ``c ^ (r & 7)`` (the 128-byte swizzle of a K-major tensor-core operand).
* W4:  ``[N_pad/16 strips][K/128][2 row halves][8 g][4 t][4 words]`` uint32; word w of lane
  (g, t) holds the 8 codes at k = 128*kb + 32*w + 8*t + j, code j in nibble
  ``(j & 1) * 4 + (j >> 1)`` (even k in the low half-word, odd k in the high half-word), as
  offset-binary 0..15. ``wsz`` keeps the reference's dword: f16 scale low, f16 of
  -(1024 + zero) high, ``[N_pad/16, K/128, 16]``.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0
MIN_SCALE = 1.0 / (FP8_MAX * 512.0)        # fused_silu_mul_quant.py:22,96
GROUP_EPS = 1e-10                          # per_token_group_quant_fp8 default eps
BLK = 128                                  # fp8_target_lmhead.py:30
W4_GROUP = 128                             # draft_w4_lmhead.py:70
CLIP_GRID = (1.0, 0.95, 0.9, 0.85, 0.8, 0.75, 0.7, 0.65, 0.6)   # draft_w4_lmhead.py:151


def _amax_rows(xf: torch.Tensor, dim, keepdim: bool = False) -> torch.Tensor:
    """max |x| along `dim` with NaNs ignored (the kernels' and the reference's fmax-based
    reduction: fmax(m, NaN) = m)."""
    a = xf.abs()
    return torch.where(torch.isnan(a), torch.zeros_like(a), a).amax(dim=dim, keepdim=keepdim)


def _clamp_fp8(v: torch.Tensor) -> torch.Tensor:
    """maximum(-448, minimum(v, 448)) with C fmin / fmax semantics (fused_silu_mul_quant.py:56,
    vLLM's fmaxf(-max, fminf(v, max))): a NaN becomes +448."""
    hi = torch.full_like(v, FP8_MAX)
    return torch.fmax(torch.fmin(v, hi), -hi)


# ---------------------------------------------------------------------------------------
# fused SiLU * mul -> FP8
# ---------------------------------------------------------------------------------------

def silu_mul(x: torch.Tensor) -> torch.Tensor:
    """``silu_and_mul`` with the storage-dtype rounding of silu before the multiply and of
    the product on store (fused_silu_mul_quant.py:45-48): ``F.silu`` on the storage dtype
    (one fused ``x / (1 + exp(-x))`` in fp32, rounded on store), then the product of the
    stored values rounded on store. On CUDA tensors this is torch's own silu kernel, the
    same expression vLLM's act_and_mul_kernel evaluates."""
    d = x.shape[1] // 2
    s = F.silu(x[:, :d])
    return (s.float() * x[:, d:].float()).to(x.dtype)


def silu_mul_quant(x: torch.Tensor, write_act: bool = False):
    """(act | None, q e4m3 [rows, d], scale fp32 [rows, 1]) -- per-row scale
    ``max(amax/448, 1/(448*512))`` and a true division (fused_silu_mul_quant.py:51-57)."""
    a = silu_mul(x)
    af = a.float()
    amax = _amax_rows(af, 1, keepdim=True) if af.shape[1] else af.new_zeros(af.shape[0], 1)
    # a true division by 448: a tensor divisor (torch turns a Python-scalar divisor into a
    # reciprocal multiply on CUDA, which is not the reference's `amax / FP8_MAX`)
    scale = torch.clamp_min(amax / torch.full_like(amax, FP8_MAX), MIN_SCALE)
    q = _clamp_fp8(af / scale).to(FP8)
    return (a if write_act else None), q, scale


def group_quant_fp8(x: torch.Tensor, group: int = BLK, eps: float = GROUP_EPS):
    """Per-token group quant: (q e4m3 [M, K], scale fp32 [M, K/group]) row-major."""
    M, K = x.shape
    xf = x.float().reshape(M, K // group, group)
    amax = torch.clamp_min(_amax_rows(xf, -1), eps)
    s = amax * torch.full_like(amax, 1.0 / FP8_MAX)          # amax * fp32(1/448)
    q = _clamp_fp8(xf / s.unsqueeze(-1)).to(FP8).reshape(M, K)
    return q, s.contiguous()


def per_token_quant_fp8(x: torch.Tensor, scale_ub: torch.Tensor | None = None):
    """vLLM ``scaled_fp8_quant(x, use_per_token_if_dynamic=True)`` as fp8_quant_shared calls
    it (r4dhip.py.diff L19-34): row amax (capped by ``scale_ub``), scale = max(amax / 448,
    1/(448*512)) with a true division, q = e4m3(clamp(x / scale)). -> (q [M, K], scale [M, 1])."""
    xf = x.float()
    amax = _amax_rows(xf, 1, keepdim=True) if xf.shape[1] else xf.new_zeros(xf.shape[0], 1)
    if scale_ub is not None:
        amax = torch.fmin(amax, scale_ub.float().reshape(1, 1).to(amax.device))
    scale = torch.clamp_min(amax / torch.full_like(amax, FP8_MAX), MIN_SCALE)
    q = _clamp_fp8(xf / scale).to(FP8)
    return q, scale


def silu_mul_quant_group(x: torch.Tensor, group: int = BLK, write_act: bool = False):
    """SiLU*mul followed by the per-token group-128 quant of the stored activation."""
    a = silu_mul(x)
    q, s = group_quant_fp8(a, group)
    return (a if write_act else None), q, s


# ---------------------------------------------------------------------------------------
# FP8 128x128 block-scaled lm_head
# ---------------------------------------------------------------------------------------

def pack_fp8_block(w: torch.Tensor):
    """bf16 [N, K] -> (e4m3 [N, K] row-major, fp32 [N/128, K/128]) per
    fp8_target_lmhead.py:56-65: scale = max(amax, 1e-12) / 448, w_q = e4m3(clamp(w/scale))."""
    N, K = w.shape
    assert N % BLK == 0 and K % BLK == 0, (N, K)
    out = torch.empty(N, K, dtype=FP8)
    ws = torch.empty(N // BLK, K // BLK, dtype=torch.float32)
    rows = 4096
    for r0 in range(0, N, rows):
        r1 = min(N, r0 + rows)
        wf = w[r0:r1].float().view((r1 - r0) // BLK, BLK, K // BLK, BLK)
        amax = wf.abs().amax(dim=(1, 3), keepdim=True).clamp(min=1e-12)
        scale = amax / FP8_MAX
        out[r0:r1] = (wf / scale).clamp(-FP8_MAX, FP8_MAX).to(FP8).view(r1 - r0, K)
        ws[r0 // BLK:r1 // BLK] = scale.view((r1 - r0) // BLK, K // BLK)
    return out, ws


def fp8_tile_swizzle(wq_rowmajor: torch.Tensor) -> torch.Tensor:
    """Row-major e4m3 [N, K] -> the B200 strip layout (bytes, viewed [N, K])."""
    N, K = wq_rowmajor.shape
    b = wq_rowmajor.view(torch.uint8).reshape(N // 16, 16, K // 128, 8, 16)  # st, r, kb, c, byte
    r = torch.arange(16).view(1, 16, 1, 1)
    c = torch.arange(8).view(1, 1, 1, 8)
    dst_c = (c ^ (r & 7)).expand(N // 16, 16, K // 128, 8)
    out = torch.empty_like(b)
    out.scatter_(3, dst_c.unsqueeze(-1).expand_as(b), b)
    return out.permute(0, 2, 1, 3, 4).contiguous().view(FP8).view(N, K)


def fp8_tile_unswizzle(wq_packed: torch.Tensor) -> torch.Tensor:
    """Inverse of ``fp8_tile_swizzle``."""
    N, K = wq_packed.shape
    b = wq_packed.contiguous().view(torch.uint8).reshape(N // 16, K // 128, 16, 8, 16)
    b = b.permute(0, 2, 1, 3, 4)                                            # st, r, kb, c', byte
    r = torch.arange(16).view(1, 16, 1, 1)
    c = torch.arange(8).view(1, 1, 1, 8)
    src_c = (c ^ (r & 7)).expand(N // 16, 16, K // 128, 8)
    out = torch.gather(b, 3, src_c.unsqueeze(-1).expand(N // 16, 16, K // 128, 8, 16))
    return out.reshape(N, K).view(FP8)


def dequant_fp8_block(wq: torch.Tensor, ws: torch.Tensor) -> torch.Tensor:
    """fp32 W = w_q * ws broadcast over 128x128 blocks (tests/k3/test_fp8sk.py:69)."""
    return wq.float() * ws.repeat_interleave(BLK, 0).repeat_interleave(BLK, 1)


def fp8_block_gemm_ref(qx: torch.Tensor, xs: torch.Tensor, wdq: torch.Tensor) -> torch.Tensor:
    """fp32 logits ``(qx * xs) @ W^T`` (tests/k3/test_fp8sk.py:77)."""
    return (qx.float() * xs.repeat_interleave(BLK, 1)) @ wdq.T


def row_stats(logits: torch.Tensor, n_valid: int | None = None):
    """(max, first-index argmax, logsumexp) per row of fp32 logits, computed in float64."""
    lg = logits.double()
    if n_valid is not None:
        lg = lg[:, :n_valid]
    mx, idx = lg.max(dim=1)          # torch returns the first maximal index
    lse = torch.logsumexp(lg, dim=1)
    return mx.float(), idx.to(torch.int32), lse.float()


def top2_gap(logits: torch.Tensor) -> torch.Tensor:
    """Per-row gap between the largest and second-largest logit (argmax robustness)."""
    t = torch.topk(logits.double(), 2, dim=1).values
    return (t[:, 0] - t[:, 1]).float()


# ---------------------------------------------------------------------------------------
# W4 group-128 draft lm_head
# ---------------------------------------------------------------------------------------

def quantize_w4(w: torch.Tensor, group: int = W4_GROUP, clip_grid=None):
    """[N, K] -> (q uint8 0..15, scale f16 [N, K/g], zero int16 [N, K/g]).

    Asymmetric per (row, group); clip fraction chosen per (row, group) by squared error;
    the f16 rounding of the scale is applied before the codes are chosen
    (draft_w4_lmhead.py:154-198)."""
    n, k = w.shape
    assert k % group == 0
    wf = w.float().view(n, k // group, group)
    lo, hi = wf.amin(-1), wf.amax(-1)
    mid, half = (hi + lo) / 2, (hi - lo) / 2
    best_err = torch.full_like(lo, float("inf"))
    best_scale = torch.zeros_like(lo, dtype=torch.float16)
    best_zero = torch.zeros_like(lo)
    for c in (clip_grid if clip_grid is not None else CLIP_GRID):
        lo_c, hi_c = mid - c * half, mid + c * half
        scale = ((hi_c - lo_c) / 15.0).clamp(min=0.0).half()
        flat = (scale.float() == 0) & (lo != 0)          # constant non-zero group -> code 8
        scale = torch.where(flat, (lo.abs() / 7.0).half(), scale)
        sf = scale.float()
        inv = torch.where(sf > 0, 1.0 / sf.clamp(min=1e-30), torch.zeros_like(sf))
        zero = torch.where(flat, torch.full_like(lo, 8.0),
                           torch.round(-lo_c * inv)).clamp_(-1024, 1024)
        q = torch.round(wf * inv.unsqueeze(-1) + zero.unsqueeze(-1)).clamp_(0, 15)
        err = ((q - zero.unsqueeze(-1)) * sf.unsqueeze(-1) - wf).square().sum(-1)
        take = err < best_err
        best_err = torch.where(take, err, best_err)
        best_scale = torch.where(take, scale, best_scale)
        best_zero = torch.where(take, zero, best_zero)
    sf = best_scale.float()
    inv = torch.where(sf > 0, 1.0 / sf.clamp(min=1e-30), torch.zeros_like(sf))
    q = torch.round(wf * inv.unsqueeze(-1) + best_zero.unsqueeze(-1)).clamp_(0, 15)
    return q.to(torch.uint8).view(n, k), best_scale, best_zero.to(torch.int16)


def quantize_w4_sym(w: torch.Tensor, group: int = W4_GROUP):
    """[N, K] -> (q uint8 0..15 standing for q - 8, scale bf16 [N, K/g]).

    The symmetric int4 format with bf16 group scales that the benchmark's draft-head
    configuration names (restated from that description: the reference module packs only its
    asymmetric f16 scale + zero format, so there is no reference implementation to pin this
    one to): per (row, group of 128) scale = bf16(amax / 7), q = clamp(round(w / scale), -8, 7)
    + 8 by true division and round-half-even; an all-zero group keeps scale 0 and code 8."""
    n, k = w.shape
    assert k % group == 0
    wf = w.float().view(n, k // group, group)
    scale = (wf.abs().amax(-1) / 7.0).to(torch.bfloat16)
    sf = scale.float().unsqueeze(-1)
    r = torch.where(sf > 0, wf / torch.where(sf > 0, sf, torch.ones_like(sf)), torch.zeros_like(wf))
    q = torch.round(r).clamp_(-8, 7) + 8
    return q.to(torch.uint8).view(n, k), scale


def w4_dequant_sym(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """(q - 8) * scale, fp32 [N, K]."""
    n, k = q.shape
    ng = scale.shape[1]
    return ((q.float().view(n, ng, k // ng) - 8.0) * scale.float().unsqueeze(-1)).view(n, k)


def w4_dequant(q: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """fp32 ``(q - zero) * scale`` per (row, group) (draft_w4_lmhead.py:49-50, 281)."""
    n, k = q.shape
    g = k // scale.shape[1]
    return ((q.float().view(n, -1, g) - zero.float().unsqueeze(-1))
            * scale.float().unsqueeze(-1)).view(n, k)


def pack_sz(scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """(f16 scale, integer zero) [N, K/g] -> int32 [N/16, K/g, 16]: f16 scale bits low,
    f16 bits of -(1024 + zero) high (draft_w4_lmhead.py:215-225)."""
    n, ng = scale.shape
    sb = scale.contiguous().view(torch.int16).to(torch.int64) & 0xFFFF
    nz = (-(1024.0 + zero.float())).half().view(torch.int16).to(torch.int64) & 0xFFFF
    dw = sb | (nz << 16)
    dw = torch.where(dw >= 2 ** 31, dw - 2 ** 32, dw).to(torch.int32)
    return dw.view(n // 16, 16, ng).permute(0, 2, 1).contiguous()


def unpack_sz(wsz: torch.Tensor):
    """Inverse of ``pack_sz`` -> (scale f16 [N, ng], zero fp32 [N, ng])."""
    nt, ng, _ = wsz.shape
    sz = wsz.permute(0, 2, 1).reshape(nt * 16, ng)
    scale = (sz & 0xFFFF).to(torch.int16).view(torch.float16)
    zero = -(sz >> 16).to(torch.int16).view(torch.float16).float() - 1024.0
    return scale, zero


# nibble position of code j (0..7) inside a B200 W4 word: even k low half-word, odd k high
W4_NIBBLE = [(j & 1) * 4 + (j >> 1) for j in range(8)]


def pack_codes_b200(q: torch.Tensor) -> torch.Tensor:
    """uint8 codes [N_pad, K] (0..15) -> uint32-as-int32 [N_pad/16, K/128, 2, 8, 4, 4]."""
    n, k = q.shape
    c = q.to(torch.int64).view(n // 16, 2, 8, k // 128, 4, 4, 8)   # st, half, g, kb, w, t, j
    c = c.permute(0, 3, 1, 2, 5, 4, 6)                            # st, kb, half, g, t, w, j
    shifts = torch.tensor(W4_NIBBLE, dtype=torch.int64) * 4
    word = (c << shifts).sum(-1)
    word = torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)
    return word.contiguous()


def unpack_codes_b200(wq: torch.Tensor, n_pad: int, k: int) -> torch.Tensor:
    """Inverse of ``pack_codes_b200`` -> uint8 [N_pad, K]."""
    w = wq.reshape(n_pad // 16, k // 128, 2, 8, 4, 4).to(torch.int64) & 0xFFFFFFFF
    shifts = torch.tensor(W4_NIBBLE, dtype=torch.int64) * 4
    c = (w.unsqueeze(-1) >> shifts) & 0xF                            # st, kb, half, g, t, w, j
    c = c.permute(0, 2, 3, 1, 5, 4, 6)                              # st, half, g, kb, w, t, j
    return c.reshape(n_pad, k).to(torch.uint8)


def w4_gemm_ref(x: torch.Tensor, wdq: torch.Tensor) -> torch.Tensor:
    """fp32 logits of the f16-rounded activation on the dequantized W
    (tests/k3/w4_verify.py:50: ``F.linear(x.float().half().float(), wref)``)."""
    return x.float().half().float() @ wdq.T

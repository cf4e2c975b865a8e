"""W4 group-128 draft lm_head: the host-side mirror of kernels/draft_w4_lmhead.py
(``GROUP``, ``MAX_M``, ``PackedW4``, ``available``, ``quantize_w4``, ``pack_w4a16``,
``unpack_w4``, ``_legal``, ``pick_cfg``, ``torch.ops.vllm.draft_w4_lmhead_gemm``,
``gemm_w4a16``), backed by the sm_100a GEMV of csrc/lmhead.cu (``b200_w4_lmhead``; the
reference's C entry ``r4d_gemm_w4a16_nt_m64`` is exported with the same ABI).

Quantizer: the reference's codes (draft_w4_lmhead.py:154-198) -- asymmetric per (row, group
of 128), clip fraction chosen by squared error, the f16 rounding of the scale folded in before
the codes, integer zero in [-1024, 1024], codes 0..15, dequant ``(q - zero) * scale`` --
computed for all clip fractions at once.
The activation is rounded to f16 exactly as ``x.to(float16)`` (draft_w4_lmhead.py:31-39),
inside the kernel.

Layout: the reference packs nibbles in gfx1201 WMMA fragment order. The B200 pack is
``[N_pad/16][K/128][2][8 g][4 t][4 words]`` u32 (``N_pad * K / 2`` bytes, the same size):
word w of lane (g, t) holds the codes of k = 128kb + 32w + 8t + j, code j in nibble
``(j & 1) * 4 + (j >> 1)`` as offset binary, so one 128-bit shared load gives a lane its A
fragments and ``(word >> 4i) & 0x000F000F | 0x64006400`` widens two codes to f16 at once.
``wsz`` keeps the reference's dword exactly (f16 scale | f16 of -(1024 + zero) << 16,
[N_pad/16, K/128, 16]).

The launch-config helpers keep the reference's signatures, legality rules and choices so
callers and env overrides behave the same; the B200 kernel plans its own launch.
"""
from __future__ import annotations

import functools
import os
from dataclasses import dataclass

import torch

from . import _lib
from ._workspace import workspace

GROUP = 128
MAX_M = 64
_WAVE32 = 32
_MAX_THREADS = 1024
_MAX_SMEM = 64 * 1024

_CLIP_GRID = (1.0, 0.95, 0.9, 0.85, 0.8, 0.75, 0.7, 0.65, 0.6)


@dataclass(frozen=True)
class PackedW4:
    """Everything ``gemm_w4a16`` needs; hold this on the layer. ``sym`` marks the symmetric
    format (pack_w4a16_sym): ``wsz`` then holds bf16 scales and every zero is 8."""
    wq: torch.Tensor     # uint8  [N_pad/16, K/128, 1024]  (= N_pad*K/2 bytes)
    wsz: torch.Tensor    # int32  [N_pad/16, K/128, 16]  (bf16 [N_pad/16, K/128, 16] when sym)
    n: int
    n_pad: int
    k: int
    sym: bool = False

    @property
    def nbytes(self) -> int:
        return self.wq.numel() + self.wsz.numel() * self.wsz.element_size()


@functools.lru_cache(maxsize=1)
def _fns():
    """The bound kernel entry, or None when disabled / unavailable (draft_w4_lmhead.py:99-131)."""
    global GROUP, MAX_M
    if os.environ.get("VLLM_DRAFT_W4_LMHEAD", "1") != "1":
        return None
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        return None
    try:
        lib = _lib.lmhead()
    except _lib.NativeLibraryError:
        return None
    MAX_M = int(lib.r4d_gemm_w4a16_nt_m64_max_m())
    GROUP = int(lib.r4d_gemm_w4a16_nt_m64_group())
    return lib.b200_w4_lmhead


def available() -> bool:
    """True when pack_w4a16 / gemm_w4a16 can use the kernel on this machine."""
    return _fns() is not None


# ---------------------------------------------------------------------------------------
# packing (load time, on the weight's device)
# ---------------------------------------------------------------------------------------

def quantize_w4(w: torch.Tensor, group: int = 0, clip_grid: tuple[float, ...] | None = None
                ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """[N, K] -> (q uint8 in 0..15, scale f16 [N, K/group], zero int16 [N, K/group]).

    The reference's quantizer (draft_w4_lmhead.py:154-198), evaluated for every clip fraction
    at once: candidate c of a (row, group) spans [mid - c r, mid + c r] around the group's
    midpoint mid and half-range r; its scale is that span / 15 rounded to f16 (a constant
    non-zero group instead gets |lo| / 7 and code 8 for its value), its zero the integer
    nearest to -start / scale within [-1024, 1024], its codes round(w / scale + zero) in 0..15;
    the candidate with the smallest squared dequantization error wins (the first one on a tie).
    An all-zero group keeps scale 0, codes 0. Same fp32 operations, so the same codes."""
    group = group or GROUP
    n, k = w.shape
    assert k % group == 0, f"K={k} must be a multiple of the group {group}"
    ng = k // group
    vals = w.float().view(n, ng, 1, group)
    lo, hi = vals.amin(-1, keepdim=True), vals.amax(-1, keepdim=True)          # [n, ng, 1, 1]
    fr = torch.tensor(clip_grid if clip_grid is not None else _CLIP_GRID, dtype=torch.float32,
                      device=w.device).view(1, 1, -1, 1)
    mid, rad = (hi + lo) / 2, (hi - lo) / 2
    start = mid - fr * rad                                                     # [n, ng, C, 1]
    step = ((mid + fr * rad - start) / 15.0).clamp(min=0.0).half()
    const = (step.float() == 0) & (lo != 0)
    step = torch.where(const, (lo.abs() / 7.0).half(), step)
    sf = step.float()
    rcp = torch.where(sf > 0, 1.0 / sf.clamp(min=1e-30), torch.zeros_like(sf))
    zero = torch.where(const, torch.full_like(start, 8.0), torch.round(-start * rcp)).clamp_(-1024, 1024)
    q = torch.round(vals * rcp + zero).clamp_(0, 15)                           # [n, ng, C, group]
    err = ((q - zero) * sf - vals).square().sum(-1, keepdim=True)              # [n, ng, C, 1]
    pick = err.argmin(dim=2, keepdim=True)                                     # first minimum
    q = q.gather(2, pick.expand(n, ng, 1, group))
    scale = step.gather(2, pick).view(n, ng)
    zero = zero.gather(2, pick).view(n, ng)
    return q.to(torch.uint8).view(n, k), scale, zero.to(torch.int16)


_NIBBLE = (0, 4, 1, 5, 2, 6, 3, 7)   # nibble of code j: (j & 1) * 4 + (j >> 1)


def _pack_codes(codes: torch.Tensor) -> torch.Tensor:
    """uint8 codes [R, K] (0..15, R % 16 == 0) -> uint8 [R/16, K/128, 1024] (B200 words)."""
    r, k = codes.shape
    c = codes.to(torch.int32).view(r // 16, 2, 8, k // 128, 4, 4, 8)    # st, half, g, kb, w, t, j
    c = c.permute(0, 3, 1, 2, 5, 4, 6)                                 # st, kb, half, g, t, w, j
    shifts = torch.tensor(_NIBBLE, dtype=torch.int32, device=codes.device) * 4
    word = (c << shifts).sum(-1, dtype=torch.int32)
    return word.contiguous().view(torch.uint8).view(r // 16, k // 128, 1024)


def _unpack_codes(wq: torch.Tensor, n_pad: int, k: int, t0: int = 0, t1: int | None = None) -> torch.Tensor:
    t1 = n_pad // 16 if t1 is None else t1
    w = wq[t0:t1].contiguous().view(torch.int32).view(t1 - t0, k // 128, 2, 8, 4, 4)
    shifts = torch.tensor(_NIBBLE, dtype=torch.int32, device=wq.device) * 4
    c = (w.unsqueeze(-1) >> shifts) & 0xF                               # st, kb, half, g, t, w, j
    return c.permute(0, 2, 3, 1, 5, 4, 6).reshape((t1 - t0) * 16, k).to(torch.uint8)


def _pack_sz(scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    """(f16 scale, integer zero) [N, K/GROUP] -> int32 [N/16, K/GROUP, 16]: the reference's
    dword (draft_w4_lmhead.py:215-225), low half the scale's f16 bits, high half the f16 of
    -(1024 + zero) (exact for |zero| <= 1024), built as two int16 halves viewed as one int32."""
    n, ng = scale.shape
    halves = torch.stack((scale.contiguous().view(torch.int16),
                          (-(1024.0 + zero.float())).half().view(torch.int16)), dim=-1)
    return halves.view(torch.int32).view(n // 16, 16, ng).transpose(1, 2).contiguous()


def pack_w4a16(weight: torch.Tensor, group: int = 0, chunk_tiles: int = 64,
               clip_grid: tuple[float, ...] | None = None) -> PackedW4:
    """[N, K] bf16/f32 lm_head weight -> PackedW4 in the B200 layout. N is padded to a
    multiple of 16 with zero rows; chunked over 16-row tiles to bound the transient (the
    quantizer holds every clip candidate: ~36 x the chunk's fp32 bytes)."""
    assert weight.dim() == 2, f"expected [N, K], got {tuple(weight.shape)}"
    _fns()
    group = group or GROUP
    n, k = weight.shape
    if k % 128 or k % group or group != 128:
        raise ValueError(f"draft_w4_lmhead: K={k} must be a multiple of 128 (group 128)")
    n_pad = (n + 15) // 16 * 16
    dev = weight.device
    wq_out = torch.empty((n_pad // 16, k // 128, 1024), dtype=torch.uint8, device=dev)
    sz_out = torch.empty((n_pad // 16, k // group, 16), dtype=torch.int32, device=dev)
    rows = chunk_tiles * 16
    for r0 in range(0, n_pad, rows):
        r1 = min(r0 + rows, n_pad)
        w = weight[r0:min(r1, n)]
        if w.shape[0] < r1 - r0:
            w = torch.cat([w, w.new_zeros(r1 - r0 - w.shape[0], k)], 0)
        q, scale, zero = quantize_w4(w, group, clip_grid)
        wq_out[r0 // 16:r1 // 16] = _pack_codes(q)
        sz_out[r0 // 16:r1 // 16] = _pack_sz(scale, zero)
        del q, scale, zero, w
    return PackedW4(wq=wq_out, wsz=sz_out, n=n, n_pad=n_pad, k=k)


def quantize_w4_sym(w: torch.Tensor, group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """[N, K] -> (q uint8 in 0..15 meaning q - 8, scale bf16 [N, K/group]): symmetric int4 per
    (row, group) with a bf16 scale = amax / 7 (the benchmark's draft-head format); codes by true
    division and round-half-even, clamped to [-8, 7]; an all-zero group keeps scale 0."""
    group = group or GROUP
    n, k = w.shape
    assert k % group == 0, f"K={k} must be a multiple of the group {group}"
    wf = w.float().view(n, k // group, group)
    scale = (wf.abs().amax(-1) / 7.0).to(torch.bfloat16)
    sf = scale.float().unsqueeze(-1)
    ratio = torch.where(sf > 0, wf / torch.where(sf > 0, sf, torch.ones_like(sf)), torch.zeros_like(wf))
    q = torch.round(ratio).clamp_(-8, 7) + 8
    return q.to(torch.uint8).view(n, k), scale


def pack_w4a16_sym(weight: torch.Tensor, group: int = 0, chunk_tiles: int = 512) -> PackedW4:
    """[N, K] lm_head weight -> PackedW4 in the symmetric format (bf16 group scales, zero 8):
    the same code layout as pack_w4a16, scales as bf16 [N_pad/16, K/128, 16]."""
    assert weight.dim() == 2, f"expected [N, K], got {tuple(weight.shape)}"
    _fns()
    group = group or GROUP
    n, k = weight.shape
    if k % 128 or k % group or group != 128:
        raise ValueError(f"draft_w4_lmhead: K={k} must be a multiple of 128 (group 128)")
    n_pad = (n + 15) // 16 * 16
    dev = weight.device
    wq_out = torch.empty((n_pad // 16, k // 128, 1024), dtype=torch.uint8, device=dev)
    sc_out = torch.empty((n_pad // 16, k // group, 16), dtype=torch.bfloat16, device=dev)
    rows = chunk_tiles * 16
    for r0 in range(0, n_pad, rows):
        r1 = min(r0 + rows, n_pad)
        w = weight[r0:min(r1, n)]
        if w.shape[0] < r1 - r0:
            w = torch.cat([w, w.new_zeros(r1 - r0 - w.shape[0], k)], 0)
        q, scale = quantize_w4_sym(w, group)
        wq_out[r0 // 16:r1 // 16] = _pack_codes(q)
        sc_out[r0 // 16:r1 // 16] = scale.view((r1 - r0) // 16, 16, k // group).permute(0, 2, 1)
        del q, scale, w
    return PackedW4(wq=wq_out, wsz=sc_out, n=n, n_pad=n_pad, k=k, sym=True)


def unpack_w4(packed: PackedW4, dtype: torch.dtype = torch.bfloat16,
              rows: slice | None = None) -> torch.Tensor:
    """Dequantize back to [N_pad, K] -- the inverse of pack_w4a16, for the numeric reference
    (draft_w4_lmhead.py:262-285). ``rows`` selects a slice of rows."""
    k = packed.k
    nt_all = packed.n_pad // 16
    t0, t1 = (0, nt_all) if rows is None else (rows.start // 16, -(-rows.stop // 16))
    t1 = min(t1, nt_all)
    q = _unpack_codes(packed.wq, packed.n_pad, k, t0, t1).float()
    ng = packed.wsz.shape[1]
    sz = packed.wsz[t0:t1].permute(0, 2, 1).reshape((t1 - t0) * 16, ng)
    if packed.sym:
        scale = sz.float()
        zero = torch.full_like(scale, 8.0)
    else:
        scale = (sz & 0xFFFF).to(torch.int16).view(torch.float16).float()
        zero = -(sz >> 16).to(torch.int16).view(torch.float16).float() - 1024.0
    w = (q.view((t1 - t0) * 16, ng, k // ng) - zero.unsqueeze(-1)) * scale.unsqueeze(-1)
    w = w.view((t1 - t0) * 16, k).to(dtype)
    if rows is not None:
        w = w[rows.start - t0 * 16:rows.stop - t0 * 16]
    return w


# ---------------------------------------------------------------------------------------
# launch configuration (reference signatures and legality; draft_w4_lmhead.py:292-344)
# ---------------------------------------------------------------------------------------

def _legal(k: int, ntiles: int, wv: int, sk: int, npw: int) -> bool:
    """The reference's resource rules for a (waves, split-K, tiles per wave) launch: K splits
    into sk whole groups per wave, a block holds at most 1024 threads of 32-wide waves and 64 KB
    of shared memory (1 KB per wave, tile and split), npw is 1 or 4, and the waves' tiles do not
    outnumber the N tiles."""
    threads = wv * sk * _WAVE32
    smem = wv * npw * sk * 1024
    return (min(wv, sk) >= 1 and npw in (1, 4) and k % (sk * GROUP) == 0
            and threads <= _MAX_THREADS and smem <= _MAX_SMEM and wv * npw <= max(1, ntiles))


@functools.lru_cache(maxsize=None)
def pick_cfg(m: int, n_pad: int, k: int) -> tuple[int, int, int, int]:
    """(WV, SK, NPW, NT) as the reference picks it for gfx1201 (draft_w4_lmhead.py:292-344),
    so that callers and the R4D_W4_LMHEAD_CFG="WV,SK,NPW,NT" override behave the same; the
    B200 kernel validates the choice and plans its own launch. Rule: one wave, one tile pass;
    up to 16 rows the deepest split-K of (10, 4, 2, 1) that K allows, above 16 rows four
    tiles per wave with split-K 4, 2 or 1 (split-K 4 or 1 with one tile per wave once the
    tiles run short); else a heuristic fill of the block."""
    ntiles = n_pad // 16
    override = os.environ.get("R4D_W4_LMHEAD_CFG")
    if override:
        try:
            wv, sk, npw, nt = (int(v) for v in override.split(","))
        except ValueError:
            wv = sk = npw = nt = 0
        if _legal(k, ntiles, wv, sk, npw) and nt in (0, 1):
            return wv, sk, npw, nt
    if m <= 16:
        tries = [(sk, 1) for sk in (10, 4, 2, 1)]
    else:
        tries = [(sk, 4) for sk in (4, 2, 1)] + [(4, 1), (1, 1)]
    for sk, npw in tries:
        if _legal(k, ntiles, 1, sk, npw):
            return 1, sk, npw, 1
    sk = next((s for s in (4, 2, 1) if k % (s * GROUP) == 0), 1)
    wv = max(1, min(8, _MAX_THREADS // (sk * _WAVE32), _MAX_SMEM // (sk * 1024), ntiles))
    return wv, sk, 1, 1


# ---------------------------------------------------------------------------------------
# the op
# ---------------------------------------------------------------------------------------

def _run(x: torch.Tensor, wq: torch.Tensor, wsz: torch.Tensor, n: int, k: int,
         stats: bool, vocab_offset: int = 0, y: torch.Tensor | None = None):
    fn = _fns()
    if fn is None:
        raise RuntimeError("draft_w4_lmhead: the B200 kernel is unavailable on this machine")
    sym = wsz.dtype == torch.bfloat16                       # the symmetric format's scales
    if sym:
        fn = _lib.lmhead().b200_w4_lmhead_sym
    _lib.require_cuda("draft_w4_lmhead", x, wq, wsz)
    m = x.shape[0]
    n_pad = wq.shape[0] * 16
    if x.dtype not in (torch.bfloat16, torch.float16):
        x = x.to(torch.bfloat16)
    x = x.contiguous()
    if y is None:
        y = torch.empty((m, n_pad), dtype=torch.bfloat16, device=x.device)
    mx = arg = lse = None
    wsp = None
    if stats:
        mx = torch.empty(m, dtype=torch.float32, device=x.device)
        arg = torch.empty(m, dtype=torch.int64, device=x.device)
        lse = torch.empty(m, dtype=torch.float32, device=x.device)
        wsp = workspace(x.device)
    rc = fn(_lib.ptr(x), 0 if x.dtype == torch.bfloat16 else 1, m, k, _lib.ptr(wq), _lib.ptr(wsz),
            n_pad, n, int(vocab_offset), _lib.ptr(y), y.stride(0), _lib.ptr(mx), _lib.ptr(arg),
            _lib.ptr(lse), _lib.ptr(wsp), 0 if wsp is None else wsp.numel(), _lib.stream_ptr())
    _lib.check(rc, "b200_w4_lmhead_sym" if sym else "b200_w4_lmhead")
    _lib.debug_check("b200_w4_lmhead")
    return y, mx, arg, lse


def _draft_w4_lmhead_gemm(x: torch.Tensor, wq: torch.Tensor, wsz: torch.Tensor, n: int, k: int,
                          wv: int, sk: int, npw: int, nt: int) -> torch.Tensor:
    """One opaque op (draft_w4_lmhead.py:351-377). Every M runs on the B200 kernel (in
    16-token passes); the reference's launch-knob contract is still asserted."""
    assert k % (sk * GROUP) == 0 and wv * sk * _WAVE32 <= _MAX_THREADS and npw in (1, 4) \
        and wv * npw * sk * 256 * 4 <= _MAX_SMEM
    y, _, _, _ = _run(x, wq, wsz, n, k, stats=False)
    n_pad = wq.shape[0] * 16
    return y if n_pad == n else y[:, :n].contiguous()


def _register_op() -> None:
    if hasattr(torch.ops.vllm, "draft_w4_lmhead_gemm"):
        return

    @torch.library.custom_op("vllm::draft_w4_lmhead_gemm", mutates_args=())
    def _op(x: torch.Tensor, wq: torch.Tensor, wsz: torch.Tensor, n: int, k: int, wv: int,
            sk: int, npw: int, nt: int) -> torch.Tensor:
        return _draft_w4_lmhead_gemm(x, wq, wsz, n, k, wv, sk, npw, nt)

    @_op.register_fake
    def _fake(x, wq, wsz, n, k, wv, sk, npw, nt):
        return torch.empty((x.size(0), n), dtype=torch.bfloat16, device=x.device)


_register_op()


def gemm_w4a16(x: torch.Tensor, packed: PackedW4) -> torch.Tensor:
    """[n_tokens, K] bf16 hidden states -> [n_tokens, N] bf16 logits (draft_w4_lmhead.py:393-403).
    No host sync and no allocation beyond the output: safe inside a CUDA-graph capture."""
    _fns()
    assert x.dim() == 2 and x.shape[1] == packed.k, f"expected [*, {packed.k}], got {tuple(x.shape)}"
    wv, sk, npw, nt = pick_cfg(min(x.shape[0], MAX_M + 1), packed.n_pad, packed.k)
    return torch.ops.vllm.draft_w4_lmhead_gemm(x, packed.wq, packed.wsz, packed.n, packed.k,
                                               wv, sk, npw, nt)


def gemm_w4a16_top(x: torch.Tensor, packed: PackedW4, vocab_offset: int = 0,
                   want_logits: bool = True):
    """Fused draft head: (logits [M, n] | None, row max, argmax int64 (+ vocab_offset),
    logsumexp) in one pass over the packed weight; padding rows never win the argmax."""
    assert x.dim() == 2 and x.shape[1] == packed.k
    y, mx, arg, lse = _run(x, packed.wq, packed.wsz, packed.n, packed.k, stats=True,
                           vocab_offset=vocab_offset)
    logits = None
    if want_logits:
        logits = y if packed.n_pad == packed.n else y[:, :packed.n]
    return logits, mx, arg, lse

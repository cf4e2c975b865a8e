"""The FP8 lm_head entry with built-in scratch (b200_fp8_lmhead_static_scratch), called through
the C ABI, against the workspace entry b200_fp8_lmhead on the same inputs.

Both entries run the same kernels with the same work split on the same operands, so every
output must be identical, bit for bit: logits, row max, argmax, logsumexp and the quantized
activation. Three calls in a row share the static array: the tcgen05 path at M=40, the GEMV
path at M=5, then the tcgen05 path again at M=64, which must not read anything the earlier
calls left in the array. Sizes beyond the array are refused with -9. The file name sorts last
so that the test also runs after every other GPU test in one session."""
from __future__ import annotations

import pytest
import torch

from conftest import load_pkg

pytestmark = pytest.mark.gpu
P = load_pkg()
F8 = P.fp8_target_lmhead
L = P._lib


def _outputs(M, N, K, dev):
    return (torch.empty(M, N, device=dev, dtype=torch.bfloat16),
            torch.empty(M, device=dev, dtype=torch.float32),
            torch.empty(M, device=dev, dtype=torch.int64),
            torch.empty(M, device=dev, dtype=torch.float32),
            torch.empty(M, K, device=dev, dtype=torch.uint8),
            torch.empty(M, K // 128, device=dev, dtype=torch.float32))


def _call(lib, static, x, wq, ws, N, off, outs, ws_buf=None):
    y, mx, arg, lse, qx, xs = outs
    M, K = x.shape
    args = [L.ptr(x), M, K, L.ptr(wq), L.ptr(ws), N, off, L.ptr(y), N, L.ptr(mx), L.ptr(arg),
            L.ptr(lse), L.ptr(qx), L.ptr(xs)]
    if static:
        return lib.b200_fp8_lmhead_static_scratch(*args, L.stream_ptr())
    return lib.b200_fp8_lmhead(*args, L.ptr(ws_buf), ws_buf.numel(), L.stream_ptr())


def test_static_scratch_matches_workspace_entry(cuda):
    lib = L.lmhead()
    N, K, off = 4096, 2560, 1 << 16
    g = torch.Generator(device=cuda).manual_seed(4242)
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    wq, ws = F8.pack_fp8_block(w)
    ws_buf = torch.zeros(lib.b200_lmhead_workspace_bytes(), device=cuda, dtype=torch.uint8)
    for M in (40, 5, 64):                   # tcgen05 path, the GEMV path, tcgen05 again
        x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16, generator=g)
        a, b = _outputs(M, N, K, cuda), _outputs(M, N, K, cuda)
        assert _call(lib, False, x, wq, ws, N, off, a, ws_buf) == 0
        assert _call(lib, True, x, wq, ws, N, off, b) == 0
        torch.cuda.synchronize()
        assert lib.b200_lmhead_error(1) == 0
        for name, u, v in zip(("logits", "max", "argmax", "lse", "q", "scales"), a, b):
            assert torch.equal(u, v), (M, name)


def test_static_scratch_rejects_large_k(cuda):
    lib = L.lmhead()
    N, K, M = 128, 16384 + 128, 1
    x = torch.zeros(M, K, device=cuda, dtype=torch.bfloat16)
    wq = torch.zeros(N, K, device=cuda, dtype=torch.uint8)
    ws = torch.zeros(1, K // 128, device=cuda, dtype=torch.float32)
    assert _call(lib, True, x, wq, ws, N, 0, _outputs(M, N, K, cuda)) == -9

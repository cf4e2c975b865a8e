"""GPU parity of the MoE block tail: the shared-expert gate kernels (csrc/gate.cu, through
fused_gate_mul.py) and moe_sum (csrc/moe_sum.cu, through moe_ops.py; bit-exact against the
oracle, torch.sum over top_k and vLLM's ops.moe_sum where it loads).

sigmoid_gate_mul: bit-identical to the stock ``F.sigmoid(g) * out`` on the GPU, the
reference's own check (tests/k4/test_gate_mul.py:24-37: H = 2560, T in (1, 4, 20, 64, 2048),
gate scales (0.02, 1, 30)), for bf16, f16 and f32, and to the oracle on the same tensors;
plus ragged widths, strided and unaligned rows, non-finite values, no rows, and one launch
per call (test_gate_mul.py:39-44).

gemv_sigmoid_gate_mul: not bit-identical by design (the gate dot's fp32 summation order is
the kernel's, fused_gate_mul.py:84-88). Every row must equal the oracle's output for the
correctly rounded gate or for a gate one ulp of the dtype away, and at least 90 % of rows
must use the correctly rounded gate; f32 within the error bound of the kernel's fp32 dot
(32 * 2^-24 * sum|x w|, carried through the sigmoid) of the float64-dot oracle."""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F
from torch.profiler import ProfilerActivity, profile

from conftest import load_pkg
from oracle import moe_tail_oracle as G

pytestmark = pytest.mark.gpu
P = load_pkg()
FG = P.fused_gate_mul
DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _same(a, b):
    return a.shape == b.shape and torch.equal(_bits(a.contiguous()), _bits(b.contiguous()))


@pytest.mark.parametrize("dt", DTYPES)
def test_bit_identical_to_stock_on_reference_grid(cuda, dt):
    torch.manual_seed(0)
    for T, sc in G.GATE_CASES:
        out = torch.randn(T, G.H, dtype=dt, device=cuda) * 2.0
        g = torch.randn(T, 1, dtype=dt, device=cuda) * sc
        assert FG.supported(g, out), (T, sc)
        got = FG.sigmoid_gate_mul(g, out)
        assert _same(got, F.sigmoid(g) * out), (T, sc)
        assert _same(got, G.sigmoid_gate_mul(g, out)), (T, sc)


@pytest.mark.parametrize("cols", [1, 7, 8, 2562, 4100, 8192])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_ragged_widths(cuda, cols, dt):
    torch.manual_seed(cols)
    out = torch.randn(37, cols, dtype=dt, device=cuda)
    g = torch.randn(37, 1, dtype=dt, device=cuda) * 3
    assert _same(FG.sigmoid_gate_mul(g, out), F.sigmoid(g) * out)


@pytest.mark.parametrize("pad", [8, 3])
def test_strided_rows(cuda, pad):
    """out is a column slice of a wider buffer (row stride H + pad: aligned for pad 8)."""
    big = torch.randn(64, G.H + pad, dtype=torch.bfloat16, device=cuda)
    out = big[:, :G.H]
    g = torch.randn(64, 1, dtype=torch.bfloat16, device=cuda)
    assert FG.supported(g, out)
    assert _same(FG.sigmoid_gate_mul(g, out), F.sigmoid(g) * out)


def test_unaligned_base(cuda):
    flat = torch.randn(20 * G.H + 1, dtype=torch.bfloat16, device=cuda)
    out = flat[1:].view(20, G.H)                       # 2-byte offset: no 16-byte loads
    g = torch.randn(20, 1, dtype=torch.bfloat16, device=cuda)
    assert _same(FG.sigmoid_gate_mul(g, out), F.sigmoid(g) * out)


def test_non_finite_values(cuda):
    out = torch.randn(6, 16, dtype=torch.bfloat16, device=cuda)
    out[0, 0], out[1, 1], out[2, 2] = float("inf"), float("-inf"), float("nan")
    g = torch.tensor([[0.5], [float("inf")], [float("-inf")], [float("nan")], [0.0], [-0.0]],
                     dtype=torch.bfloat16, device=cuda)
    assert _same(FG.sigmoid_gate_mul(g, out), F.sigmoid(g) * out)


def test_no_rows_and_large_batch(cuda):
    out = torch.empty(0, G.H, dtype=torch.bfloat16, device=cuda)
    g = torch.empty(0, 1, dtype=torch.bfloat16, device=cuda)
    assert FG.sigmoid_gate_mul(g, out).shape == (0, G.H)
    out = torch.randn(8192, G.H, dtype=torch.bfloat16, device=cuda)    # prefill-sized
    g = torch.randn(8192, 1, dtype=torch.bfloat16, device=cuda)
    assert _same(FG.sigmoid_gate_mul(g, out), F.sigmoid(g) * out)


def _kernels(fn, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA]) as p:
        fn()
        torch.cuda.synchronize()
    return sum(1 for e in p.events()
               if e.device_type == torch.autograd.DeviceType.CUDA and e.device_index >= 0)


def test_one_launch_per_call(cuda):
    out = torch.randn(20, G.H, dtype=torch.bfloat16, device=cuda)
    g = torch.randn(20, 1, dtype=torch.bfloat16, device=cuda)
    x = torch.randn(20, G.H, dtype=torch.bfloat16, device=cuda)
    w = torch.randn(1, G.H, dtype=torch.bfloat16, device=cuda)
    assert _kernels(lambda: F.sigmoid(g) * out) == 2
    assert _kernels(lambda: FG.sigmoid_gate_mul(g, out)) == 1
    assert _kernels(lambda: FG.gemv_sigmoid_gate_mul(x, w, out)) == 1


def test_supported_refusals(cuda):
    """test_gate_mul.py:46-48 and fused_gate_mul.py:124-147."""
    out = torch.randn(20, G.H, dtype=torch.bfloat16, device=cuda)
    g = torch.randn(20, 1, dtype=torch.bfloat16, device=cuda)
    assert not FG.supported(torch.randn(4, 2, dtype=torch.bfloat16, device=cuda), out)
    assert not FG.supported(g.float(), out)
    x = torch.randn(20, G.H, dtype=torch.bfloat16, device=cuda)
    w = torch.randn(1, G.H, dtype=torch.bfloat16, device=cuda)
    assert FG.supported_gemv(x, w, out, 64)
    assert not FG.supported_gemv(x, w, out, 16)                       # over max_rows
    assert not FG.supported_gemv(x[:0], w, out[:0], 64)               # no rows
    assert not FG.supported_gemv(x, w.float(), out, 64)
    assert not FG.supported_gemv(x, torch.randn(2, G.H, dtype=torch.bfloat16, device=cuda), out, 64)


def _check_gemv(x, w, out, y, dt):
    ref_rows = 0
    if dt == torch.float32:
        # fp32 dot: the kernel sums at most ~8 products per thread, a 5-level warp tree and 16
        # warp totals, so |dg| <= 32 * 2^-24 * sum|x w| (+ half an ulp of g). Since
        # d ln sigmoid(g) / dg = 1 - sigmoid(g), y's relative error is (1 - s) |dg| plus a few
        # ulps of rounding in exp, the division and the multiply.
        want = G.gemv_sigmoid_gate_mul(x, w, out).double()
        gd = x.double() @ w.double().T
        dg = 32 * 2.0 ** -24 * (x.double().abs() @ w.double().abs().T) + 2.0 ** -24 * gd.abs()
        tol = want.abs() * (6e-7 + (1 - torch.sigmoid(gd)) * dg)
        assert ((y.double() - want).abs() <= tol).all()
        return
    cands = [G.gemv_sigmoid_gate_mul(x, w, out, c) for c in G.ulp_neighbours(G.gate_dot(x, w))]
    for t in range(x.shape[0]):
        hits = [_same(y[t], c[t]) for c in cands]
        assert any(hits), t
        ref_rows += hits[0]
    assert ref_rows >= int(0.9 * x.shape[0]), (ref_rows, x.shape[0])     # (a lone row may round either way)


@pytest.mark.parametrize("dt", DTYPES)
def test_gemv_fold_within_one_gate_ulp(cuda, dt):
    torch.manual_seed(3)
    for T in (1, 4, 20, 64):
        for sc in (0.02, 1.0, 30.0):
            x = torch.randn(T, G.H, dtype=dt, device=cuda)
            w = torch.randn(1, G.H, dtype=dt, device=cuda) * (sc / 50)
            out = torch.randn(T, G.H, dtype=dt, device=cuda) * 2.0
            assert FG.supported_gemv(x, w, out, 64)
            y = FG.gemv_sigmoid_gate_mul(x, w, out)
            _check_gemv(x, w, out, y, dt)
            if dt != torch.float32:                   # and the stock path agrees on most rows
                stock = F.sigmoid(F.linear(x, w)) * out
                same = sum(_same(y[t], stock[t]) for t in range(T))
                assert same >= int(0.9 * T), (T, sc, same)


@pytest.mark.parametrize("K,N,pad", [(2562, G.H, 0), (G.H, 7, 0), (G.H, G.H, 8), (G.H, G.H, 3),
                                     (8192, 4096, 0), (64, 16384, 0)])
def test_gemv_shapes(cuda, K, N, pad):
    torch.manual_seed(K + N + pad)
    T = 12
    xb = torch.randn(T, K + pad, dtype=torch.bfloat16, device=cuda)
    ob = torch.randn(T, N + pad, dtype=torch.bfloat16, device=cuda)
    x, out = xb[:, :K], ob[:, :N]
    w = torch.randn(1, K, dtype=torch.bfloat16, device=cuda) * 0.02
    y = FG.gemv_sigmoid_gate_mul(x, w, out)
    _check_gemv(x, w, out, y, torch.bfloat16)


# ---- moe_sum ----

MS = P.moe_ops


@pytest.mark.parametrize("topk", [1, 2, 3, 4, 5, 8, 10, 32])
@pytest.mark.parametrize("T,H", [(20, 2560), (1, 2560), (2048, 2560), (7, 1000), (5, 3)])
def test_moe_sum_bit_exact(cuda, topk, T, H):
    torch.manual_seed(topk * 31 + T + H)
    x = torch.randn(T, topk, H, device=cuda, dtype=torch.bfloat16)
    out = torch.empty(T, H, device=cuda, dtype=torch.bfloat16)
    MS.moe_sum(x, out)
    assert _same(out, G.moe_sum(x)), (topk, T, H)
    if not 2 <= topk <= 4:
        assert _same(out, x.sum(dim=1)), (topk, T, H)       # torch's own reduction


@pytest.mark.parametrize("dt", [torch.float16, torch.float32])
def test_moe_sum_dtypes_and_strided_out(cuda, dt):
    torch.manual_seed(9)
    x = torch.randn(20, 10, G.H, device=cuda, dtype=dt)
    big = torch.zeros(20, G.H + 8, device=cuda, dtype=dt)
    out = big[:, :G.H]
    MS.moe_sum(x, out)
    assert _same(out, G.moe_sum(x))
    assert big[:, G.H:].eq(0).all()                          # nothing written past the row


def test_moe_sum_follows_torch_reduction_order(cuda):
    """The case that separates torch's four-accumulator order from a k-order sum (rows
    [e, e, e, e, 1], e = 2^-24, f32): the kernel, the oracle and torch.sum all give 1."""
    e = 2.0 ** -24
    x = torch.tensor([e, e, e, e, 1.0], device=cuda).view(1, 5, 1).expand(3, 5, 8).contiguous()
    out = torch.empty(3, 8, device=cuda)
    MS.moe_sum(x, out)
    assert out.eq(1.0).all() and _same(out, x.sum(dim=1)) and _same(out, G.moe_sum(x))


def test_moe_sum_matches_vllm_op(cuda):
    """Against vLLM's own ops.moe_sum where it loads (both rounding forms reported)."""
    try:
        from vllm import _custom_ops as ops
        ops.moe_sum(torch.randn(2, 2, 64, device=cuda, dtype=torch.bfloat16),
                    torch.empty(2, 64, device=cuda, dtype=torch.bfloat16))
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM moe ops unavailable here: {type(e).__name__}")
    for topk in (2, 3, 4, 8, 10):
        x = torch.randn(20, topk, G.H, device=cuda, dtype=torch.bfloat16)
        ref = torch.empty(20, G.H, device=cuda, dtype=torch.bfloat16)
        ops.moe_sum(x, ref)
        out = torch.empty_like(ref)
        MS.moe_sum(x, out)
        n_each = int((G.moe_sum(x, True) != ref).sum())
        n_once = int((G.moe_sum(x, False) != ref).sum())
        print(f"topk={topk}: vs round-each {n_each}, vs fp32-once {n_once}, vs kernel {int((out != ref).sum())}")
        assert _same(out, ref), topk

"""CPU checks of the MoE block tail (shared-expert gate, moe_sum): the gate oracle pinned to
the reference test's own oracle, the moe_sum oracle's two rounding forms, the host-side
``supported`` logic, and the C-ABI argument codes (returned before any launch).

The reference's check (tests/k4/test_gate_mul.py:24-37) is bit-identity with the stock
``F.sigmoid(g) * out`` at H = 2560 over T in (1, 4, 20, 64, 2048) and gate scales
(0.02, 1, 30). The oracle meets it on CPU tensors for bf16 and f16. For f32 torch's
vectorised CPU sigmoid uses its own exp, so there the bound is 2 ulp (relative 2.5e-7); the
GPU tests hold f32 to bit-identity against torch's CUDA sigmoid."""
from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

from conftest import load_pkg
from oracle import moe_tail_oracle as G

P = load_pkg()
L = P._lib
FG = P.fused_gate_mul
NULL = ctypes.c_void_p(0)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_oracle_bit_identical_to_stock_on_reference_grid(dt):
    torch.manual_seed(0)
    for T, sc in G.GATE_CASES:
        out = (torch.randn(T, G.H) * 2.0).to(dt)
        g = (torch.randn(T, 1) * sc).to(dt)
        assert torch.equal(G.sigmoid_gate_mul(g, out), F.sigmoid(g) * out), (T, sc)


def test_oracle_f32_within_two_ulp_of_cpu_stock():
    torch.manual_seed(1)
    for T, sc in G.GATE_CASES:
        out = torch.randn(T, G.H) * 2.0
        g = torch.randn(T, 1) * sc
        ref, got = F.sigmoid(g) * out, G.sigmoid_gate_mul(g, out)
        assert ((ref - got).abs() <= 2.5e-7 * ref.abs()).all(), (T, sc)


def test_saturating_gates():
    """sigmoid of +-large and of +-0 rounds to exactly 1, 0 and 0.5 (the scale-30 cases)."""
    out = torch.full((4, 8), 3.0, dtype=torch.bfloat16)
    g = torch.tensor([[100.0], [-100.0], [0.0], [-0.0]], dtype=torch.bfloat16)
    y = G.sigmoid_gate_mul(g, out)
    assert y[0].eq(3.0).all() and y[1].eq(0.0).all() and y[2].eq(1.5).all() and y[3].eq(1.5).all()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_gemv_oracle_brackets_stock_linear(dt):
    """The stock path ``F.sigmoid(F.linear(x, w)) * out`` lands on the oracle's output for the
    correctly rounded gate or a neighbour one ulp away, row by row."""
    torch.manual_seed(2)
    for T in (1, 4, 20, 64):
        for sc in (0.02, 1.0, 30.0):
            x = torch.randn(T, G.H).to(dt)
            w = (torch.randn(1, G.H) * sc / 50).to(dt)
            out = (torch.randn(T, G.H) * 2.0).to(dt)
            ref = F.sigmoid(F.linear(x, w)) * out
            cands = [G.gemv_sigmoid_gate_mul(x, w, out, c) for c in G.ulp_neighbours(G.gate_dot(x, w))]
            for t in range(T):
                assert any(torch.equal(ref[t], c[t]) for c in cands), (T, sc, t)


def test_ulp_neighbours_step_one_value():
    g = torch.tensor([[1.0], [-2.5], [0.0]], dtype=torch.bfloat16)
    _, lo, hi = G.ulp_neighbours(g)
    assert lo.flatten().tolist()[:2] == [0.99609375, -2.484375]
    assert hi.flatten().tolist()[:2] == [1.0078125, -2.515625]
    assert lo[2].item() < 0 < hi[2].item()


def test_supported_refuses_what_the_reference_refuses():
    """supported() needs CUDA tensors; on CPU every shape is refused, and the predicate's shape
    rules are the reference's (fused_gate_mul.py:41-53, test_gate_mul.py:46-48)."""
    out = torch.randn(20, G.H, dtype=torch.bfloat16)
    g = torch.randn(20, 1, dtype=torch.bfloat16)
    assert not FG.supported(g, out)                      # host tensors
    assert not FG.supported_gemv(out, g.T.contiguous(), out, 64)


def test_gate_entry_codes():
    lib = L.lmhead()
    assert lib.b200_sigmoid_gate_mul(NULL, NULL, NULL, -1, 8, 8, 0, NULL) == -1
    assert lib.b200_sigmoid_gate_mul(NULL, NULL, NULL, 4, 8, 4, 0, NULL) == -1      # stride < cols
    assert lib.b200_sigmoid_gate_mul(NULL, NULL, NULL, 4, 8, 8, 3, NULL) == -2
    assert lib.b200_sigmoid_gate_mul(NULL, NULL, NULL, 0, 8, 8, 0, NULL) == 0       # no rows: no-op
    assert lib.b200_gemv_sigmoid_gate_mul(NULL, NULL, NULL, NULL, 0, 8, 8, 8, 8, 0, NULL) == -1
    assert lib.b200_gemv_sigmoid_gate_mul(NULL, NULL, NULL, NULL, 65536, 8, 8, 8, 8, 0, NULL) == -1
    assert lib.b200_gemv_sigmoid_gate_mul(NULL, NULL, NULL, NULL, 2, 8, 8, 4, 8, 0, NULL) == -1
    assert lib.b200_gemv_sigmoid_gate_mul(NULL, NULL, NULL, NULL, 2, 8, 8, 8, 8, 7, NULL) == -2


def test_gate_ops_fail_loudly_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    out = torch.randn(2, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        FG.sigmoid_gate_mul(torch.zeros(2, 1, dtype=torch.bfloat16), out)
    with pytest.raises(ValueError):
        FG.gemv_sigmoid_gate_mul(out, torch.zeros(1, 16, dtype=torch.bfloat16), out)


# ---- moe_sum ----

def test_moe_sum_oracle_wide_topk_order():
    """top_k outside {2, 3, 4}: four interleaved fp32 accumulators, ((a0 + a1) + a2) + a3.
    Rows [e, e, e, e, 1] (f32, e = 2^-24) tell the orders apart: in k order the four e sum to
    4e exactly and 1 + 4e = 1 + 2^-22 is representable; in torch's order a0 = e + 1 rounds to
    1 and every later e is lost against 1."""
    e = 2.0 ** -24
    x = torch.tensor([[[e], [e], [e], [e], [1.0]]], dtype=torch.float32)
    assert G.moe_sum(x).item() == 1.0
    seq = torch.tensor(0.0)
    for k in range(5):
        seq = seq + x[0, k, 0]
    assert seq.item() == 1.0 + 2.0 ** -22
    torch.manual_seed(4)
    for topk in (1, 5, 8, 10):
        xb = torch.randn(20, topk, G.H, dtype=torch.bfloat16)
        assert torch.equal(G.moe_sum(xb), xb.sum(dim=1)), topk      # torch's CPU sum agrees here


def test_moe_sum_oracle_rounds_each_add_for_small_topk():
    """top_k in {2, 3, 4}: every partial sum is stored in the dtype (1 + 2^-8 + 2^-8 in bf16
    is 1 when rounded after each add, 1 + 2^-7 when summed in fp32)."""
    x = torch.tensor([[[1.0], [2.0 ** -8], [2.0 ** -8]]], dtype=torch.bfloat16)
    assert G.moe_sum(x).item() == 1.0
    assert G.moe_sum(x, round_each=False).item() == 1.0 + 2.0 ** -7


def test_moe_sum_entry_codes():
    lib = L.lmhead()
    assert lib.b200_moe_sum(NULL, NULL, -1, 10, 8, 8, 0, NULL) == -1
    assert lib.b200_moe_sum(NULL, NULL, 4, 0, 8, 8, 0, NULL) == -1
    assert lib.b200_moe_sum(NULL, NULL, 4, 33, 8, 8, 0, NULL) == -1
    assert lib.b200_moe_sum(NULL, NULL, 4, 10, 8, 4, 0, NULL) == -1
    assert lib.b200_moe_sum(NULL, NULL, 4, 10, 8, 8, 3, NULL) == -2
    assert lib.b200_moe_sum(NULL, NULL, 0, 10, 8, 8, 0, NULL) == 0
    if not torch.cuda.is_available():
        x = torch.zeros(2, 10, 16, dtype=torch.bfloat16)
        with pytest.raises(ValueError):
            P.moe_ops.moe_sum(x, torch.zeros(2, 16, dtype=torch.bfloat16))

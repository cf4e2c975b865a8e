"""GPU parity of the fused SiLU*mul -> FP8 quant and the per-token group quant.

Bit-exact (activation, scales, FP8 bytes) against the torch-GPU eager restatement in
oracle/quant_oracle.py over the reference probe's grid (tests/k4/probe_silu_quant.py:22-53:
rows {1,10,50,80,2048} x d {320,640} x input scale {1, 1e-3, 60}) plus the decode
[8, 2x512] bf16 case, f16 inputs, strided and unaligned rows, the zero row; and against
vLLM's silu_and_mul + scaled_fp8_quant pair when those ops load here. The CPU oracle is
compared too and the number of CPU/GPU expf disagreements is reported."""
from __future__ import annotations

import pytest
import torch

from conftest import load_pkg
from oracle import quant_oracle as Q

pytestmark = pytest.mark.gpu
P = load_pkg()
FQ = P.fused_silu_mul_quant
FP8 = torch.float8_e4m3fn


def _eq(a, b):
    return torch.equal(a.view(torch.uint8) if a.dtype == FP8 else a,
                       b.view(torch.uint8) if b.dtype == FP8 else b)


GRID = [(r, d, s) for r in (1, 10, 50, 80, 2048) for d in (320, 640) for s in (1.0, 1e-3, 60.0)]
# row widths at the one-pass kernel's register bounds (256 / 512 / 1024) and past them (two-pass)
GRID += [(33, d, 1.0) for d in (8, 256, 264, 512, 1024, 1032, 4096, 8192)]


@pytest.mark.parametrize("rows,d,sc", GRID)
def test_silu_quant_bit_exact_grid(cuda, rows, d, sc):
    torch.manual_seed(rows * 7 + d)
    x = torch.randn(rows, 2 * d, device=cuda, dtype=torch.bfloat16) * sc
    assert FQ.supported(x)
    act, q, s = FQ.silu_mul_quant(x, FP8, write_act=True)
    ra, rq, rs = Q.silu_mul_quant(x, write_act=True)          # torch on the GPU
    assert _eq(act, ra) and _eq(s, rs) and _eq(q, rq)
    _, q2, s2 = FQ.silu_mul_quant(x, FP8)                      # write_act=False path
    assert _eq(q2, q) and _eq(s2, s)


def test_silu_quant_baseline_config_and_cpu_oracle(cuda):
    """Decode config: bf16 [8, 2x512] ~N(0,1) from seed 0. GPU exact; CPU oracle compared
    and its (expf-ulp) disagreements reported."""
    torch.manual_seed(0)
    x = torch.randn(8, 1024, dtype=torch.bfloat16)
    act, q, s = FQ.silu_mul_quant(x.to(cuda), FP8, write_act=True)
    ra, rq, rs = Q.silu_mul_quant(x.to(cuda), write_act=True)
    assert _eq(act, ra) and _eq(q, rq) and _eq(s, rs)
    ca, cq, cs = Q.silu_mul_quant(x, write_act=True)
    n_act = int((act.cpu() != ca).sum())
    n_q = int((q.cpu().view(torch.uint8) != cq.view(torch.uint8)).sum())
    print(f"CPU-oracle disagreements: act {n_act}/{ca.numel()}, q {n_q}/{cq.numel()}")
    assert n_act <= ca.numel() // 100


def test_silu_quant_f16_strided_unaligned(cuda):
    torch.manual_seed(1)
    base = torch.randn(33, 2 * 77 + 6, device=cuda, dtype=torch.float16)
    x = base[:, : 2 * 77]                                      # row stride 160, d = 77 (scalar path)
    act, q, s = FQ.silu_mul_quant(x, FP8, write_act=True)
    ra, rq, rs = Q.silu_mul_quant(x, write_act=True)
    assert _eq(act, ra) and _eq(q, rq) and _eq(s, rs)
    xb = torch.randn(20, 2 * 512 + 64, device=cuda, dtype=torch.bfloat16)[:, :1024]  # strided, aligned
    _, q, s = FQ.silu_mul_quant(xb, FP8)
    _, rq, rs = Q.silu_mul_quant(xb)
    assert _eq(q, rq) and _eq(s, rs)


def test_silu_quant_zero_row_and_empty(cuda):
    z = torch.zeros(4, 640, device=cuda, dtype=torch.bfloat16)
    _, q, s = FQ.silu_mul_quant(z, FP8)
    assert torch.all(s == torch.tensor(1.0 / (448.0 * 512.0), device=cuda))
    assert torch.all(q.view(torch.uint8) == 0)
    _, q0, s0 = FQ.silu_mul_quant(torch.zeros(0, 640, device=cuda, dtype=torch.bfloat16), FP8)
    assert q0.shape == (0, 320) and s0.shape == (0, 1)
    assert not FQ.supported(torch.empty(2, 2 * 16384, device=cuda, dtype=torch.bfloat16))


def _vllm_pair_ops(cuda):
    try:
        from vllm import _custom_ops as ops
        t = torch.randn(2, 64, device=cuda, dtype=torch.bfloat16)
        o = torch.empty(2, 32, device=cuda, dtype=torch.bfloat16)
        torch.ops._C.silu_and_mul(o, t)
        ops.scaled_fp8_quant(o, use_per_token_if_dynamic=True)
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM _C ops unavailable here: {type(e).__name__}")
    return ops


def test_silu_quant_matches_vllm_pair(cuda):
    """The reference probe's own oracle, asserted as the probe asserts it
    (tests/k4/probe_silu_quant.py:20-53): vLLM's silu_and_mul followed by
    scaled_fp8_quant(use_per_token_if_dynamic=True) must give the same activation, the same
    fp32 scale and the same FP8 bytes, bit for bit, over rows {1,10,50,80,2048} x d {320,640}
    x input scale {1, 1e-3, 60} (seed 0, drawn in the probe's order) and the all-zero row,
    whose scale is the floor 1/(448*512)."""
    ops = _vllm_pair_ops(cuda)
    torch.manual_seed(0)
    bad = []
    for rows in (1, 10, 50, 80, 2048):
        for d in (320, 640):
            for sc in (1.0, 1e-3, 60.0):
                x = torch.randn(rows, 2 * d, device=cuda, dtype=torch.bfloat16) * sc
                ic2 = torch.empty(rows, d, device=cuda, dtype=torch.bfloat16)
                torch.ops._C.silu_and_mul(ic2, x)
                qr, sr = ops.scaled_fp8_quant(ic2, use_per_token_if_dynamic=True)
                act, q, s = FQ.silu_mul_quant(x, FP8, write_act=True)
                na = int((act != ic2).sum())
                ns = int((s.view(-1) != sr.view(-1)).sum())
                nq = int((q.view(torch.uint8) != qr.view(torch.uint8)).sum())
                if na or ns or nq:
                    bad.append(f"rows={rows} d={d} x{sc}: act {na} scale {ns} q {nq}")
    z = torch.zeros(4, 640, device=cuda, dtype=torch.bfloat16)
    ic2 = torch.empty(4, 320, device=cuda, dtype=torch.bfloat16)
    torch.ops._C.silu_and_mul(ic2, z)
    qr, sr = ops.scaled_fp8_quant(ic2, use_per_token_if_dynamic=True)
    _, q, s = FQ.silu_mul_quant(z, FP8)
    if not (_eq(s.view(-1), sr.view(-1)) and _eq(q, qr)):
        bad.append("zero row")
    assert bool(s[0, 0] == torch.tensor(1.0 / (448.0 * 512.0), device=cuda))
    assert not bad, "; ".join(bad)


@pytest.mark.parametrize("rows,d", [(8, 512), (50, 384), (1, 128), (3, 1024)])
def test_silu_quant_group128(cuda, rows, d):
    torch.manual_seed(rows + d)
    x = torch.randn(rows, 2 * d, device=cuda, dtype=torch.bfloat16)
    act, q, s = FQ.silu_mul_quant_group(x, write_act=True)
    ra, rq, rs = Q.silu_mul_quant_group(x, write_act=True)
    assert _eq(act, ra) and _eq(q, rq) and _eq(s, rs)
    assert s.shape == (rows, d // 128)


@pytest.mark.parametrize("M,K", [(1, 2560), (5, 2560), (20, 2560), (64, 2560), (3, 128)])
def test_group_quant_bit_exact(cuda, M, K):
    torch.manual_seed(M * 11 + K)
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16)
    x[0, :128] = 0.0                                           # eps floor group
    q, s = FQ.per_token_group_quant_fp8(x, 128)
    rq, rs = Q.group_quant_fp8(x, 128)
    assert _eq(q, rq) and _eq(s, rs)
    cq, cs = Q.group_quant_fp8(x.cpu(), 128)
    assert _eq(q.cpu(), cq) and _eq(s.cpu(), cs)


def test_group_quant_matches_vllm_triton(cuda):
    """vLLM's Triton _per_token_group_quant_fp8 (the ROCm path the reference runs), as a checker."""
    try:
        from vllm.model_executor.layers.quantization.utils import fp8_utils as fu
        kern = fu._per_token_group_quant_fp8
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM Triton group quant unavailable: {type(e).__name__}")
    M, K = 20, 2560
    x = torch.randn(M, K, device=cuda, dtype=torch.bfloat16) * 3
    xq = torch.empty(M, K, device=cuda, dtype=FP8)
    xs = torch.empty(M, K // 128, device=cuda, dtype=torch.float32)
    try:
        kern[(M * K // 128,)](x, xq, xs, 128, K, x.stride(0), 1e-10, fp8_min=-448.0, fp8_max=448.0,
                               use_ue8m0=False, BLOCK=128, num_warps=1, num_stages=1)
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"Triton launch failed here: {type(e).__name__}: {e}")
    q, s = FQ.per_token_group_quant_fp8(x, 128)
    # Triton's fp32 `/` need not be IEEE-rounded on every target, so this third-party
    # cross-check bounds the disagreement instead of requiring identity; the bit-exact
    # contract is test_group_quant_bit_exact.
    ns = int((s != xs).sum())
    nq = int((q.view(torch.uint8) != xq.view(torch.uint8)).sum())
    print(f"vs vLLM Triton group quant: scales {ns}/{s.numel()} differ, bytes {nq}/{q.numel()} differ")
    assert ns == 0 and nq <= q.numel() // 100


# ---- per-token hidden-state quant (scaled_fp8_quant, use_per_token_if_dynamic=True) ----

HQ = P.fp8_hidden_quant
TOKEN_GRID = [(r, k, s) for r in (1, 5, 20, 64, 2048) for k in (2560,) for s in (1.0, 1e-3, 60.0)]
# widths at the register kernel's bounds (1024 / 2048 / 3072 / 4096), past them (two-pass),
# unaligned (K % 8 != 0) and tiny
TOKEN_GRID += [(33, k, 1.0) for k in (7, 8, 128, 1024, 1032, 2048, 3072, 4096, 4104, 8192)]


@pytest.mark.parametrize("rows,K,sc", TOKEN_GRID)
def test_per_token_quant_bit_exact(cuda, rows, K, sc):
    torch.manual_seed(rows * 13 + K)
    x = torch.randn(rows, K, device=cuda, dtype=torch.bfloat16) * sc
    if rows > 1:
        x[1] = 0.0                                             # the min-scale floor
    q, s = HQ.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
    rq, rs = Q.per_token_quant_fp8(x)
    assert s.shape == (rows, 1) and _eq(s, rs) and _eq(q, rq)


def test_per_token_quant_f16_strided_scale_ub(cuda):
    torch.manual_seed(5)
    big = torch.randn(20, 2560 + 8, device=cuda, dtype=torch.float16) * 4
    x = big[:, :2560]                                          # row stride 2568
    q, s = HQ.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
    rq, rs = Q.per_token_quant_fp8(x)
    assert _eq(q, rq) and _eq(s, rs)
    ub = torch.tensor([2.0], device=cuda)
    q, s = HQ.scaled_fp8_quant(x, use_per_token_if_dynamic=True, scale_ub=ub)
    rq, rs = Q.per_token_quant_fp8(x, ub)
    assert _eq(q, rq) and _eq(s, rs)
    unal = torch.randn(20 * 2560 + 1, device=cuda, dtype=torch.bfloat16)[1:].view(20, 2560)
    q, s = HQ.scaled_fp8_quant(unal, use_per_token_if_dynamic=True)
    rq, rs = Q.per_token_quant_fp8(unal)
    assert _eq(q, rq) and _eq(s, rs)


def test_per_token_quant_matches_vllm_op(cuda):
    """Against vLLM's own scaled_fp8_quant(use_per_token_if_dynamic=True) where it loads."""
    try:
        from vllm import _custom_ops as ops
        ops.scaled_fp8_quant(torch.randn(2, 64, device=cuda, dtype=torch.bfloat16),
                             use_per_token_if_dynamic=True)
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"vLLM _C ops unavailable here: {type(e).__name__}")
    for rows in (1, 20, 64, 2048):
        x = torch.randn(rows, 2560, device=cuda, dtype=torch.bfloat16)
        qr, sr = ops.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
        q, s = HQ.scaled_fp8_quant(x, use_per_token_if_dynamic=True)
        nd = int((q.view(torch.uint8) != qr.view(torch.uint8)).sum())
        print(f"rows={rows}: scale equal {torch.equal(s, sr)}, q diffs {nd}")
        assert torch.equal(s, sr) and nd == 0, rows


def test_fp8_quant_shared_reuses_on_gpu(cuda):
    x = torch.randn(20, 2560, device=cuda, dtype=torch.bfloat16)
    HQ.set_share(True)
    try:
        a = HQ.fp8_quant_shared(x)
        b = HQ.fp8_quant_shared(x)
        assert a[0] is b[0]
        c = HQ.fp8_quant_shared(x)
        assert c[0] is not a[0] and _eq(c[0], a[0]) and _eq(c[1], a[1])
    finally:
        HQ.set_share(False)


def test_non_finite_rows_match_oracle(cuda):
    """NaN / inf values through all three quant kernels: the reference's clamp order sends NaN
    to +448, infinities saturate, and the row / group amax ignores NaNs."""
    torch.manual_seed(11)
    x = torch.randn(6, 2 * 512, device=cuda, dtype=torch.bfloat16)
    x[0, 5] = float("nan")
    x[1, 7] = float("inf")
    x[2, 600] = float("-inf")
    x[3, 9] = float("nan")
    x[3, 700] = float("nan")
    act, q, s = FQ.silu_mul_quant(x, FP8, write_act=True)
    ra, rq, rs = Q.silu_mul_quant(x, write_act=True)
    # NaN payloads of the activation may differ between conversions: compare NaN positions
    assert torch.equal(act.isnan(), ra.isnan()) and torch.equal(act.nan_to_num(), ra.nan_to_num())
    assert _eq(q, rq)
    assert torch.equal(s.isnan(), rs.isnan()) and torch.equal(s.nan_to_num(), rs.nan_to_num())
    h = torch.randn(6, 2560, device=cuda, dtype=torch.bfloat16)
    h[0, 3], h[1, 1000], h[2, 2559], h[4, 0] = float("nan"), float("inf"), float("-inf"), float("nan")
    for ub in (None, torch.tensor([2.0], device=cuda)):
        hq, hs = HQ.scaled_fp8_quant(h, use_per_token_if_dynamic=True, scale_ub=ub)
        rq, rs = Q.per_token_quant_fp8(h, ub)
        assert _eq(hq, rq) and torch.equal(hs, rs)
    gq, gs = FQ.per_token_group_quant_fp8(h, 128)
    rq, rs = Q.group_quant_fp8(h, 128)
    assert _eq(gq, rq) and torch.equal(gs, rs)

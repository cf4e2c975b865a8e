"""CPU checks of the MoE hidden-state quant: the fp8_quant_shared handoff rules
(patches/model_executor/kernels/linear/mxfp4/r4dhip.py.diff L7-34), the oracle's known
answers for vLLM's per-token scaled_fp8_quant, and the C-ABI argument codes."""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import load_pkg
from oracle import quant_oracle as Q

P = load_pkg()
HQ = P.fp8_hidden_quant
L = P._lib
NULL = ctypes.c_void_p(0)


class _Counter:
    def __init__(self):
        self.calls = 0

    def __call__(self, t):
        self.calls += 1
        return Q.per_token_quant_fp8(t)


@pytest.fixture
def share():
    HQ.set_share(True)
    yield
    HQ.set_share(False)


def test_share_off_quantizes_every_call():
    HQ.set_share(False)
    f, x = _Counter(), torch.randn(4, 64, dtype=torch.bfloat16)
    HQ.fp8_quant_shared(x, f)
    HQ.fp8_quant_shared(x, f)
    assert f.calls == 2


def test_share_hit_is_served_once(share):
    """Shared expert then routed experts on the same tensor: one quant; a third call on the
    same tensor quantizes again (the hit cleared the slot)."""
    f, x = _Counter(), torch.randn(4, 64, dtype=torch.bfloat16)
    a = HQ.fp8_quant_shared(x, f)
    b = HQ.fp8_quant_shared(x, f)
    assert f.calls == 1 and a[0] is b[0] and a[1] is b[1]
    HQ.fp8_quant_shared(x, f)
    assert f.calls == 2


def test_share_keys_on_identity_not_address(share):
    """An equal tensor, or a view of the same storage, is another object: no hit."""
    f, x = _Counter(), torch.randn(4, 64, dtype=torch.bfloat16)
    HQ.fp8_quant_shared(x, f)
    HQ.fp8_quant_shared(x.clone(), f)
    HQ.fp8_quant_shared(x.view(4, 64), f)
    assert f.calls == 3


def test_share_slot_keeps_key_alive(share):
    """The slot holds a strong reference, so the key's storage cannot be freed and reused."""
    f = _Counter()
    x = torch.randn(4, 64, dtype=torch.bfloat16)
    HQ.fp8_quant_shared(x, f)
    assert HQ._a8_slot is not None and HQ._a8_slot[0] is x


def test_per_token_oracle_known_answers():
    x = torch.zeros(4, 16, dtype=torch.bfloat16)
    x[1, 3] = 448.0                        # amax 448 -> scale exactly 1, q = x
    x[2, :] = -3.5                         # constant row -> every code is -448
    x[3, 0] = 1e-30                        # below the floor -> scale 1/(448*512)
    q, s = Q.per_token_quant_fp8(x)
    assert s[0, 0].item() == pytest.approx(Q.MIN_SCALE, rel=0) and s[1, 0].item() == 1.0
    assert q[1, 3].float().item() == 448.0 and q[0].float().abs().max().item() == 0.0
    assert (q[2].float() == -448.0).all()
    assert s[3, 0].item() == pytest.approx(Q.MIN_SCALE, rel=0)
    # scale_ub caps the amax: values past it clamp to +-448
    q2, s2 = Q.per_token_quant_fp8(x, torch.tensor([1.0]))
    assert s2[1, 0].item() == pytest.approx(1.0 / 448.0) and q2[1, 3].float().item() == 448.0


def test_per_token_oracle_is_silu_quant_tail():
    """Without the SiLU it is the same scale and division as fused_silu_mul_quant."""
    torch.manual_seed(0)
    x = torch.randn(8, 1024, dtype=torch.bfloat16)
    a = Q.silu_mul(x)
    _, q1, s1 = Q.silu_mul_quant(x)
    q2, s2 = Q.per_token_quant_fp8(a)
    assert torch.equal(s1, s2) and torch.equal(q1.view(torch.uint8), q2.view(torch.uint8))


def test_per_token_entry_codes_and_forms():
    lib = L.lmhead()
    assert lib.b200_per_token_quant_fp8(NULL, -1, 16, 16, 0, NULL, NULL, NULL, NULL) == -1
    assert lib.b200_per_token_quant_fp8(NULL, 2, 16, 8, 0, NULL, NULL, NULL, NULL) == -1
    assert lib.b200_per_token_quant_fp8(NULL, 2, 16, 16, 2, NULL, NULL, NULL, NULL) == -2
    assert lib.b200_per_token_quant_fp8(NULL, 0, 16, 16, 0, NULL, NULL, NULL, NULL) == 0
    x = torch.zeros(2, 16, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        HQ.scaled_fp8_quant(x)                            # per-tensor form is not built
    with pytest.raises(NotImplementedError):
        HQ.scaled_fp8_quant(x, scale=torch.ones(1), use_per_token_if_dynamic=True)
    if not torch.cuda.is_available():
        with pytest.raises(ValueError):
            HQ.scaled_fp8_quant(x, use_per_token_if_dynamic=True)   # no CPU fallback


def test_non_finite_inputs_follow_the_reference_clamp():
    """maximum(-448, minimum(v, 448)) (fused_silu_mul_quant.py:56; vLLM's fmaxf(-max,
    fminf(v, max))): NaN -> +448 (0x7E), +-inf -> +-448; the row amax ignores NaNs."""
    x = torch.tensor([[1.0, float("nan"), -2.0, 0.5]], dtype=torch.bfloat16)
    q, s = Q.per_token_quant_fp8(x)
    assert s.item() == pytest.approx(2.0 / 448.0)
    assert q.view(torch.uint8).tolist()[0][1] == 0x7E
    assert q.view(torch.uint8).tolist()[0][2] == 0xFE                 # -2 / (2/448) = -448
    q, s = Q.per_token_quant_fp8(x, torch.tensor([1.0]))               # capped: -2 clamps
    assert q.view(torch.uint8).tolist()[0][2] == 0xFE
    y = torch.tensor([[float("-inf"), 1.0]], dtype=torch.bfloat16)
    q, s = Q.per_token_quant_fp8(y)                                    # inf amax -> inf scale
    assert s.item() == float("inf") and q.view(torch.uint8).tolist()[0] == [0x7E, 0x00]

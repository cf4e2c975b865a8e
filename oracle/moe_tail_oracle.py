"""CPU restatement of the MoE block's tail (the shared-expert gate and the routed experts'
sum) -- TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use this
module, as the checker; the product path is csrc/gate.cu and csrc/moe_sum.cu behind
fused_gate_mul.py and moe_ops.py.

Sources followed (davetha/r9700-lru-expert-cache):
* ``sigmoid_gate_mul``      -- kernels/fused_gate_mul.py:19-38 (rounding spelled out :7-10):
  s = dtype(1 / (1 + exp(-fp32(g)))), y = dtype(fp32(s) * fp32(out)).
* ``gemv_sigmoid_gate_mul`` -- kernels/fused_gate_mul.py:91-121: g = dtype(x . w) first.
* ``moe_sum`` -- vLLM ``ops.moe_sum(input, output)`` as the MoE block calls it
  (patches/model_executor/layers/fused_moe/experts/r4d_mxfp4_moe.py.lru.diff L638, L696).
* The reference's own check (tests/k4/test_gate_mul.py:25-37) is bit-identity with the stock
  ``F.sigmoid(g) * out`` over T in (1, 4, 20, 64, 2048) and gate scales (0.02, 1, 30) at
  H = 2560; ``GATE_CASES`` restates that grid.

Device-agnostic torch code: on CPU tensors this is the CPU oracle; on CUDA tensors its
``exp`` and division are the device functions the kernels call.
"""
from __future__ import annotations

import torch

H = 2560                                             # tests/k4/test_gate_mul.py:8
GATE_CASES = [(t, s) for t in (1, 4, 20, 64, 2048) for s in (0.02, 1.0, 30.0)]   # :24-25


def gate_scale(g: torch.Tensor) -> torch.Tensor:
    """aten's sigmoid of a stored gate: fp32 ``1 / (1 + exp(-g))`` (a true division), rounded
    to the gate's dtype (fused_gate_mul.py:27-30)."""
    gf = g.float()
    d = 1.0 + torch.exp(-gf)
    return (torch.ones_like(d) / d).to(g.dtype)


def sigmoid_gate_mul(gate: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """[T, 1] gate times [T, H] out, rounded as ``F.sigmoid(gate) * out``."""
    return (gate_scale(gate).float() * out.float()).to(out.dtype)


def gate_dot(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """The [T, 1] gate GEMV ``x @ w.T`` accumulated in float64 and rounded once to x's dtype:
    the correctly rounded value any fp32-accumulating GEMM approximates."""
    return (x.double() @ w.double().T).to(x.dtype)


def gemv_sigmoid_gate_mul(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor,
                          gate: torch.Tensor | None = None) -> torch.Tensor:
    """``sigmoid(dtype(x @ w.T)) * out`` (fused_gate_mul.py:112-121); ``gate`` overrides the
    rounded dot (the tests try its neighbours one ulp away)."""
    g = gate_dot(x, w) if gate is None else gate
    return sigmoid_gate_mul(g, out)


def ulp_neighbours(g: torch.Tensor) -> list[torch.Tensor]:
    """g and the values one step of its own dtype away on either side (for bf16 / f16 a +-1
    on the bit pattern; a step across zero gives the smallest subnormal of either sign)."""
    if g.dtype in (torch.bfloat16, torch.float16):
        bits = g.view(torch.int16).to(torch.int32)
        mag = bits & 0x7FFF
        sgn = bits & 0x8000
        up = torch.where(mag == 0x7FFF, bits, sgn | (mag + 1))
        down = torch.where(mag == 0, (sgn ^ 0x8000) | 1, sgn | (mag - 1))
        as_t = lambda b: torch.where(b >= 0x8000, b - 0x10000, b).to(torch.int16).view(g.dtype)
        return [g, as_t(down), as_t(up)]
    inf = torch.tensor(float("inf"), dtype=g.dtype, device=g.device)
    return [g, torch.nextafter(g, -inf), torch.nextafter(g, inf)]


def moe_sum(x: torch.Tensor, round_each: bool | None = None) -> torch.Tensor:
    """[T, top_k, H] -> [T, H]. ``round_each`` (default: top_k in {2, 3, 4}, vLLM's
    storage-dtype kernel) adds the rows in k order and rounds the running sum to x's dtype after
    every add. Otherwise torch.sum's CUDA order for this layout (ATen native/cuda/Reduce.cuh,
    thread_reduce_impl, vt0 = 4): fp32 accumulators a_i over k = i, i + 4, ..., combined as
    ((a0 + a1) + a2) + a3 and rounded once."""
    topk = x.shape[1]
    if round_each is None:
        round_each = 2 <= topk <= 4
    if round_each:
        acc = torch.zeros(x.shape[0], x.shape[2], dtype=torch.float32, device=x.device)
        for k in range(topk):
            acc = (acc + x[:, k].float()).to(x.dtype).float()
        return acc.to(x.dtype)
    accs = [torch.zeros(x.shape[0], x.shape[2], dtype=torch.float32, device=x.device) for _ in range(4)]
    for k in range(topk):
        accs[k % 4] = accs[k % 4] + x[:, k].float()
    return (((accs[0] + accs[1]) + accs[2]) + accs[3]).to(x.dtype)

"""B200-native (sm_100a) rebuild of the quantized decode hot path of
davetha/r9700-lru-expert-cache, behind the reference's own Python entry points and
librlu's C ABI:

* ``fused_silu_mul_quant`` -- fused SiLU*mul -> FP8-e4m3 activation quant
* ``draft_w4_lmhead``      -- W4 group-128 draft lm_head GEMV (+ fused argmax / logsumexp)
* ``fp8_target_lmhead``    -- FP8 128x128 block-scaled target lm_head (+ fused argmax / lse)
* ``lru``                  -- device-side LRU expert-slot cache (manage / fused / gather)
* ``fused_gate_mul``       -- the MoE shared expert's sigmoid(gate) * out (+ the gate GEMV fold)
* ``fp8_hidden_quant``     -- per-token FP8 quant of MoE hidden states (fp8_quant_shared)
* ``moe_ops``              -- moe_sum, the routed experts' outputs summed over top_k
* ``packs``                -- persisted W4 / FP8 head packs (save, load, cached)
* ``sharded``              -- vocab-sharded lm_head combine and expert-id-sharded LRU

The kernels live in two in-tree shared libraries (librlu.so, libb200lmhead.so) built from
``csrc/`` by ``build.py``; there is no CPU fallback.
"""
from . import _lib  # noqa: F401
from . import (draft_w4_lmhead, fp8_hidden_quant, fp8_target_lmhead, fused_gate_mul,  # noqa: F401
               fused_silu_mul_quant, lru, moe_ops, packs, sharded)

__all__ = ["draft_w4_lmhead", "fp8_hidden_quant", "fp8_target_lmhead", "fused_gate_mul",
           "fused_silu_mul_quant", "lru", "moe_ops", "packs", "sharded"]

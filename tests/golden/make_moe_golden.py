"""Generate tests/golden/moe_gemm_reference.npz from the REFERENCE's own MoE harness.

Runs only where davetha/r9700-lru-expert-cache is checked out (pass its path as argv[1]); the
fixture it writes is committed so the tests never need the reference at run time.

What runs from the reference, unmodified: ``tests/k1/moe_ref_harness.py`` -- its pure-torch
``dequant_expert`` (checkpoint MXFP4 -> fp32), ``quant_fp8_per_token`` (the per-token FP8
quant it feeds the kernel) and ``moe_align_block_size_torch`` (the block packing), imported as
a module (its top level only defines constants and functions; nothing touches a GPU). The
harness builds its cases on the GPU inside ``build_case``; here the same construction (E8M0
exponents ref - drop, ref in [120, 136), drop in [0, 8]; random codes; x ~ 0.4 N(0, 1); routed
weights U(0, 1)) is drawn on the CPU from a seeded generator, and the fp32 reference output is
the harness's own formula (moe_ref_harness.py:196-203): for every routed expert, the rows it
takes times the dequantised expert.
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (E, N, K, M tokens, top_k, seed): small cases with the model's K / N ratios, an expert
# spanning several blocks (E=4, 40 routed rows), and top_k = 1 (the down projection's form)
CASES = [(8, 32, 128, 3, 2, 1), (16, 64, 320, 5, 4, 2), (4, 48, 256, 20, 2, 3),
         (32, 16, 64, 6, 1, 4), (8, 80, 160, 1, 8, 5)]


def load_harness(ref: str):
    path = os.path.join(ref, "tests", "k1", "moe_ref_harness.py")
    spec = importlib.util.spec_from_file_location("moe_ref_harness", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def make_case(H, E, N, K, M, top_k, seed):
    g = torch.Generator().manual_seed(seed)
    nb = K // H.GROUP
    ref = torch.randint(120, 136, (E, N, 1), generator=g, dtype=torch.int32)
    drop = torch.randint(0, 9, (E, N, nb), generator=g, dtype=torch.int32)
    s = (ref - drop).clamp(0, 254).to(torch.uint8)
    w = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.uint8)
    topk = torch.randint(0, E, (M, top_k), generator=g, dtype=torch.int32)
    x = torch.randn(M, K, generator=g, dtype=torch.float32) * 0.4
    tw = torch.rand(M * top_k, generator=g, dtype=torch.float32)
    qx, xs = H.quant_fp8_per_token(x)
    sorted_ids, expert_ids, npad = H.moe_align_block_size_torch(topk, H.BLOCK, E)
    flat = topk.reshape(-1)
    a = qx.float() * xs.unsqueeze(1)
    out = torch.zeros(M * top_k, N, dtype=torch.float32)
    for e in range(E):
        wd = H.dequant_expert(w[e], s[e])
        rows = (flat == e).nonzero(as_tuple=True)[0]
        if rows.numel():
            out[rows] = a[(rows // top_k).long()] @ wd.T
    return {"w": w, "s": s, "topk": topk, "x": x, "tw": tw, "qx": qx.view(torch.uint8), "xs": xs,
            "sorted_ids": sorted_ids, "expert_ids": expert_ids, "npad": npad, "out": out,
            "deq0": H.dequant_expert(w[0], s[0])}


def main(ref: str) -> None:
    H = load_harness(ref)
    arrays = {}
    for i, (E, N, K, M, top_k, seed) in enumerate(CASES):
        c = make_case(H, E, N, K, M, top_k, seed)
        arrays[f"c{i}_shape"] = np.array([E, N, K, M, top_k], dtype=np.int64)
        for k, v in c.items():
            arrays[f"c{i}_{k}"] = v.numpy()
    np.savez_compressed(os.path.join(HERE, "moe_gemm_reference.npz"), **arrays)
    print(f"wrote {len(CASES)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_moe_golden.py <path of the reference checkout>")
    main(sys.argv[1])

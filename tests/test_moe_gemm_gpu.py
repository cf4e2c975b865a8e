"""GPU parity of the grouped MXFP4 x FP8 MoE GEMM (r4d_gemm_moe_mxfp4a8_nt_b16's contract,
csrc/moe_gemm.cu) against the fp32 dequant reference of the reference's own harness
(tests/k1/moe_ref_harness.py, restated in oracle/moe_gemm_oracle.py), on its shapes: the
gate_up projection (N=640, K=2560, top_k=10) and the down projection (N=2560, K=320, top_k=1
with routed weights) at M in {1, 4, 8, 16} tokens, and its "tail" shape (N=80). The
harness's scales make every weight exact, so the only slack is fp32 accumulation order and the
bf16 output: max|y - ref| / max|ref| < 8e-3. The ABI probes the harness runs hold too: only
the rows the live blocks name are written, a block with expert id -1 is skipped, num_post_pad
is read on the device. And the hot / cold split of the MoE layer: the resident experts'
compact copies with r4d_lru_fused's by-slot blocks, the full tensors with its by-expert
blocks, together equal to one unsplit call."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_pkg
from oracle import lru_oracle as LO
from oracle import moe_gemm_oracle as O

pytestmark = pytest.mark.gpu
P = load_pkg()
MO = P.moe_ops
TOL = 8e-3


def _check(y, ref, tag):
    written = ~torch.isnan(y.float()).any(dim=1)
    expected = ~torch.isnan(ref).any(dim=1)
    assert torch.equal(written, expected), f"{tag}: rows written {int(written.sum())} vs {int(expected.sum())}"
    if int(expected.sum()) == 0:
        return 0.0
    d = (y.float()[expected] - ref[expected]).abs().max().item()
    rel = d / ref[expected].abs().max().item()
    assert rel < TOL, f"{tag}: rel {rel:.3e}"
    return rel


def _run(cuda, E, N, K, M, top_k, use_tw, seed):
    w, s, x, topk, tw = O.build_case(E, N, K, M, top_k, seed, cuda)
    qx, xs = O.quant_fp8_per_token(x)
    mtk = M * top_k
    sorted_ids, eids, npad = O.moe_align_block_size(topk, 16, E)
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)
    y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
    MO.mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, sorted_ids, eids, npad, tw if use_tw else None, mtk, top_k)
    ref = O.gemm_ref(qx, xs, w, s, sorted_ids, eids, npad, tw if use_tw else None, mtk, top_k)
    torch.cuda.synchronize()
    assert P._lib.lmhead().b200_moe_gemm_error(1) == 0
    return y, ref


@pytest.mark.parametrize("M", [1, 4, 8, 16])
def test_gate_up(cuda, M):
    y, ref = _run(cuda, 64, 640, 2560, M, 10, False, M)
    print(f"gate_up M={M}: rel {_check(y, ref, f'gate_up M={M}'):.2e}")


@pytest.mark.parametrize("M", [1, 4, 16])
def test_down_with_routed_weights(cuda, M):
    y, ref = _run(cuda, 64, 2560, 320, M * 10, 1, True, 100 + M)
    print(f"down M={M}: rel {_check(y, ref, f'down M={M}'):.2e}")


def test_tail_shape_and_many_rows_per_expert(cuda):
    """N=80 (five 16-row strips) and 8 experts for 40 x 10 routed rows, so blocks are full and
    experts span several blocks."""
    y, ref = _run(cuda, 64, 80, 2560, 8, 10, False, 7)
    _check(y, ref, "tail")
    y, ref = _run(cuda, 8, 640, 2560, 40, 10, False, 9)
    _check(y, ref, "dense")


def test_abi_probes(cuda):
    """The harness's probes (moe_ref_harness.py:262-302): with c pre-filled, exactly the live
    rows are written; expert id -1 skips its block and leaves the rest unchanged; a device
    num_post_pad of 16 writes block 0 only."""
    E, N, K, M, top_k = 64, 640, 2560, 8, 10
    w, s, x, topk, _ = O.build_case(E, N, K, M, top_k, 3, cuda)
    qx, xs = O.quant_fp8_per_token(x)
    mtk = M * top_k
    si, ei, npad = O.moe_align_block_size(topk, 16, E)
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)

    def run(sorted_ids, expert_ids, np_):
        y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        MO.mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, sorted_ids, expert_ids, np_, None, mtk, top_k)
        torch.cuda.synchronize()
        return y, ~torch.isnan(y.float()).any(dim=1)

    y0, written = run(si, ei, npad)
    n = int(npad.item())
    live = torch.zeros(mtk, dtype=torch.bool, device=cuda)
    live[si[:n][si[:n] < mtk].long()] = True
    assert torch.equal(written, live)
    eid = ei.clone()
    eid[0] = -1
    y1, w1 = run(si, eid, npad)
    b0 = si[:16][si[:16] < mtk].long()
    assert not w1[b0].any()
    rest = live.clone()
    rest[b0] = False
    assert torch.equal(w1, rest) and torch.equal(y1[rest], y0[rest])
    y2, w2 = run(si, ei, torch.tensor([16], dtype=torch.int32, device=cuda))
    assert torch.equal(w2.nonzero().flatten().sort().values, b0.sort().values)
    assert torch.equal(y2[b0], y0[b0])


def test_hot_cold_split_through_the_lru(cuda):
    """The MoE layer's split (r4d_mxfp4_moe.py.lru.diff L584-606): the cache's fused step gives
    the by-slot blocks of the resident experts and the by-expert blocks of the others; the hot
    call reads the resident experts' compact copies (gathered by slot), the cold call the full
    tensors; every routed row is written once and the result equals the unsplit call."""
    E, S, N, K, M, top_k = 64, 24, 640, 2560, 4, 10
    w, s, x, topk, _ = O.build_case(E, N, K, M, top_k, 21, cuda)
    qx, xs = O.quant_fp8_per_token(x)
    mtk = M * top_k
    rng = np.random.default_rng(5)
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    lay = P.lru.LruLayer.warm(hot, E, cuda, stamps=torch.as_tensor(rng.permutation(S) + 1), step=S,
                              max_inserts=4)
    align_hot, align_cold = lay.fused(topk.reshape(-1).contiguous())
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)
    slot_e = lay.slot_expert.long()
    hot_w = (wq[slot_e], ws[slot_e], wref[slot_e])                  # compact copies, by slot
    y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
    MO.gemm_split(y, qx, xs, (wq, ws, wref), hot_w, align_hot, align_cold, None, mtk, top_k)
    si, ei, npad = O.moe_align_block_size(topk, 16, E)
    ref = O.gemm_ref(qx, xs, w, s, si, ei, npad, None, mtk, top_k)
    torch.cuda.synchronize()
    assert not torch.isnan(y.float()).any()
    _check(y, ref, "hot/cold")
    y_one = torch.full_like(y, float("nan"))
    MO.mxfp4_moe_gemm_into(y_one, qx, xs, wq, ws, wref, si, ei, npad, None, mtk, top_k)
    torch.cuda.synchronize()
    assert torch.equal(y, y_one)          # same per-row arithmetic whichever call writes the row


def test_graph_replay(cuda):
    E, N, K, M, top_k = 64, 640, 2560, 4, 10
    w, s, x, topk, _ = O.build_case(E, N, K, M, top_k, 31, cuda)
    qx, xs = O.quant_fp8_per_token(x)
    mtk = M * top_k
    si, ei, npad = O.moe_align_block_size(topk, 16, E)
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)
    y = torch.empty(mtk, N, dtype=torch.bfloat16, device=cuda)
    MO.mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, si, ei, npad, None, mtk, top_k)
    torch.cuda.synchronize()
    want = y.clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        torch.ops.vllm.r4d_mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, si, ei, npad, None, mtk, top_k, 1, 1, 1)
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        torch.ops.vllm.r4d_mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, si, ei, npad, None, mtk, top_k, 1, 1, 1)
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, want)


def test_reference_harness_cases(cuda):
    """The kernel on the cases tests/golden/make_moe_golden.py made with the reference's own
    harness functions, against that harness's fp32 output (routed weights applied here, as
    the harness's down-projection check does)."""
    from conftest import golden
    z = golden("moe_gemm_reference.npz")
    for i in range(len([k for k in z.files if k.endswith("_shape")])):
        c = {k[len(f"c{i}_"):]: torch.from_numpy(z[k]) for k in z.files if k.startswith(f"c{i}_")}
        E, N, K, M, top_k = (int(v) for v in c["shape"])
        mtk = M * top_k
        wq, ws, wref = MO.pack_mxfp4_moe(c["w"].to(cuda), c["s"].to(cuda))
        qx = c["qx"].to(cuda).view(torch.float8_e4m3fn)
        xs, tw = c["xs"].to(cuda), c["tw"].to(cuda)
        si, ei, npad = c["sorted_ids"].to(cuda), c["expert_ids"].to(cuda), c["npad"].to(cuda)
        for use_tw in (False, True):
            y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
            MO.mxfp4_moe_gemm_into(y, qx, xs, wq, ws, wref, si, ei, npad, tw if use_tw else None, mtk, top_k)
            torch.cuda.synchronize()
            want = c["out"].to(cuda) * (tw.unsqueeze(1) if use_tw else 1.0)
            assert not torch.isnan(y.float()).any(), i
            rel = ((y.float() - want).abs().max() / want.abs().max()).item()
            assert rel < TOL, (i, use_tw, rel)


@pytest.mark.parametrize("E,N,K,M,top_k", [
    (16, 96, 1280, 6, 4),      # two strips per unit: teams of four (or of eight at few units)
    (8, 16, 64, 20, 2),        # one strip, 32 strips per unit (whole-strip warps, team of 16)
    (12, 48, 160, 3, 3),       # ragged run: 3 strips in a 16-strip unit
    (64, 640, 2560, 40, 10),   # many units per CTA: K split in pairs
    (64, 640, 2560, 1, 2),     # at most four units per CTA: K split eight ways
])
def test_team_plans(cuda, E, N, K, M, top_k):
    """Every consumer team plan against the oracle (the split of a strip's K between warps and
    the reduction of their partial sums), with routed weights."""
    y, ref = _run(cuda, E, N, K, M, top_k, True, E * 1000 + K + M)
    _check(y, ref, f"{E}x{N}x{K} M={M} k={top_k}")


def test_hot_cold_entry_edges(cuda):
    """b200_moe_gemm_hot_cold with an empty hot list, an empty cold list and both empty, and
    with expert id -1 in either list: the rows of the live blocks, nothing else."""
    E, N, K, M, top_k = 32, 64, 256, 6, 3
    w, s, x, topk, tw = O.build_case(E, N, K, M, top_k, 41, cuda)
    qx, xs = O.quant_fp8_per_token(x)
    mtk = M * top_k
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)
    si, ei, npad = O.moe_align_block_size(topk, 16, E)
    ref = O.gemm_ref(qx, xs, w, s, si, ei, npad, tw, mtk, top_k)
    empty = (torch.full_like(si, mtk), torch.full_like(ei, -1), torch.zeros_like(npad))
    full = (wq, ws, wref)
    for hot_a, cold_a, want in (((si, ei, npad), empty, ref), (empty, (si, ei, npad), ref),
                                (empty, empty, torch.full_like(ref, float("nan")))):
        y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
        MO.gemm_split(y, qx, xs, full, full, hot_a, cold_a, tw, mtk, top_k)
        torch.cuda.synchronize()
        _check(y, want, "edge")
    # expert -1 on the first block of the hot list and on the last live block of the cold list
    nb = int(npad.item()) // 16
    half = nb // 2
    h_si, c_si = si.clone(), si.clone()
    h_ei, c_ei = ei.clone(), ei.clone()
    h_ei[half:] = -1
    c_ei[:half] = -1
    h_ei[0] = -1
    c_ei[nb - 1] = -1
    y = torch.full((mtk, N), float("nan"), dtype=torch.bfloat16, device=cuda)
    MO.gemm_split(y, qx, xs, full, full, (h_si, h_ei, npad), (c_si, c_ei, npad), tw, mtk, top_k)
    torch.cuda.synchronize()
    want = ref.clone()
    dead = torch.cat([si[0:16], si[(nb - 1) * 16: nb * 16]])
    dead = dead[dead < mtk].long()
    want[dead] = float("nan")
    _check(y, want, "expert -1")
    assert P._lib.lmhead().b200_moe_gemm_error(1) == 0

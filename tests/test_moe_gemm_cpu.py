"""CPU checks of the grouped MoE GEMM's host side: the B200 packing round-trips the
checkpoint codes and scales exactly and puts each code at the mma.sync A-fragment position its
kernel reads; the oracle's dequantization and align follow the reference harness's
definitions on hand-made cases; the C entry's argument checks (no GPU call is made)."""
from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import load_pkg
from oracle import moe_gemm_oracle as O

P = load_pkg()
MO = P.moe_ops


@pytest.mark.parametrize("E,N,K", [(3, 32, 128), (2, 640, 2560), (2, 2560, 320), (1, 80, 64)])
def test_pack_round_trip(E, N, K):
    g = torch.Generator().manual_seed(N + K)
    w = torch.randint(0, 256, (E, N, K // 2), generator=g, dtype=torch.uint8)
    s = torch.randint(100, 140, (E, N, K // 32), generator=g, dtype=torch.uint8)
    wq, ws, wref = MO.pack_mxfp4_moe(w, s)
    assert wq.shape == (E, N // 16, (K // 32) * 272) and ws.shape == (E, N // 16, 16, K // 32)
    assert torch.equal(wref, s.max(dim=2).values)
    assert torch.equal(wq[:, :, (K // 32) * 256:].reshape(E, N, K // 32), s)     # exponents in the record
    w2, s2 = MO.unpack_mxfp4_moe(wq)
    assert torch.equal(w2, w) and torch.equal(s2, s)


def test_pack_fragment_positions():
    """Code of (row r, k) lands in lane 4 (r % 8) + (k % 8) // 2 of its group, byte
    4 (k // 16) + 2 ((k % 16) // 8) + r // 8, nibble k % 2."""
    for r, k in ((1, 27), (9, 0), (15, 31), (0, 17), (8, 12)):
        codes = torch.zeros(16, 32, dtype=torch.uint8)
        codes[r, k] = 0xB
        w = (codes[:, 0::2] | (codes[:, 1::2] << 4)).unsqueeze(0)
        wq, _, _ = MO.pack_mxfp4_moe(w, torch.full((1, 16, 1), 127, dtype=torch.uint8))
        lane = 4 * (r % 8) + (k % 8) // 2
        h, pair, j = k // 16, 2 * ((k % 16) // 8) + r // 8, k % 2
        b = wq[0, 0, :256].view(32, 8)[lane]
        word = sum(int(b[4 * h + i]) << (8 * i) for i in range(4))
        assert word == 0xB << (8 * pair + 4 * j), (r, k, hex(word))
        assert int(wq[0, 0, :256].view(torch.int64).ne(0).sum()) == 1


def test_dequant_and_align_hand_cases():
    w = torch.tensor([[0x21, 0xF9] + [0] * 14], dtype=torch.uint8)     # k0=1 (0.5) k1=2 (1.0) k2=9 (-0.5) k3=15 (-6)
    s = torch.tensor([[128]], dtype=torch.uint8)                        # 2^1
    d = O.dequant_expert(w, s)
    assert d[0, :4].tolist() == [1.0, 2.0, -1.0, -12.0] and d[0, 4:].abs().sum() == 0
    topk = torch.tensor([[3, 1], [3, 0]], dtype=torch.int32)            # flat ids 0..3 -> experts 3,1,3,0
    si, ei, npad = O.moe_align_block_size(topk, 4, 4)
    assert npad.item() == 12
    assert si[:12].tolist() == [3, 4, 4, 4, 1, 4, 4, 4, 0, 2, 4, 4]
    assert ei[:3].tolist() == [0, 1, 3]
    si2, ei2, np2 = O.moe_align_block_size(topk, 4, 4, expert_map=torch.tensor([-1, 0, -1, 1]))
    assert np2.item() == 8 and si2[:8].tolist() == [1, 4, 4, 4, 0, 2, 4, 4] and ei2[:2].tolist() == [0, 1]


def test_c_entry_argument_codes():
    lib = P._lib.lmhead()
    f = lib.r4d_gemm_moe_mxfp4a8_nt_b16
    last = lib.r4d_gemm_moe_mxfp4a8_nt_b16_last_error
    base = [16 * 1024] * 10                                  # aligned placeholder addresses
    f(*base, 8, 40, 10, 2560, 640, 1, 1, 1, 0)               # em < 16
    assert last() == -1
    f(*base, 800, 40, 10, 2560, 648 + 1, 1, 1, 1, 0)         # N % 16
    assert last() == -2
    f(*base, 800, 40, 10, 2560 + 16, 640, 1, 1, 1, 0)        # K % 32
    assert last() == -3
    bad = list(base)
    bad[2] = 16 * 1024 + 8                                   # wq not 16-byte aligned
    f(*bad, 800, 40, 10, 2560, 640, 1, 1, 1, 0)
    assert last() == -10
    assert lib.b200_moe_gemm_smem_bytes(2560) > 0 and lib.b200_moe_gemm_smem_bytes(320) > 0
    assert lib.b200_moe_gemm_smem_bytes(1 << 16) == -1 and lib.b200_moe_gemm_smem_bytes(48) == -1
    assert lib.r4d_gemm_moe_mxfp4a8_nt_b16_block() == 16 and lib.r4d_gemm_moe_mxfp4a8_nt_b16_group() == 32


def _golden_cases():
    from conftest import golden
    z = golden("moe_gemm_reference.npz")
    n = len([k for k in z.files if k.endswith("_shape")])
    for i in range(n):
        yield i, {k[len(f"c{i}_"):]: z[k] for k in z.files if k.startswith(f"c{i}_")}


def test_oracle_matches_reference_harness():
    """The oracle against fixtures made by the reference's own MoE harness
    (tests/golden/make_moe_golden.py): dequantisation, per-token FP8 quant and the block
    alignment bit for bit; the fp32 reference output to fp32 rounding (the harness multiplies
    each expert's rows at once, the oracle each block's)."""
    for i, c in _golden_cases():
        E, N, K, M, top_k = (int(v) for v in c["shape"])
        w, s = torch.from_numpy(c["w"]), torch.from_numpy(c["s"])
        assert torch.equal(O.dequant_expert(w[0], s[0]), torch.from_numpy(c["deq0"])), i
        qx, xs = O.quant_fp8_per_token(torch.from_numpy(c["x"]))
        assert torch.equal(qx.view(torch.uint8), torch.from_numpy(c["qx"])), i
        assert torch.equal(xs, torch.from_numpy(c["xs"])), i
        si, ei, npad = O.moe_align_block_size(torch.from_numpy(c["topk"]), 16, E)
        assert torch.equal(si, torch.from_numpy(c["sorted_ids"])), i
        assert torch.equal(ei, torch.from_numpy(c["expert_ids"])), i
        assert torch.equal(npad, torch.from_numpy(c["npad"])), i
        ref = O.gemm_ref(qx, xs, w, s, si, ei, npad, None, M * top_k, top_k)
        want = torch.from_numpy(c["out"])
        assert not torch.isnan(ref).any(), i                  # every routed row is named
        assert torch.allclose(ref, want, rtol=1e-5, atol=1e-5 * want.abs().max().item()), i


def test_pack_of_reference_cases_round_trips():
    for i, c in _golden_cases():
        w, s = torch.from_numpy(c["w"]), torch.from_numpy(c["s"])
        wq, _, wref = MO.pack_mxfp4_moe(w, s)
        w2, s2 = MO.unpack_mxfp4_moe(wq)
        assert torch.equal(w2, w) and torch.equal(s2, s) and torch.equal(wref, s.max(dim=2).values), i


def test_hot_cold_entry_argument_codes():
    """b200_moe_gemm_hot_cold refuses bad arguments before any CUDA call (no GPU here)."""
    lib = P._lib.lmhead()
    f = lib.b200_moe_gemm_hot_cold
    A = 16 * 1024
    def call(wq_cold=A, em_hot=800, em_cold=800, N=640, K=2560, mtk=40, top_k=10, qx=A):
        return f(qx, A, A, wq_cold, A, A, A, A, em_hot, A, A, A, em_cold, None, mtk, top_k, K, N, None)
    assert call(wq_cold=A + 8) == -10
    assert call(qx=A + 4) == -10
    assert call(em_hot=8) == -1 and call(em_cold=8) == -1
    assert call(top_k=0) == -1 and call(mtk=-1) == -1
    assert call(N=650) == -2
    assert call(K=2560 + 16) == -3
    assert call(mtk=0) == 0                      # nothing to do: returns before any launch

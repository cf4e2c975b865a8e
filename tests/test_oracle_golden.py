"""The CPU oracle, pinned against fixtures produced by the reference's own code
(tests/golden/make_golden.py): W4 quantize/pack/unpack, FP8 block pack, the numpy LRU
model ``ref_step`` over test_lru.py's five policy suites and test_victim_equiv.py's 19
victim-selection cases. Also the B200 packed layouts' round trips. CPU only."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import lru_oracle as LO
from oracle import quant_oracle as Q


# ---------------------------------------------------------------------------------------
# W4
# ---------------------------------------------------------------------------------------

W4_SHAPES = [(48, 256), (200, 256), (32, 384)]


@pytest.mark.parametrize("n,k", W4_SHAPES)
@pytest.mark.parametrize("tag", ["clip", "minmax"])
def test_quantize_w4_matches_reference(n, k, tag):
    g = golden("w4_reference.npz")
    w = torch.from_numpy(g[f"{n}x{k}_{tag}_w"]).view(torch.bfloat16)
    clip = None if tag == "clip" else (1.0,)
    q, s, z = Q.quantize_w4(w.float(), 128, clip)
    assert np.array_equal(q.numpy(), g[f"{n}x{k}_{tag}_q"])
    assert np.array_equal(s.view(torch.int16).numpy(), g[f"{n}x{k}_{tag}_scale"])
    assert np.array_equal(z.numpy(), g[f"{n}x{k}_{tag}_zero"])


@pytest.mark.parametrize("n,k", W4_SHAPES)
@pytest.mark.parametrize("tag", ["clip", "minmax"])
def test_w4_sz_and_unpack_match_reference(n, k, tag):
    """The reference's wsz dword format and unpack_w4 values, reproduced exactly from the
    oracle's (q, scale, zero) -- with N padded to 16 by zero rows (draft_w4_lmhead.py:242-253)."""
    g = golden("w4_reference.npz")
    w = torch.from_numpy(g[f"{n}x{k}_{tag}_w"]).view(torch.bfloat16)
    n_pad = int(g[f"{n}x{k}_{tag}_npad"][0])
    assert n_pad == (n + 15) // 16 * 16
    wp = torch.cat([w, w.new_zeros(n_pad - n, k)]) if n_pad > n else w
    clip = None if tag == "clip" else (1.0,)
    q, s, z = Q.quantize_w4(wp.float(), 128, clip)
    assert np.array_equal(Q.pack_sz(s, z).numpy(), g[f"{n}x{k}_{tag}_wsz"])
    up = Q.w4_dequant(q, s, z)
    ref_sum = g[f"{n}x{k}_{tag}_unpack_sum"]
    assert up.double().sum().item() == pytest.approx(ref_sum[0], rel=0, abs=1e-9)
    assert up.double().abs().sum().item() == pytest.approx(ref_sum[1], rel=0, abs=1e-9)
    if n == 48:
        assert np.array_equal(up.numpy(), g[f"{n}x{k}_{tag}_unpack"])
    s2, z2 = Q.unpack_sz(Q.pack_sz(s, z))
    assert torch.equal(s2, s) and torch.equal(z2, z.float())


def test_w4_b200_code_layout_roundtrip():
    g = torch.Generator().manual_seed(3)
    q = torch.randint(0, 16, (64, 512), generator=g, dtype=torch.uint8)
    packed = Q.pack_codes_b200(q)
    assert packed.numel() * 4 == q.numel() // 2
    assert torch.equal(Q.unpack_codes_b200(packed, 64, 512), q)
    # lane (g=1, t=2), word w=3 of strip 0, kb 0 holds k = 32*3 + 8*2 + j of row 1
    word = int(packed.view(-1)[((0 * 8 + 1) * 4 + 2) * 4 + 3].item()) & 0xFFFFFFFF
    for j in range(8):
        assert (word >> (4 * Q.W4_NIBBLE[j])) & 0xF == int(q[1, 96 + 16 + j])


# ---------------------------------------------------------------------------------------
# FP8
# ---------------------------------------------------------------------------------------

def test_pack_fp8_block_matches_reference():
    g = golden("fp8_pack_reference.npz")
    w = torch.from_numpy(g["w"]).view(torch.bfloat16)
    wq, ws = Q.pack_fp8_block(w)
    assert np.array_equal(wq.view(torch.uint8).numpy(), g["wq"])
    assert np.array_equal(ws.numpy(), g["ws"])
    assert ws[1, 1].item() == pytest.approx(1e-12 / 448.0, rel=1e-6)   # all-zero block floor


def test_fp8_strip_swizzle_roundtrip():
    g = golden("fp8_pack_reference.npz")
    wq = torch.from_numpy(g["wq"]).view(Q.FP8)
    sw = Q.fp8_tile_swizzle(wq)
    assert torch.equal(Q.fp8_tile_unswizzle(sw).view(torch.uint8), wq.view(torch.uint8))
    N, K = wq.shape
    raw = sw.view(torch.uint8).reshape(-1)
    for (n, k) in [(0, 0), (5, 17), (127, 383), (200, 130), (255, 255)]:
        st, r, kb, c, b = n // 16, n % 16, k // 128, (k % 128) // 16, k % 16
        off = ((st * (K // 128) + kb) * 16 + r) * 128 + ((c ^ (r & 7)) * 16) + b
        assert raw[off] == wq.view(torch.uint8)[n, k]


def test_group_quant_known_answers():
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    x[1, 0] = 448.0
    x[1, 130] = -1.0
    q, s = Q.group_quant_fp8(x)
    eps_scale = torch.tensor(1e-10, dtype=torch.float32) * torch.tensor(1 / 448.0, dtype=torch.float32)
    assert s[0, 0].item() == eps_scale.item()
    assert s[1, 0].item() == pytest.approx(1.0, rel=1e-7)
    assert q.float()[1, 0].item() == 448.0
    assert q.float()[1, 130].item() == -448.0


def test_silu_quant_zero_row_floor():
    """A zero row lands on the floor 1/(448*512) (tests/k4/probe_silu_quant.py:46-53)."""
    z = torch.zeros(4, 640, dtype=torch.bfloat16)
    _, q, s = Q.silu_mul_quant(z)
    assert torch.all(s == torch.tensor(1.0 / (448.0 * 512.0), dtype=torch.float32))
    assert float(s[0, 0]) == pytest.approx(4.35965e-6, rel=1e-5)
    assert torch.all(q.view(torch.uint8) == 0)


# ---------------------------------------------------------------------------------------
# LRU
# ---------------------------------------------------------------------------------------

@pytest.mark.parametrize("name", list(LO.SUITES))
def test_lru_oracle_matches_ref_step_every_step(name):
    g = golden("lru_reference.npz")
    E, S, nsteps, md, maxi = LO.SUITES[name]
    rng, st = LO.suite_start(name, seed=0)
    assert np.array_equal(st.table, g[f"{name}/init_table"])
    ids_all = g[f"{name}/ids"]
    digests = g[f"{name}/digest"]
    nm_all = g[f"{name}/n_miss"]
    misses = g[f"{name}/miss"].reshape(-1, 2)
    off = 0
    gen = LO.suite_gen(name)
    for n in range(nsteps):
        ids = np.asarray(gen(rng, n)).ravel()
        assert np.array_equal(ids, ids_all[n]), "restated generator drifted from the fixture"
        nm = LO.manage(st, ids, md, maxi)
        assert nm == nm_all[n]
        assert np.array_equal(st.miss[:nm], misses[off:off + nm])
        off += nm
        assert LO.state_digest(st) == digests[n], f"{name} step {n}"
        assert not LO.check_invariants(st)
    assert np.array_equal(st.slot_stamp, g[f"{name}/final_st"])


def _case_state(g, i):
    k = f"case{i}"
    E, S, mk, maxi, md = (int(v) for v in g[f"{k}/params"])
    st = LO.LruState(g[f"{k}/table"].copy(), g[f"{k}/map_cold"].copy(),
                     g[f"{k}/slot_expert"].copy(), g[f"{k}/slot_stamp"].copy(),
                     int(g[f"{k}/step"][0]))
    st.miss = np.full((max(maxi, 1), 2), -1, dtype=np.int32)
    return st, g[f"{k}/ids"], md, maxi


@pytest.mark.parametrize("i", range(19))
def test_lru_oracle_matches_ref_step_victim_cases(i):
    g = golden("lru_reference.npz")
    st, ids, md, maxi = _case_state(g, i)
    LO.manage(st, ids, md, maxi)
    assert LO.state_digest(st) == g[f"case{i}/digest"][0], str(g["case_names"][i])


def test_lru_fused_oracle_equals_manage_plus_two_aligns():
    """lru_fused == manage + moe_align(table) + moe_align(map_cold) from the same state
    (tests/lru/test_fused.py:198-222), exact with stable in-bucket order."""
    g = golden("lru_reference.npz")
    for i in range(19):
        a, ids, md, maxi = _case_state(g, i)
        b = a.copy()
        out = LO.fused(a, ids, md, maxi, 16)
        LO.manage(b, ids, md, maxi)
        assert LO.state_digest(a) == LO.state_digest(b)
        hot = LO.moe_align_block_size(ids, 16, a.E, b.table)
        cold = LO.moe_align_block_size(ids, 16, a.E, b.map_cold)
        for x, y in zip(out, (*hot, *cold)):
            assert np.array_equal(x, y)
        mk = len(ids)
        tok = np.concatenate([out[0][:out[2][0]], out[3][:out[5][0]]])
        tok = np.sort(tok[tok != mk])
        assert np.array_equal(tok, np.arange(mk)), "hot+cold must partition [0, mk)"


def test_align_sizes_formula():
    assert LO.align_sizes(50, 512, 16) == (800, 50)
    assert LO.align_sizes(200, 512, 16) == (3200, 200)
    assert LO.align_sizes(2048, 512, 16) == (2048 + 512 * 15, (2048 + 512 * 15 + 15) // 16)


def test_residency_audit_catches_a_planted_byte():
    """The audit of tests/lru/test_slots_prod.py, with its negative control done on the CPU:
    a consistent cache passes, one flipped byte in one slot's slab is reported (slot, buffer)."""
    rng = np.random.default_rng(2)
    E, S, sizes = 64, 16, [32, 16]
    src = [rng.integers(0, 256, E * b, dtype=np.uint8) for b in sizes]
    hot = sorted(rng.choice(E, S, replace=False).tolist())
    st = LO.warm_state(E, S, hot, cap=8)
    dst = [np.zeros(S * b, dtype=np.uint8) for b in sizes]
    for sl, e in enumerate(hot):
        for d, sv, b in zip(dst, src, sizes):
            d[sl * b:(sl + 1) * b] = sv[e * b:(e + 1) * b]
    assert LO.residency_audit(st.slot_expert, dst, src, sizes) == []
    for step in range(5):                                   # manage + gather keep it consistent
        LO.manage(st, rng.choice(E, size=10, replace=False), 32, 8)
        LO.gather_expected(dst, src, sizes, st.miss, st.n_miss)
        assert LO.residency_audit(st.slot_expert, dst, src, sizes) == []
    dst[1][5 * sizes[1] + 3] ^= 0x10                        # the planted mistake
    assert LO.residency_audit(st.slot_expert, dst, src, sizes) == [(5, 1)]

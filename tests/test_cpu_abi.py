"""CPU-only checks of the boundary: both C-ABI libraries load and export every symbol the
headers in include/ declare; argument validation returns the reference's codes before any
launch (so these run without a GPU); the host logic mirrors the reference (pick_cfg/_legal
against the reference's own outputs, align sizes, warm start); the product's packers, run on
CPU tensors, reproduce the reference's quantizer output exactly."""
from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, golden, load_pkg
from oracle import lru_oracle as LO
from oracle import quant_oracle as Q

P = load_pkg()
L = P._lib


def _declared(header: str) -> list[str]:
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    return re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\([^;{]*\)\s*;", src)


@pytest.mark.parametrize("headers,lib", [(["r4d_lru.h"], "librlu.so"),
                                         (["b200_lmhead.h", "b200_moe_tail.h", "b200_moe_gemm.h"],
                                          "libb200lmhead.so")])
def test_every_declared_symbol_is_exported(headers, lib):
    names = [n for h in headers for n in _declared(h)]
    assert len(names) >= 3
    cdll = L.load(lib)
    for n in names:
        assert hasattr(cdll, n), f"{lib} does not export {n}"
    # and the ctypes prototypes cover exactly the declared entry points
    assert set(names) == set(L.LIB_FILES[lib]), set(names) ^ set(L.LIB_FILES[lib])


NULL = ctypes.c_void_p(0)


def _manage(**kw):
    a = dict(mk=10, E=512, S=257, md=128, maxi=64)
    a.update(kw)
    return L.rlu().r4d_lru_manage(NULL, a["mk"], a["E"], a["S"], a["md"], a["maxi"],
                                  *([NULL] * 8), NULL)


def test_lru_manage_precondition_codes():
    """r4d_lru.hip:583-584: E<=0, S<=0, S>1024, max_inserts outside [0,1024] -> -1."""
    assert _manage(E=0) == -1
    assert _manage(S=0) == -1
    assert _manage(S=1025) == -1
    assert _manage(maxi=-1) == -1
    assert _manage(maxi=1025) == -1


def _fused(**kw):
    a = dict(mk=50, E=512, S=257, md=128, maxi=64, bs=16, L=800, NB=50)
    a.update(kw)
    return L.rlu().r4d_lru_fused(NULL, a["mk"], a["E"], a["S"], a["md"], a["maxi"],
                                 *([NULL] * 8), a["bs"], a["L"], a["NB"], *([NULL] * 6), NULL)


def test_lru_fused_precondition_codes():
    """r4d_lru.hip:602-604."""
    assert _fused(E=1025) == -1
    assert _fused(S=1025) == -1
    assert _fused(bs=0) == -1
    assert _fused(L=0) == -1
    assert _fused(NB=0) == -1
    assert _fused(mk=-1) == -1
    assert _fused(maxi=1025) == -1


def test_lru_gather_precondition_codes():
    """r4d_lru.hip:617-620: every slab size a positive multiple of 16, chunks/lanes > 0."""
    def g(sizes, chunks=8, lanes=16):
        args = []
        for b in sizes:
            args += [NULL, NULL, ctypes.c_long(b)]
        return L.rlu().r4d_lru_gather(*args, NULL, NULL, chunks, lanes, NULL)
    ok = [819200, 409600, 51200, 640, 25600, 2560]
    assert g([8] + ok[1:]) == -1
    assert g(ok[:5] + [0]) == -1
    assert g(ok, chunks=0) == -1
    assert g(ok, lanes=0) == -1


def test_hcq_precondition_codes():
    """The reference's own precondition table (tests/k3/test_fp8sk.py:111-117)."""
    lib = L.lmhead()
    N, K = 2560, 3072
    for args, want in [((17, K, N, 2, 4, 1), -1), ((0, K, N, 2, 4, 1), -1),
                       ((16, K, N + 16, 2, 4, 1), -2), ((16, K, N, 2, 5, 1), -4),
                       ((16, K, N, 64, 4, 1), -5), ((16, K, N, 2, 4, 3), -6)]:
        assert lib.hcq_gemm_fp8blk_nt_m16(NULL, NULL, NULL, NULL, NULL, *args, NULL) == want, args
    assert lib.hcq_gemm_fp8blk_nt_m16(NULL, NULL, NULL, NULL, NULL, 16, K + 64, N, 2, 4, 1, NULL) == -3
    # -7: the reference's LDS budget ((WV*NPW*SK*256 + 16*K/128) * 4 > 64 KB)
    assert lib.hcq_gemm_fp8blk_nt_m16(NULL, NULL, NULL, NULL, NULL, 16, K, N, 8, 4, 4, NULL) == -7
    assert lib.hcq_gemm_fp8blk_nt_m16_max_m() == 16


def test_lmhead_entry_codes():
    lib = L.lmhead()
    assert lib.b200_fp8_lmhead(NULL, -1, 2560, NULL, NULL, 256, 0, NULL, 0, NULL, NULL, NULL,
                               NULL, NULL, NULL, 0, NULL) == -1
    assert lib.b200_fp8_lmhead(NULL, 1, 2560, NULL, NULL, 200, 0, NULL, 0, NULL, NULL, NULL,
                               NULL, NULL, NULL, 0, NULL) == -2
    assert lib.b200_fp8_lmhead(NULL, 1, 2500, NULL, NULL, 256, 0, NULL, 0, NULL, NULL, NULL,
                               NULL, NULL, NULL, 0, NULL) == -3
    # stats asked for without a workspace
    out = ctypes.c_void_p(16)
    assert lib.b200_fp8_lmhead(NULL, 1, 2560, NULL, NULL, 256, 0, NULL, 0, out, NULL, NULL,
                               NULL, NULL, NULL, 0, NULL) == -9
    assert lib.b200_w4_lmhead(NULL, 0, 1, 2560, NULL, NULL, 1000, 1000, 0, NULL, 0, NULL, NULL,
                              NULL, NULL, 0, NULL) == -2
    assert lib.b200_w4_lmhead(NULL, 7, 1, 2560, NULL, NULL, 1008, 1000, 0, NULL, 0, NULL, NULL,
                              NULL, NULL, 0, NULL) == -11
    assert lib.b200_silu_mul_quant(NULL, 4, 16384, 32768, 0, NULL, NULL, NULL, 0, NULL) == -1
    assert lib.b200_silu_mul_quant(NULL, 4, 512, 1024, 5, NULL, NULL, NULL, 0, NULL) == -2
    assert lib.b200_silu_mul_quant(NULL, 0, 512, 1024, 0, NULL, NULL, NULL, 0, NULL) == 0
    assert lib.r4d_gemm_w4a16_nt_m64_max_m() == 64 and lib.r4d_gemm_w4a16_nt_m64_group() == 128
    assert lib.b200_lmhead_workspace_bytes() >= 16 + 148 * 16 * 12
    # the built-in-scratch entry refuses sizes before it touches any device
    big_k = 16384 + 128
    assert lib.b200_fp8_lmhead_static_scratch(NULL, 1, big_k, NULL, NULL, 256, 0, NULL, 0, NULL, NULL,
                                              NULL, NULL, NULL, NULL) == -9
    assert lib.b200_fp8_lmhead_static_scratch(NULL, -1, 2560, NULL, NULL, 256, 0, NULL, 0, NULL, NULL,
                                              NULL, NULL, NULL, NULL) == -1
    assert lib.b200_fp8_lmhead_static_scratch(NULL, 0, 2560, NULL, NULL, 256, 0, NULL, 0, NULL, NULL,
                                              NULL, NULL, NULL, NULL) == 0
    # peer buffer of the NVLink combine: [2 parities][world][M_cap][4 tagged 8-byte words]
    for world, m_cap in ((1, 64), (2, 64), (8, 256)):
        assert lib.b200_p2p_combine_bytes(world, m_cap) == 2 * world * m_cap * 4 * 8
    # bad sizes and ranks are refused before any launch
    for M, m_cap, rank, world in ((65, 64, 0, 2), (-1, 64, 0, 2), (8, 64, 2, 2), (8, 64, 0, 0)):
        assert lib.b200_p2p_combine_row_stats(NULL, NULL, NULL, M, m_cap, NULL, rank, world, NULL, NULL,
                                              NULL, NULL, NULL) == -1


def test_pick_cfg_and_legal_match_reference():
    g = golden("w4_reference.npz")
    W = P.draft_w4_lmhead
    for m, n_pad, k, wv, sk, npw, nt in g["pick_cfg"].tolist():
        assert W.pick_cfg(m, n_pad, k) == (wv, sk, npw, nt), (m, n_pad, k)
    for k, nt, wv, sk, npw, ok in g["legal"].tolist():
        assert bool(W._legal(k, nt, wv, sk, npw)) == bool(ok)


def test_align_sizes_match_vllm_wrapper():
    for mk in (0, 1, 50, 200, 511, 512, 2048):
        assert P.lru._align_sizes(mk, 512, 16) == LO.align_sizes(mk, 512, 16)


def test_lru_layer_warm_start_profile_rank():
    """Hottest profile expert gets stamp S, coldest 1; step = S; max_distinct = int(S*thresh)
    (r4d_mxfp4_moe.py.lru.diff L512-533)."""
    hot = [5, 1, 9, 3]
    rank = {9: 0, 5: 1, 3: 2, 1: 3}
    lay = P.lru.LruLayer.warm(hot, 16, "cpu", profile_rank=rank, thresh=0.5, max_inserts=64)
    assert lay.slot_stamp.tolist() == [3, 1, 4, 2]
    assert lay.step.item() == 4 and lay.max_distinct == 2 and lay.max_inserts == 4
    assert lay.table[9].item() == 2 and lay.map_cold[9].item() == -1 and lay.map_cold[0].item() == 0


@pytest.mark.parametrize("n,k", [(48, 256), (200, 256), (32, 384)])
def test_product_w4_packer_reproduces_reference(n, k):
    """pack_w4a16 / unpack_w4 of the package, run on CPU tensors: codes, scales and zeros
    identical to the reference's quantize_w4, unpack identical to the reference's unpack_w4."""
    g = golden("w4_reference.npz")
    W = P.draft_w4_lmhead
    for tag, clip in (("clip", None), ("minmax", (1.0,))):
        w = torch.from_numpy(g[f"{n}x{k}_{tag}_w"]).view(torch.bfloat16)
        p = W.pack_w4a16(w, 128, clip_grid=clip)
        assert p.n_pad == int(g[f"{n}x{k}_{tag}_npad"][0]) and p.nbytes == p.n_pad * k // 2 + p.n_pad * k // 128 * 4
        assert np.array_equal(p.wsz.numpy(), g[f"{n}x{k}_{tag}_wsz"])
        codes = W._unpack_codes(p.wq, p.n_pad, k)[:n]
        assert np.array_equal(codes.numpy(), g[f"{n}x{k}_{tag}_q"])
        assert torch.equal(W._unpack_codes(p.wq, p.n_pad, k), Q.unpack_codes_b200(
            p.wq.view(torch.int32), p.n_pad, k))
        up = W.unpack_w4(p, torch.float32)
        if n == 48:
            assert np.array_equal(up.numpy(), g[f"{n}x{k}_{tag}_unpack"])
        s = g[f"{n}x{k}_{tag}_unpack_sum"]
        assert up.double().sum().item() == pytest.approx(s[0], abs=1e-9)


@pytest.mark.parametrize("n,k", [(48, 256), (200, 384)])
def test_product_w4_sym_packer_matches_oracle(n, k):
    """The symmetric bf16-scale format (no reference implementation exists): the package's
    quantizer equals the oracle's restatement bit for bit (all-zero and single-spike groups
    included), and unpack(pack) equals the oracle's dequantization exactly."""
    W = P.draft_w4_lmhead
    g = torch.Generator().manual_seed(n * k)
    w = (torch.randn(n, k, generator=g) * 0.02).bfloat16()
    w[1, :128] = 0
    w[2, 128:256] = 0
    w[2, 130] = 0.3
    q1, s1 = W.quantize_w4_sym(w)
    q2, s2 = Q.quantize_w4_sym(w)
    assert torch.equal(q1, q2) and torch.equal(s1.view(torch.int16), s2.view(torch.int16))
    assert q1.max().item() <= 15 and s1[1, 0].item() == 0 and q1[1, :128].eq(8).all()
    p = W.pack_w4a16_sym(w)
    assert p.sym and p.wsz.dtype == torch.bfloat16 and p.nbytes == p.n_pad * k // 2 + p.n_pad * k // 128 * 2
    assert torch.equal(W._unpack_codes(p.wq, p.n_pad, k)[:n], q2)
    assert torch.equal(W.unpack_w4(p, torch.float32)[:n], Q.w4_dequant_sym(q2, s2))


def test_product_fp8_packer_reproduces_reference():
    g = golden("fp8_pack_reference.npz")
    F8 = P.fp8_target_lmhead
    w = torch.from_numpy(g["w"]).view(torch.bfloat16)
    wq, ws = F8.pack_fp8_block(w)
    assert np.array_equal(F8.unpack_fp8_block(wq).view(torch.uint8).numpy(), g["wq"])
    assert np.array_equal(ws.numpy(), g["ws"])
    assert torch.equal(wq.view(torch.uint8), Q.fp8_tile_swizzle(torch.from_numpy(g["wq"]).view(Q.FP8)).view(torch.uint8))


def test_ops_fail_loudly_without_gpu():
    """The product path has no CPU fallback."""
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    assert not P.draft_w4_lmhead.available() and not P.fp8_target_lmhead.available()
    x = torch.zeros(2, 64, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        P.fused_silu_mul_quant.silu_mul_quant(x, torch.float8_e4m3fn)

"""Persisted W4 / FP8 head packs (packs.py): round trips of every format on CPU tensors, the
refusals (corrupt, truncated, foreign kind, other layout or format version, other source
weight), the digest, the cached re-pack path; on the GPU, a head run from a loaded pack
gives the same outputs as the in-memory pack."""
from __future__ import annotations

import json
import struct

import pytest
import torch

from conftest import load_pkg

P = load_pkg()
PK = P.packs
W4 = P.draft_w4_lmhead
F8 = P.fp8_target_lmhead


def _w(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * 0.02).bfloat16()


@pytest.mark.parametrize("sym", [False, True])
def test_w4_round_trip(tmp_path, sym):
    w = _w(1000, 512)
    p = W4.pack_w4a16_sym(w) if sym else W4.pack_w4a16(w)
    f = str(tmp_path / "w4.pack")
    PK.save_w4(f, p, PK.weight_digest(w))
    q = PK.load_w4(f, expect_source=PK.weight_digest(w), sym=sym)
    assert (q.n, q.n_pad, q.k, q.sym) == (p.n, p.n_pad, p.k, p.sym)
    assert torch.equal(q.wq, p.wq) and torch.equal(q.wsz.view(torch.uint8), p.wsz.view(torch.uint8))
    assert torch.equal(W4.unpack_w4(q, torch.float32), W4.unpack_w4(p, torch.float32))
    with pytest.raises(PK.PackFormatError):
        PK.load_w4(f, sym=not sym)                          # the other format's kind


def test_fp8_round_trip(tmp_path):
    w = _w(1024, 512)
    wq, ws = F8.pack_fp8_block(w)
    f = str(tmp_path / "f.pack")
    PK.save_fp8(f, wq, ws, PK.weight_digest(w))
    a, b = PK.load_fp8(f, expect_source=PK.weight_digest(w))
    assert a.dtype == wq.dtype and torch.equal(a.view(torch.uint8), wq.view(torch.uint8))
    assert torch.equal(b, ws)
    with pytest.raises(PK.PackFormatError):
        PK.load_w4(f)                                       # not a W4 pack


def _pack_file(tmp_path):
    w = _w(512, 256, 1)
    wq, ws = F8.pack_fp8_block(w)
    f = tmp_path / "f.pack"
    PK.save_fp8(str(f), wq, ws, PK.weight_digest(w))
    return f, w


def test_refuses_corruption_truncation_and_foreign_files(tmp_path):
    f, w = _pack_file(tmp_path)
    data = bytearray(f.read_bytes())
    bad = tmp_path / "bad.pack"
    hlen = struct.unpack_from("<II", data, 8)[1]
    start = (16 + hlen + PK.ALIGN - 1) // PK.ALIGN * PK.ALIGN
    d = bytearray(data)
    d[start + 10] ^= 0x40                                   # a byte of the first tensor
    bad.write_bytes(bytes(d))
    with pytest.raises(PK.PackFormatError, match="checksum"):
        PK.load_fp8(str(bad))
    bad.write_bytes(bytes(data[:-100]))
    with pytest.raises(PK.PackFormatError, match="truncated"):
        PK.load_fp8(str(bad))
    bad.write_bytes(b"not a pack at all")
    with pytest.raises(PK.PackFormatError, match="not a B200 pack"):
        PK.load_fp8(str(bad))
    with pytest.raises(PK.PackFormatError, match="another weight"):
        PK.load_fp8(str(f), expect_source=PK.weight_digest(_w(512, 256, 2)))


def _rewrite_header(src, dst, edit=None, version=None):
    data = src.read_bytes()
    ver, hlen = struct.unpack_from("<II", data, 8)
    hdr = json.loads(data[16:16 + hlen])
    if edit:
        edit(hdr)
    h2 = json.dumps(hdr, sort_keys=True).encode()
    assert len(h2) <= hlen
    h2 = h2 + b" " * (hlen - len(h2))                       # same length: offsets unchanged
    dst.write_bytes(data[:8] + struct.pack("<II", version or ver, hlen) + h2 + data[16 + hlen:])


def test_refuses_other_layout_or_version(tmp_path):
    f, _ = _pack_file(tmp_path)
    g = tmp_path / "g.pack"
    _rewrite_header(f, g, edit=lambda h: h.update(layout="fp8-other"))
    with pytest.raises(PK.PackFormatError, match="layout"):
        PK.load_fp8(str(g))
    _rewrite_header(f, g, version=PK.VERSION + 1)
    with pytest.raises(PK.PackFormatError, match="version"):
        PK.load_fp8(str(g))
    _rewrite_header(f, g, edit=lambda h: h["tensors"][0].update(dtype="q9"))
    with pytest.raises(PK.PackFormatError, match="header"):
        PK.load_fp8(str(g))
    _rewrite_header(f, g)                                   # unedited copy still loads
    PK.load_fp8(str(g))


def test_weight_digest():
    w = _w(4096, 256)
    assert PK.weight_digest(w) == PK.weight_digest(w.clone())
    w2 = w.clone()
    w2[4095, 0] += 1.0                                      # the last row is always sampled
    assert PK.weight_digest(w2) != PK.weight_digest(w)
    assert PK.weight_digest(w[:4000]) != PK.weight_digest(w)


def test_cached_packs_reuse_and_repack(tmp_path):
    w = _w(1000, 512)
    f = str(tmp_path / "c.pack")
    a = PK.cached_w4(w, f)                                  # packs and writes
    mtime = (tmp_path / "c.pack").stat().st_mtime_ns
    b = PK.cached_w4(w, f)                                  # reads
    assert torch.equal(a.wq, b.wq) and (tmp_path / "c.pack").stat().st_mtime_ns == mtime
    w2 = _w(1000, 512, 5)
    c = PK.cached_w4(w2, f)                                 # another weight: re-packed
    assert torch.equal(c.wq, W4.pack_w4a16(w2).wq)
    wq, ws = PK.cached_fp8(_w(1024, 512), str(tmp_path / "d.pack"))
    wq2, ws2 = PK.cached_fp8(_w(1024, 512), str(tmp_path / "d.pack"))
    assert torch.equal(wq.view(torch.uint8), wq2.view(torch.uint8)) and torch.equal(ws, ws2)


@pytest.mark.gpu
def test_head_from_loaded_pack_matches(tmp_path, cuda):
    w = (torch.randn(4096, 2560, device=cuda) * 0.02).bfloat16()
    f = str(tmp_path / "h.pack")
    wq, ws = F8.pack_fp8_block(w)
    PK.save_fp8(f, wq, ws, PK.weight_digest(w))
    head = F8.Fp8TargetHead(None, w, pack_path=f)           # reads the pack
    x = torch.randn(20, 2560, device=cuda, dtype=torch.bfloat16)
    assert torch.equal(F8.gemm_fp8_block(x, head.wq, head.ws), F8.gemm_fp8_block(x, wq, ws))
    p = W4.pack_w4a16(w)
    PK.save_w4(str(tmp_path / "w.pack"), p)
    q = PK.load_w4(str(tmp_path / "w.pack"), cuda)
    assert torch.equal(W4.gemm_w4a16(x[:4], q), W4.gemm_w4a16(x[:4], p))

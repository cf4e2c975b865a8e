"""Persisted weight packs: the packed W4 draft head (``PackedW4``, either format) and the packed
FP8 target head (``wq``, ``ws``) written to and read from disk, so a server start can skip the
load-time packing (the reference packs at first use: 0.75 s for the real lm_head on its GPU,
kernels/draft_w4_lmhead.py:22, and the FP8 pack at ``Fp8TargetHead`` construction).

File format (little endian): ``b"B200PACK"``, u32 format version, u32 header length, a JSON
header, then each tensor's raw bytes at a 4096-byte aligned offset. The header names the pack
kind, the B200 layout tag the kernels read (a pack written for another layout is refused),
the logical shape (n, n_pad, k), every tensor's dtype, shape, offset, byte count and CRC-32,
and an optional digest of the source weight (``weight_digest``) that ``load_*`` compares
with the caller's so a pack cannot silently outlive a changed checkpoint.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
import zlib

import numpy as np
import torch

from .draft_w4_lmhead import PackedW4

MAGIC = b"B200PACK"
VERSION = 1
ALIGN = 4096
# layout tags of the packed formats the kernels read (bump on any change of a packer)
LAYOUT = {
    "w4": "w4-b200-strip16-nibble-v1",
    "w4sym": "w4sym-b200-strip16-nibble-bf16scale-v1",
    "fp8": "fp8-b200-strip16-swz128-v1",
}
_DTYPES = {torch.uint8: "u1", torch.int32: "i4", torch.float32: "f4", torch.bfloat16: "bf16",
           torch.float8_e4m3fn: "e4m3"}
_NP = {"u1": np.uint8, "i4": np.int32, "f4": np.float32, "bf16": np.uint16, "e4m3": np.uint8}
_TORCH = {v: k for k, v in _DTYPES.items()}


class PackFormatError(ValueError):
    pass


def weight_digest(w: torch.Tensor, samples: int = 64) -> str:
    """Fingerprint of a source weight: its shape, dtype and the bytes of `samples` evenly spaced
    rows (SHA-256). Cheap on a 150k-row head; any re-trained or re-sharded checkpoint changes
    it."""
    h = hashlib.sha256()
    h.update(repr((tuple(w.shape), str(w.dtype))).encode())
    n = w.shape[0]
    idx = torch.linspace(0, n - 1, min(samples, n)).round().long().unique()
    rows = w[idx.to(w.device)].contiguous().cpu()
    h.update(rows.view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def _raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.bfloat16, torch.float8_e4m3fn):
        t = t.view(torch.uint16 if t.dtype == torch.bfloat16 else torch.uint8)
    return t.numpy()


def _write(path: str, kind: str, meta: dict, tensors: dict[str, torch.Tensor],
           source: str | None) -> None:
    entries, blobs, off = [], [], 0
    for name, t in tensors.items():
        a = _raw(t)
        b = a.tobytes()
        entries.append({"name": name, "dtype": _DTYPES[t.dtype], "shape": list(t.shape),
                        "offset": off, "nbytes": len(b), "crc32": zlib.crc32(b)})
        blobs.append(b)
        off += (len(b) + ALIGN - 1) // ALIGN * ALIGN
    header = json.dumps({"kind": kind, "layout": LAYOUT[kind], **meta, "source": source,
                         "tensors": entries}, sort_keys=True).encode()
    start = (len(MAGIC) + 8 + len(header) + ALIGN - 1) // ALIGN * ALIGN
    tmp = f"{path}.{os.getpid()}.tmp"           # per writer: concurrent writers never share it
    with open(tmp, "wb") as f:
        f.write(MAGIC + struct.pack("<II", VERSION, len(header)) + header)
        for e, b in zip(entries, blobs):
            f.seek(start + e["offset"])
            f.write(b)
        f.truncate(start + (entries[-1]["offset"] + entries[-1]["nbytes"] if entries else 0))
    os.replace(tmp, path)                       # a reader never sees a half-written pack


def _read(path: str, kind: str, device, expect_source: str | None) -> tuple[dict, dict]:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < len(MAGIC) + 8 or data[:len(MAGIC)] != MAGIC:
        raise PackFormatError(f"{path}: not a B200 pack")
    version, hlen = struct.unpack_from("<II", data, len(MAGIC))
    if version != VERSION:
        raise PackFormatError(f"{path}: pack format version {version}, this build reads {VERSION}")
    try:
        hdr = json.loads(data[len(MAGIC) + 8:len(MAGIC) + 8 + hlen])
        entries = [(e["name"], _NP[e["dtype"]], _TORCH[e["dtype"]], tuple(e["shape"]), int(e["offset"]),
                    int(e["nbytes"]), int(e["crc32"])) for e in hdr["tensors"]]
    except (ValueError, KeyError, TypeError) as err:
        raise PackFormatError(f"{path}: unreadable pack header ({err})") from err
    if hdr.get("kind") != kind:
        raise PackFormatError(f"{path}: holds a {hdr.get('kind')!r} pack, expected {kind!r}")
    if hdr.get("layout") != LAYOUT[kind]:
        raise PackFormatError(f"{path}: layout {hdr.get('layout')!r}, the kernels read {LAYOUT[kind]!r}")
    if expect_source is not None and hdr.get("source") != expect_source:
        raise PackFormatError(f"{path}: packed from another weight (source digest differs)")
    start = (len(MAGIC) + 8 + hlen + ALIGN - 1) // ALIGN * ALIGN
    out = {}
    for name, npt, want, shape, off, nbytes, crc in entries:
        lo = start + off
        b = data[lo:lo + nbytes]
        if len(b) != nbytes:
            raise PackFormatError(f"{path}: truncated at tensor {name}")
        if zlib.crc32(b) != crc:
            raise PackFormatError(f"{path}: checksum mismatch in tensor {name}")
        if int(np.prod(shape, dtype=np.int64)) * np.dtype(npt).itemsize != nbytes:
            raise PackFormatError(f"{path}: tensor {name} size does not match its shape")
        t = torch.from_numpy(np.frombuffer(b, dtype=npt).reshape(shape).copy())
        if want in (torch.bfloat16, torch.float8_e4m3fn):
            t = t.view(want)
        out[name] = t.to(device) if device is not None else t
    for name in ("wq", "wsz") if kind.startswith("w4") else ("wq", "ws"):
        if name not in out:
            raise PackFormatError(f"{path}: tensor {name} missing")
    return hdr, out


def save_w4(path: str, packed: PackedW4, source: str | None = None) -> None:
    """Write a PackedW4 (either format). ``source``: ``weight_digest`` of the unpacked weight."""
    kind = "w4sym" if packed.sym else "w4"
    _write(path, kind, {"n": packed.n, "n_pad": packed.n_pad, "k": packed.k},
           {"wq": packed.wq, "wsz": packed.wsz}, source)


def load_w4(path: str, device=None, expect_source: str | None = None, sym: bool = False) -> PackedW4:
    """Read a pack written by ``save_w4``; ``sym`` selects the symmetric format."""
    hdr, t = _read(path, "w4sym" if sym else "w4", device, expect_source)
    n, n_pad, k = int(hdr["n"]), int(hdr["n_pad"]), int(hdr["k"])
    wq, wsz = t["wq"], t["wsz"]
    if n_pad % 16 or k % 128 or n > n_pad or tuple(wsz.shape) != (n_pad // 16, k // 128, 16) \
            or wq.numel() * wq.element_size() != n_pad * k // 2:
        raise PackFormatError(f"{path}: tensor shapes do not match n={n} n_pad={n_pad} k={k}")
    return PackedW4(wq=wq, wsz=wsz, n=n, n_pad=n_pad, k=k, sym=sym)


def save_fp8(path: str, wq: torch.Tensor, ws: torch.Tensor, source: str | None = None) -> None:
    """Write the FP8 head pack (``pack_fp8_block``'s wq, ws)."""
    _write(path, "fp8", {"n": int(wq.shape[0]), "k": int(wq.shape[1])}, {"wq": wq, "ws": ws}, source)


def load_fp8(path: str, device=None, expect_source: str | None = None
             ) -> tuple[torch.Tensor, torch.Tensor]:
    """Read a pack written by ``save_fp8`` -> (wq e4m3 [N, K] in the strip layout, ws fp32)."""
    hdr, t = _read(path, "fp8", device, expect_source)
    n, k = int(hdr["n"]), int(hdr["k"])
    wq, ws = t["wq"], t["ws"]
    if tuple(wq.shape) != (n, k) or tuple(ws.shape) != (n // 128, k // 128):
        raise PackFormatError(f"{path}: tensor shapes do not match n={n} k={k}")
    return wq, ws


def cached_w4(weight: torch.Tensor, path: str, sym: bool = False) -> PackedW4:
    """The packed draft head of `weight`, read from `path` when a pack of this very weight
    (same digest, same format and layout) is there, else packed now and written to `path`."""
    from .draft_w4_lmhead import pack_w4a16, pack_w4a16_sym
    digest = weight_digest(weight)
    if os.path.exists(path):
        try:
            return load_w4(path, weight.device, expect_source=digest, sym=sym)
        except PackFormatError:
            pass                                # stale or foreign: re-pack below
    packed = pack_w4a16_sym(weight) if sym else pack_w4a16(weight)
    save_w4(path, packed, digest)
    return packed


def cached_fp8(weight: torch.Tensor, path: str) -> tuple[torch.Tensor, torch.Tensor]:
    """As ``cached_w4`` for the FP8 target head (``pack_fp8_block``)."""
    from .fp8_target_lmhead import pack_fp8_block
    digest = weight_digest(weight)
    if os.path.exists(path):
        try:
            return load_fp8(path, weight.device, expect_source=digest)
        except PackFormatError:
            pass
    wq, ws = pack_fp8_block(weight)
    save_fp8(path, wq, ws, digest)
    return wq, ws

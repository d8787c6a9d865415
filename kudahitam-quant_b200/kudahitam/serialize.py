"""On-disk / wire format of a packed KV cache.

The reference keeps its compressed cache only as an in-memory dict and
accepts but ignores an ``offload`` flag (KudaHitamQuant_full.py:301,358-370).
This format stores the packed cache with everything needed to decode or score
it later:

    bytes 0..3   b"KHPK"
    bytes 4..7   format version (uint32 little endian) = 1
    bytes 8..11  header length H (uint32 little endian)
    bytes 12..   H bytes of UTF-8 JSON:
                   shape, bits, residual, head_dim,
                   d         : +-1 diagonal as a string of '+'/'-'
                   centroids : float32 bit patterns (hex), exact
                   arrays    : [{name, dtype, shape, offset, nbytes}]
    then the arrays (code, norms, res, r_norms), each at a 16-byte aligned
    offset from the start of the file, little endian.

Everything is little endian; the code / residual planes keep the engine's
uint32 layout (include/kudahitam.h), so a file written on one machine reads
on any other.
"""
from __future__ import annotations

import io
import json
import struct
from typing import BinaryIO, Optional, Union

import numpy as np
import torch

from .ops import PackedKV

MAGIC = b"KHPK"
VERSION = 1
_ALIGN = 16

_NP = {torch.int32: "<i4", torch.float32: "<f4"}
_TORCH = {"<i4": torch.int32, "<f4": torch.float32}


def _aligned(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def _encode_d(d) -> str:
    d = torch.as_tensor(d).float().flatten()
    if not torch.all((d == 1) | (d == -1)):
        raise ValueError("d must hold +1 / -1 only")
    return "".join("+" if v > 0 else "-" for v in d.tolist())


def _decode_d(s: str) -> torch.Tensor:
    return torch.tensor([1.0 if ch == "+" else -1.0 for ch in s], dtype=torch.float32)


def dump(p: PackedKV, d, centroids, f: BinaryIO) -> int:
    """Write ``p`` (any device) with its quantiser parameters; returns bytes written."""
    c = torch.as_tensor(centroids).detach().float().cpu().contiguous()
    arrays = [("code", p.code), ("norms", p.norms)]
    if p.res is not None:
        arrays += [("res", p.res), ("r_norms", p.rnorms)]
    blobs = [(n, t.detach().cpu().contiguous()) for n, t in arrays]
    meta = {
        "shape": list(p.shape), "bits": p.bits, "residual": p.residual,
        "head_dim": p.head_dim, "d": _encode_d(d),
        "centroids": [f"{v:08x}" for v in c.numpy().view(np.uint32).tolist()],
        "arrays": [],
    }
    # two passes: header length first, then offsets (header size is stable
    # because offsets are written as fixed-width decimal strings)
    for name, t in blobs:
        meta["arrays"].append({"name": name, "dtype": _NP[t.dtype], "shape": list(t.shape),
                               "offset": "0" * 16, "nbytes": t.numel() * t.element_size()})
    hdr_len = len(json.dumps(meta).encode())
    off = _aligned(12 + hdr_len)
    for a in meta["arrays"]:
        a["offset"] = f"{off:016d}"
        off = _aligned(off + a["nbytes"])
    hdr = json.dumps(meta).encode()
    assert len(hdr) == hdr_len
    f.write(MAGIC + struct.pack("<II", VERSION, hdr_len) + hdr)
    pos = 12 + hdr_len
    for (name, t), a in zip(blobs, meta["arrays"]):
        o = int(a["offset"])
        f.write(b"\0" * (o - pos))
        raw = t.numpy().astype(a["dtype"], copy=False).tobytes()
        f.write(raw)
        pos = o + len(raw)
    return pos


def load(f: BinaryIO, device: Union[str, torch.device, None] = None
         ) -> tuple[PackedKV, torch.Tensor, torch.Tensor]:
    """Read a packed cache.  Returns (PackedKV on ``device``, d, centroids)."""
    head = f.read(12)
    if len(head) != 12 or head[:4] != MAGIC:
        raise ValueError("not a KHPK packed-cache file")
    version, hdr_len = struct.unpack("<II", head[4:])
    if version != VERSION:
        raise ValueError(f"unsupported KHPK version {version}")
    meta = json.loads(f.read(hdr_len).decode())
    pos = 12 + hdr_len
    out = {}
    for a in meta["arrays"]:
        o = int(a["offset"])
        if o < pos:
            raise ValueError("corrupt KHPK file: overlapping arrays")
        f.read(o - pos)
        raw = f.read(a["nbytes"])
        if len(raw) != a["nbytes"]:
            raise ValueError("truncated KHPK file")
        arr = np.frombuffer(raw, dtype=a["dtype"]).reshape(a["shape"])
        out[a["name"]] = torch.from_numpy(arr.copy()).to(_TORCH[a["dtype"]])
        pos = o + a["nbytes"]
    dev = torch.device(device) if device is not None else torch.device("cpu")
    mv = lambda t: None if t is None else t.to(dev)  # noqa: E731
    p = PackedKV(tuple(meta["shape"]), int(meta["bits"]), mv(out["code"]), mv(out["norms"]),
                 mv(out.get("res")), mv(out.get("r_norms")))
    d = _decode_d(meta["d"])
    c = torch.from_numpy(np.array([int(h, 16) for h in meta["centroids"]],
                                  dtype=np.uint32).view(np.float32).copy())
    return p, d, c


def save(path: str, p: PackedKV, d, centroids) -> int:
    with open(path, "wb") as f:
        return dump(p, d, centroids, f)


def read(path: str, device=None):
    with open(path, "rb") as f:
        return load(f, device)


def to_bytes(p: PackedKV, d, centroids) -> bytes:
    b = io.BytesIO()
    dump(p, d, centroids, b)
    return b.getvalue()


def from_bytes(data: bytes, device=None):
    return load(io.BytesIO(data), device)

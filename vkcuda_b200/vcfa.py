"""The flash-attention demo's tensor dump format ("VCFA").

Layout (examples/flash_attn.vc:240-267 in junka/vkcuda): the 4-byte magic
``VCFA``, four little-endian float32 values {NHEAD, SEQ, HDIM, causal}, then
five float32 blobs in row-major [NHEAD][SEQ][HDIM] order: Q, K, V, the
kernel's O and the host reference's O. The reference's
examples/compare_flash_attn.py reads exactly this, so a dump written here can
be handed to that script unchanged.
"""
from __future__ import annotations

import struct
from typing import Dict, Tuple

import numpy as np

MAGIC = b"VCFA"
BLOBS = ("q", "k", "v", "o_kernel", "o_hostref")


def write(path: str, nhead: int, seq: int, hdim: int, causal: int, q, k, v, o_kernel,
          o_hostref) -> None:
    elems = nhead * seq * hdim
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<4f", float(nhead), float(seq), float(hdim), float(causal)))
        for blob in (q, k, v, o_kernel, o_hostref):
            arr = np.ascontiguousarray(blob, dtype="<f4").reshape(-1)
            if arr.size != elems:
                raise ValueError(f"blob has {arr.size} values, expected {elems}")
            f.write(arr.tobytes())


def read(path: str) -> Tuple[Dict[str, int], Dict[str, np.ndarray]]:
    raw = open(path, "rb").read()
    if raw[:4] != MAGIC:
        raise ValueError(f"{path}: bad magic {raw[:4]!r}")
    nhead, seq, hdim, causal = (int(x) for x in struct.unpack("<4f", raw[4:20]))
    body = np.frombuffer(raw[20:], "<f4")
    elems = nhead * seq * hdim
    if body.size != len(BLOBS) * elems:
        raise ValueError(f"{path}: expected {len(BLOBS)} blobs of {elems} floats")
    blobs = {name: body[i * elems:(i + 1) * elems].copy() for i, name in enumerate(BLOBS)}
    return {"nhead": nhead, "seq": seq, "hdim": hdim, "causal": causal}, blobs

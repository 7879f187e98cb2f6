"""FSOW tensor-bundle files (test infrastructure).

Format (reference src/fsow.h:28-67, pytools/fsow.py:1-44): b"FSOW0001", u32 count, then per tensor
u16 name length, utf-8 name, u8 ndim, ndim × i64 shape, u8 dtype (0 f32, 1 i32, 2 u8), raw little-endian
data.  Weights keep PyTorch names and layouts (OIHW).
"""
from __future__ import annotations

import os
import struct

import numpy as np

MAGIC = b"FSOW0001"
_CODE = {np.dtype(np.float32): 0, np.dtype(np.int32): 1, np.dtype(np.uint8): 2}
_DTYPE = {0: np.float32, 1: np.int32, 2: np.uint8}


def save(path: str, tensors: dict) -> None:
    """Write atomically (temp file + rename), like fsow_save (src/fsow.h:53-67)."""
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", len(tensors)))
        for name, arr in sorted(tensors.items()):
            a = np.ascontiguousarray(arr)
            if a.dtype not in _CODE:
                a = a.astype(np.float32)
            nb = name.encode()
            f.write(struct.pack("<H", len(nb)))
            f.write(nb)
            f.write(struct.pack("<B", a.ndim))
            f.write(struct.pack(f"<{a.ndim}q", *a.shape))
            f.write(struct.pack("<B", _CODE[a.dtype]))
            f.write(a.astype(a.dtype.newbyteorder("<"), copy=False).tobytes())
    os.replace(tmp, path)


def load(path: str) -> dict:
    out = {}
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: not an FSOW file")
        (n,) = struct.unpack("<I", f.read(4))
        for _ in range(n):
            (ln,) = struct.unpack("<H", f.read(2))
            name = f.read(ln).decode()
            (nd,) = struct.unpack("<B", f.read(1))
            shape = struct.unpack(f"<{nd}q", f.read(8 * nd)) if nd else ()
            (code,) = struct.unpack("<B", f.read(1))
            dt = np.dtype(_DTYPE[code])
            cnt = int(np.prod(shape)) if nd else 1
            buf = f.read(cnt * dt.itemsize)
            if len(buf) != cnt * dt.itemsize:
                raise ValueError(f"{path}: truncated at {name}")
            out[name] = np.frombuffer(buf, dt.newbyteorder("<")).astype(dt).reshape(shape)
    return out

"""FSOW tensor-bundle files (test infrastructure).

The reference's exchange format for weights and tensors (reference src/fsow.h:28-67): the 8-byte tag
b"FSOW0001", a little-endian u32 record count, then one record per tensor —
    u16 name length | utf-8 name | u8 rank | rank x i64 extents | u8 element code | raw little-endian data
with element codes 0 = float32, 1 = int32, 2 = uint8.  Weights keep PyTorch names and layouts (OIHW).

This module parses a whole file from one buffer with a cursor, and builds each record in memory before
the file is written (atomically: temp file, then rename), so a half-written bundle is never seen.
"""
from __future__ import annotations

import os
import struct

import numpy as np

TAG = b"FSOW0001"
CODES = (np.dtype("<f4"), np.dtype("<i4"), np.dtype("u1"))  # element code = index


def _code(dtype) -> int:
    for i, d in enumerate(CODES):
        if np.dtype(dtype).newbyteorder("<") == d:
            return i
    return -1


def encode(name: str, arr) -> bytes:
    """One record.  Element types other than the three the format knows are stored as float32."""
    a = np.asarray(arr)
    if _code(a.dtype) < 0:
        a = a.astype(np.float32)
    code = _code(a.dtype)
    raw = np.ascontiguousarray(a, dtype=CODES[code])
    key = name.encode("utf-8")
    head = struct.pack(f"<H{len(key)}sB{raw.ndim}qB", len(key), key, raw.ndim, *raw.shape, code)
    return head + raw.tobytes()


def save(path: str, tensors: dict) -> None:
    body = b"".join(encode(k, tensors[k]) for k in sorted(tensors))
    tmp = f"{path}.partial"
    with open(tmp, "wb") as f:
        f.write(TAG + struct.pack("<I", len(tensors)) + body)
    os.replace(tmp, path)


class _Cursor:
    def __init__(self, buf: bytes, where: str):
        self.buf, self.at, self.where = memoryview(buf), 0, where

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        if self.at + size > len(self.buf):
            raise ValueError(f"{self.where}: truncated at byte {self.at}")
        vals = struct.unpack_from(fmt, self.buf, self.at)
        self.at += size
        return vals

    def raw(self, n: int) -> memoryview:
        if self.at + n > len(self.buf):
            raise ValueError(f"{self.where}: truncated at byte {self.at}")
        out = self.buf[self.at:self.at + n]
        self.at += n
        return out


def load(path: str) -> dict:
    with open(path, "rb") as f:
        data = f.read()
    if data[:8] != TAG:
        raise ValueError(f"{path}: not an FSOW file")
    cur = _Cursor(data, path)
    cur.at = 8
    (count,) = cur.take("<I")
    tensors = {}
    for _ in range(count):
        (klen,) = cur.take("<H")
        name = bytes(cur.raw(klen)).decode("utf-8")
        (rank,) = cur.take("<B")
        shape = cur.take(f"<{rank}q")
        (code,) = cur.take("<B")
        if code >= len(CODES):
            raise ValueError(f"{path}: {name} has unknown element code {code}")
        dt = CODES[code]
        n = int(np.prod(shape, dtype=np.int64))
        tensors[name] = np.frombuffer(cur.raw(n * dt.itemsize), dt).astype(dt.newbyteorder("=")).reshape(shape)
    return tensors

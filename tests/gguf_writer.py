"""Minimal GGUF v3 writer for tests (header, metadata, tensor infos, 32-byte aligned data),
the same file structure the reference's test fixture builder writes
(tests/test_utils.h:16-97 of the reference)."""
from __future__ import annotations

import struct

import numpy as np


def _s(b: bytearray, text: str):
    raw = text.encode()
    b += struct.pack("<Q", len(raw)) + raw


def write_gguf(path: str, tensors: list[tuple[str, list[int], int, np.ndarray]], meta_u32=None) -> list[int]:
    """tensors: (name, dims with ne0 first, ggml type, packed bytes).  Returns data offsets."""
    meta_u32 = meta_u32 or {}
    b = bytearray()
    b += struct.pack("<IIQQ", 0x46475547, 3, len(tensors), len(meta_u32))
    for k, v in meta_u32.items():
        _s(b, k)
        b += struct.pack("<II", 4, v)
    offsets, off = [], 0
    for name, dims, t, data in tensors:
        _s(b, name)
        b += struct.pack("<I", len(dims))
        for d in dims:
            b += struct.pack("<Q", d)
        b += struct.pack("<IQ", t, off)
        offsets.append(off)
        off += (len(data.tobytes()) + 31) // 32 * 32
    b += bytes((32 - len(b) % 32) % 32)
    for (_, _, _, data), o in zip(tensors, offsets):
        raw = data.tobytes()
        b += raw + bytes((32 - len(raw) % 32) % 32)
    with open(path, "wb") as f:
        f.write(bytes(b))
    return offsets

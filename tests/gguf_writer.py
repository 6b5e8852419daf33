"""Minimal GGUF v3 writer for test models (test infrastructure).

Layout per the format the reference reads (src/gguf.rs:321-400): magic, version
3, tensor count, KV count, KV pairs, tensor infos (name, dims, type, offset),
then tensor data aligned to general.alignment (32).
"""
from __future__ import annotations

import struct

import numpy as np

T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64 = 4, 5, 6, 7, 8, 9, 10


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(v) -> tuple[int, bytes]:
    if isinstance(v, bool):
        return T_BOOL, struct.pack("<B", int(v))
    if isinstance(v, int):
        return T_U32, struct.pack("<I", v)
    if isinstance(v, float):
        return T_F32, struct.pack("<f", v)
    if isinstance(v, str):
        return T_STR, _str(v)
    if isinstance(v, (list, tuple)):
        t, _ = _value(v[0]) if v else (T_I32, b"")
        body = b"".join(_value(x)[1] for x in v)
        return T_ARR, struct.pack("<IQ", t, len(v)) + body
    raise TypeError(type(v))


def write_gguf(path: str, meta: dict, tensors: list[tuple[str, int, tuple, np.ndarray]], alignment: int = 32):
    """tensors: (name, ggml type id, shape ne0-first, raw bytes as uint8 array)."""
    out = bytearray()
    out += b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(meta))
    for k, v in meta.items():
        t, b = _value(v)
        out += _str(k) + struct.pack("<I", t) + b
    offsets = []
    off = 0
    for name, dtype, shape, data in tensors:
        offsets.append(off)
        off += data.nbytes
        off = (off + alignment - 1) // alignment * alignment
    for (name, dtype, shape, data), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        out += struct.pack("<IQ", dtype, o)
    pad = (-len(out)) % alignment
    out += b"\0" * pad
    base = len(out)
    for (name, dtype, shape, data), o in zip(tensors, offsets):
        cur = len(out) - base
        out += b"\0" * (o - cur)
        out += np.ascontiguousarray(data).view(np.uint8).tobytes()
    with open(path, "wb") as f:
        f.write(bytes(out))

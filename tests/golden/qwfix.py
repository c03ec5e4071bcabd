"""The reference's QWFIX001 fixture container (src/cli/fixture.zig:1-66).

Layout, little-endian: the 8-byte magic "QWFIX001", a u32 rank (at most 4),
four u32 dimensions (unused ones are 1), then the row-major f32 payload.
Everything is f32, token ids included (ids below 2^24 round trip exactly), so
one reader serves logits, ids and cache bytes alike.
"""

from __future__ import annotations

import struct

import numpy as np

MAGIC = b"QWFIX001"
HEADER_BYTES = 28


def encode(dims, values) -> bytes:
    """fixture.encode (fixture.zig:39-63): refuses rank > 4 and a payload whose
    length is not the product of the dimensions."""
    dims = [int(d) for d in dims]
    if len(dims) > 4:
        raise ValueError("RankTooLarge")
    v = np.ascontiguousarray(values, dtype="<f4").ravel()
    if int(np.prod(dims, dtype=np.int64)) != v.size:
        raise ValueError("TooManyElements")
    padded = dims + [1] * (4 - len(dims))
    return MAGIC + struct.pack("<5I", len(dims), *padded) + v.tobytes()


def decode(data: bytes) -> np.ndarray:
    """The reader side (tests/reference_check.zig reads the same layout): the
    payload as an f32 array of the stored shape."""
    if len(data) < HEADER_BYTES or data[:8] != MAGIC:
        raise ValueError("not a QWFIX001 container")
    rank, *dims = struct.unpack("<5I", data[8:HEADER_BYTES])
    if rank > 4:
        raise ValueError("RankTooLarge")
    shape = dims[:rank]
    n = int(np.prod(shape, dtype=np.int64)) if rank else 1
    if len(data) != HEADER_BYTES + 4 * n:
        raise ValueError("payload length does not match the dimensions")
    return np.frombuffer(data, dtype="<f4", offset=HEADER_BYTES, count=n).reshape(shape)


def write(path: str, dims, values) -> None:
    with open(path, "wb") as f:
        f.write(encode(dims, values))


def read(path: str) -> np.ndarray:
    with open(path, "rb") as f:
        return decode(f.read())

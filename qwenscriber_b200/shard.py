"""Writes `.qw` shards (the reference's QWSHARD1 container, src/core/container.zig).

A shard is a 32-byte header, an index of 40-byte entries sorted by
(layer, kind), and a payload that starts on a 256-byte boundary with every
tensor on a 16-byte boundary (container.zig:33-48, 54-62). Quantized tensors
keep the reference's two planes: f16 scales, padding to 16 bytes, codes
(src/core/quant.zig:144-176). The header carries the low 32 bits of the
FNV-1a 64 hash of the payload (container.zig:283-291).

`qwc_model_add_shard` reads these bytes; `write_model_shards` splits a
synthetic model the way the reference's converter splits a real one: the
tensors outside any layer (layer 0) go with the first layers, and each shard
holds a contiguous range of layers.
"""

from __future__ import annotations

import struct
from typing import Iterable

import numpy as np

from . import quant

MAGIC = b"QWSHARD1"
FORMAT_VERSION = 1
HEADER_BYTES = 32
ENTRY_BYTES = 40
PAYLOAD_ALIGNMENT = 256
TENSOR_ALIGNMENT = 16

FNV_OFFSET = 0xCBF29CE484222325
FNV_PRIME = 0x100000001B3


def fnv1a64(data: bytes) -> int:
    """The published 64-bit FNV-1a hash (offset basis 0xcbf29ce484222325,
    prime 0x100000001b3)."""
    h = FNV_OFFSET
    for b in data:
        h = ((h ^ b) * FNV_PRIME) & 0xFFFFFFFFFFFFFFFF
    return h


def payload_checksum(payload: bytes) -> int:
    """Low 32 bits of FNV-1a 64 of the payload, computed by the library's
    qwc_shard_checksum (host code; no GPU needed)."""
    from . import runtime

    buf = np.frombuffer(payload, np.uint8)
    return int(runtime.lib().qwc_shard_checksum(buf.ctypes.data if buf.size else None, buf.size))


def _align(v: int, a: int) -> int:
    return (v + a - 1) // a * a


def build(tensors: Iterable[tuple[int, int, int, tuple[int, ...], bytes]]) -> bytes:
    """One shard from (kind, layer, format, dims, payload) tuples, in any order.
    `payload` must already be the tensor's exact container bytes."""
    items = sorted(tensors, key=lambda t: (t[1] << 16) | t[0])
    index = bytearray()
    payload = bytearray()
    for kind, layer, fmt, dims, data in items:
        if not 1 <= len(dims) <= 4:
            raise ValueError("rank must be 1..4")
        offset = _align(len(payload), TENSOR_ALIGNMENT)
        payload.extend(b"\0" * (offset - len(payload)))
        payload.extend(data)
        padded = list(dims) + [1] * (4 - len(dims))
        index.extend(struct.pack("<HHBBH4IQQ", kind, layer, fmt, len(dims), 0, *padded, offset, len(data)))
    payload_offset = _align(HEADER_BYTES + len(index), PAYLOAD_ALIGNMENT)
    header = struct.pack("<8sIIIIII", MAGIC, FORMAT_VERSION, len(index), payload_offset, len(payload), len(items),
                         payload_checksum(bytes(payload)))
    out = bytearray(header)
    out.extend(index)
    out.extend(b"\0" * (payload_offset - len(out)))
    out.extend(payload)
    return bytes(out)


def tensor_entry(t) -> tuple[int, int, int, tuple[int, ...], bytes]:
    """A synthetic-model tensor (kind, layer, fmt, rows, cols, payload) as a
    shard item: f32 vectors are rank 1, matrices rank 2, the audio tower's f16
    convolution weights rank 4 [out][in][3][3] (layout.zig:150-175)."""
    if t.fmt == quant.F16 and t.kind in (1, 3, 5):
        dims = (t.rows, t.cols // 9, 3, 3)
    else:
        dims = (t.cols,) if t.fmt == quant.F32 and t.rows == 1 else (t.rows, t.cols)
    return (t.kind, t.layer, t.fmt, dims, np.ascontiguousarray(t.payload).tobytes())


def write_model_shards(model, shards: int = 2) -> list[bytes]:
    """The model's tensors as `shards` shards of contiguous decoder layer
    ranges; the layer-0 tensors and any audio-tower layers go to the first."""
    layers = model.config.text_layers
    bounds = [round(i * layers / shards) for i in range(shards + 1)]
    out = []
    for s in range(shards):
        lo, hi = bounds[s], bounds[s + 1]
        items = [tensor_entry(t) for t in model.tensors
                 if ((t.layer == 0 or t.layer >= 1024) and s == 0) or (lo < t.layer <= hi < 1024)]
        out.append(build(items))
    return out

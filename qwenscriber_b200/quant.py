"""Host-side q4/q5/q8 group quantizer and tensor payload layout.

Numpy restatement of the reference converter's arithmetic
(src/core/quant.zig:144-288): 64-value groups, an f16 scale of
`max_abs / bias` rounded to nearest even, codes quantized against the
*stored* scale with round-half-away-from-zero and clamping, q4 nibbles
little-endian within a byte, q5 as q4 nibbles followed by a plane of fifth
bits (quant.zig:253-269). All arithmetic stays in float32, as the Zig code
does, so the bytes match the reference bit for bit.
"""

from __future__ import annotations

import numpy as np

GROUP = 64
Q4, Q5, Q8 = 16, 17, 18
F32 = 0
F16 = 1
DATA_BYTES = {Q4: 32, Q5: 40, Q8: 64}
BIAS = {Q4: 8, Q5: 16, Q8: 128}
ALIGN = 16


def align_up(n: int, a: int = ALIGN) -> int:
    return (n + a - 1) // a * a


def plane_layout(fmt: int, rows: int, cols: int) -> tuple[int, int, int, int]:
    """(scales_offset, scales_len, data_offset, data_len) at a 16-byte-aligned base (quant.zig:144-176)."""
    if cols % GROUP:
        raise ValueError("cols must be a whole number of 64-value groups (quant.zig:77-81)")
    groups = rows * (cols // GROUP)
    scales_len = groups * 2
    data_off = align_up(scales_len)
    return 0, scales_len, data_off, groups * DATA_BYTES[fmt]


def quantize(fmt: int, values: np.ndarray, block_rows: int = 2048) -> tuple[np.ndarray, np.ndarray]:
    """quantizeRow over every row: returns (scales u16[rows, groups], codes u8[rows, groups*bytes]).
    Rows are independent, so they are taken `block_rows` at a time (bounded temporaries)."""
    if fmt not in (Q4, Q5, Q8):
        raise ValueError("q4, q5 and q8 are the formats this backend runs")
    v = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = v.shape
    if rows > block_rows:
        parts = [_quantize_block(fmt, v[r:r + block_rows]) for r in range(0, rows, block_rows)]
        return np.concatenate([p[0] for p in parts]), np.concatenate([p[1] for p in parts])
    return _quantize_block(fmt, v)


def _quantize_block(fmt: int, v: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    rows, cols = v.shape
    g = v.reshape(rows, cols // GROUP, GROUP)
    max_abs = np.abs(g).max(axis=2)
    bias = np.float32(BIAS[fmt])
    scale16 = (max_abs / bias).astype(np.float16)
    stored = scale16.astype(np.float32)[:, :, None]
    with np.errstate(divide="ignore", invalid="ignore"):
        scaled = (g / stored).astype(np.float32)
    half = np.float32(0.5)
    rounded = np.where(scaled >= 0, np.floor(scaled + half), np.ceil(scaled - half)).astype(np.float32)
    codes = np.clip(rounded, -BIAS[fmt], BIAS[fmt] - 1)
    codes = np.where(stored == 0, 0, codes).astype(np.int32) + BIAS[fmt]
    codes = codes.astype(np.uint8).reshape(rows, cols)
    if fmt == Q4:
        codes = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    elif fmt == Q5:
        codes = pack_q5(codes)
    return scale16.view(np.uint16), codes


def pack_q5(u: np.ndarray) -> np.ndarray:
    """q5 codes u8[rows, cols] (0..31) -> the group layout of quant.zig:253-269:
    per 64-value group, 32 bytes of low nibbles (weight 2i low, 2i + 1 high in
    byte i), then 8 bytes of fifth bits (weight i at bit i % 8 of byte i / 8)."""
    rows, cols = u.shape
    g = u.reshape(rows, cols // GROUP, GROUP)
    nib = g & 0x0F
    low = (nib[:, :, 0::2] | (nib[:, :, 1::2] << 4)).astype(np.uint8)
    bits = ((g >> 4) & 1).astype(np.uint8).reshape(rows, cols // GROUP, 8, 8)
    plane = np.packbits(bits, axis=-1, bitorder="little").reshape(rows, cols // GROUP, 8)
    return np.concatenate([low, plane], axis=2).reshape(rows, cols // GROUP * 40)


def unpack_q5(codes: np.ndarray, cols: int) -> np.ndarray:
    """The inverse of pack_q5: unsigned codes int32[rows, cols]."""
    rows = codes.shape[0]
    g = np.asarray(codes, dtype=np.uint8).reshape(rows, cols // GROUP, 40)
    u = np.empty((rows, cols // GROUP, GROUP), np.int32)
    u[:, :, 0::2] = g[:, :, :32] & 0x0F
    u[:, :, 1::2] = g[:, :, :32] >> 4
    bits = np.unpackbits(g[:, :, 32:], axis=-1, bitorder="little").astype(np.int32)
    return (u | (bits << 4)).reshape(rows, cols)


def dequantize(fmt: int, scales: np.ndarray, codes: np.ndarray, cols: int) -> np.ndarray:
    """dequantizeRow over every row (quant.zig:315-364)."""
    rows = scales.shape[0]
    s = np.asarray(scales).view(np.float16).astype(np.float32).reshape(rows, cols // GROUP, 1)
    c = np.asarray(codes, dtype=np.uint8).reshape(rows, -1)
    if fmt == Q4:
        u = np.empty((rows, cols), np.int32)
        u[:, 0::2] = c & 0x0F
        u[:, 1::2] = c >> 4
    elif fmt == Q5:
        u = unpack_q5(c, cols)
    else:
        u = c.astype(np.int32)
    vals = (u - BIAS[fmt]).astype(np.float32).reshape(rows, cols // GROUP, GROUP)
    return (vals * s).reshape(rows, cols)


def payload(fmt: int, scales: np.ndarray, codes: np.ndarray) -> np.ndarray:
    """One tensor's container payload: scale plane, padding to 16 bytes, code plane."""
    sb = np.ascontiguousarray(scales).view(np.uint8).reshape(-1)
    cb = np.ascontiguousarray(codes).reshape(-1)
    out = np.zeros(align_up(sb.size) + cb.size, np.uint8)
    out[: sb.size] = sb
    out[align_up(sb.size):] = cb
    return out


def split_payload(fmt: int, rows: int, cols: int, data: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of `payload`: (scales u16[rows, groups], codes u8[rows, groups*bytes])."""
    _, slen, doff, dlen = plane_layout(fmt, rows, cols)
    scales = data[:slen].view(np.uint16).reshape(rows, cols // GROUP)
    codes = data[doff:doff + dlen].reshape(rows, -1)
    return scales, codes

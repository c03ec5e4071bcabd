"""The `.qw` shard container (QWSHARD1) through the C ABI, without a GPU.

qwc_shard_validate is container.File.parse followed by verifyChecksum
(src/core/container.zig:176-291). The cases restate the reference's own
container tests (container.zig:433-522): a minimal q4 shard, its corrupted
checksum, corrupt header fields, truncation, and a recorded length that
disagrees with the shape. The remaining cases cover the index rules
(ordering, ranges, alignment), and the writer round-trips synthetic models.
"""

import struct

import numpy as np
import pytest

from qwenscriber_b200 import quant, shard, synthetic
from qwenscriber_b200 import runtime as rt

from .parity import small_config

AUDIO_CONV1_WEIGHT = 1  # container.TensorKind.audio_conv1_weight
CODE = {name: code for code, name in rt.STATUS.items()}


def one_tensor_shard(payload: bytes, fmt: int, rows: int, cols: int) -> bytearray:
    """container.zig testShard: header, one index entry, padding, payload."""
    return bytearray(shard.build([(AUDIO_CONV1_WEIGHT, 0, fmt, (rows, cols), payload)]))


def q4_64_payload() -> bytes:
    # 64 x 64 q4: 64 groups, 128 bytes of scales (already 16-aligned), 2048 of codes.
    p = bytearray(128 + 64 * 32)
    p[128] = 0x0F  # data plane
    p[0] = 0x3C    # scale plane
    return bytes(p)


def validate(b) -> tuple[int, int]:
    return rt.shard_validate(bytes(b))


def test_fnv1a_published_vectors():
    assert shard.fnv1a64(b"") == 0xCBF29CE484222325
    assert shard.fnv1a64(b"a") == 0xAF63DC4C8601EC8C
    assert shard.fnv1a64(b"foobar") == 0x85944171F73967E8
    assert shard.payload_checksum(b"foobar") == 0xF73967E8


def test_minimal_shard_parses_and_checksum_is_verified():
    good = one_tensor_shard(q4_64_payload(), quant.Q4, 64, 64)
    assert struct.unpack_from("<8sIIIIII", good)[0] == b"QWSHARD1"
    assert validate(good) == (CODE["ok"], 1)
    bad = bytearray(good)
    bad[-1] ^= 0xFF
    assert validate(bad)[0] == CODE["checksum_mismatch"]


@pytest.mark.parametrize("offset,value,expected", [
    (0, ord("X"), "bad_magic"),
    (8, 99, "bad_version"),
    (24, 3, "truncated"),   # tensor_count no longer matches index_len_bytes
    (12, 0, "truncated"),   # index_len_bytes
])
def test_corrupt_headers_are_rejected(offset, value, expected):
    b = one_tensor_shard(bytes(4224), quant.Q8, 64, 64)
    assert validate(b)[0] == CODE["ok"]
    struct.pack_into("<I", b, offset, value)
    assert validate(b)[0] == CODE[expected]


def test_truncated_buffers_are_rejected():
    good = one_tensor_shard(bytes(4224), quant.Q8, 64, 64)
    assert validate(good[:16])[0] == CODE["truncated"]
    assert validate(good[:-1])[0] == CODE["truncated"]


def test_recorded_length_must_match_the_shape():
    b = one_tensor_shard(bytes(4224), quant.Q8, 64, 64)
    struct.pack_into("<Q", b, shard.HEADER_BYTES + 32, 8)  # the entry's len_bytes
    assert validate(b)[0] == CODE["shape_mismatch"]


def test_index_rules():
    vec = np.ones(64, np.float32).tobytes()
    two = [(40, 1, quant.F32, (64,), vec), (39, 1, quant.F32, (64,), vec)]
    b = bytearray(shard.build(two))
    assert validate(b) == (CODE["ok"], 2)
    # Swap the two entries: the keys are no longer ascending.
    e0 = bytes(b[32:72])
    b[32:72] = b[72:112]
    b[72:112] = e0
    assert validate(b)[0] == CODE["invalid_argument"]
    # A tensor offset that is not 16-byte aligned (the middle of three, moved
    # 8 bytes into the gap after it, so its range stays inside the payload).
    three = two + [(41, 1, quant.F32, (64,), vec)]
    b = bytearray(shard.build(three))
    struct.pack_into("<Q", b, 72 + 24, 264)
    assert validate(b)[0] == CODE["invalid_argument"]
    # Overlapping ranges.
    b = bytearray(shard.build(three))
    struct.pack_into("<Q", b, 72 + 24, 128)
    assert validate(b)[0] == CODE["invalid_argument"]
    # Quantized formats need a matrix whose rows hold whole groups.
    assert validate(shard.build([(33, 1, quant.Q8, (2, 32), bytes(16 + 64))]))[0] == CODE["shape_mismatch"]
    # An unknown format.
    assert validate(shard.build([(33, 1, 9, (64,), bytes(64))]))[0] == CODE["unsupported_model"]


def test_misaligned_buffer_is_rejected():
    good = np.frombuffer(one_tensor_shard(bytes(4224), quant.Q8, 64, 64), np.uint8)
    store = np.zeros(good.size + 32, np.uint8)
    start = (-store.ctypes.data) % 16 + 1  # deliberately one byte past a 16-byte boundary
    store[start:start + good.size] = good
    view = store[start:start + good.size]
    status = rt.lib().qwc_shard_validate(view.ctypes.data, view.size, None)
    assert status == CODE["invalid_argument"]


@pytest.mark.parametrize("fmt", [quant.Q8, quant.Q4])
def test_model_shards_round_trip(fmt):
    model = synthetic.make_model(small_config(fmt, layers=3), fmt, seed=4)
    parts = shard.write_model_shards(model, shards=2)
    counts = [validate(p) for p in parts]
    assert all(s == CODE["ok"] for s, _ in counts)
    assert sum(n for _, n in counts) == len(model.tensors)
    # Layer-0 tensors travel with the first layers; layers are contiguous per shard.
    first = parts[0]
    count = struct.unpack_from("<I", first, 24)[0]
    layers = [struct.unpack_from("<HH", first, shard.HEADER_BYTES + i * shard.ENTRY_BYTES)[1] for i in range(count)]
    assert layers == sorted(layers) and layers[0] == 0

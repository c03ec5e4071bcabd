"""Pins the CPU oracle to the reference's own known-answer tests.

Every expected value here is stated by a test in the reference source
(file:line given per test); the oracle restates the Zig arithmetic, so these
are the checks that it restates it correctly.
"""

import math

import numpy as np
import pytest

import oracle as O


def test_quant_hash_golden(oracle_lib):
    # src/core/selftest.zig:288-298: FNV-1a over q4/q5/q8 quantizeRow of cos(i*0.19)*1.75.
    assert O.quant_hash() == 0xF247917B05691FD1


def test_exact_codes_when_step_is_one(oracle_lib):
    # src/core/quant.zig:527-542
    values = np.zeros((1, 64), np.float32)
    values[0, 0], values[0, 1] = 7.0, -8.0
    scales, data = O.quantize_rows(O.Q4, values)
    assert int(scales[0, 0]) | (int(scales[0, 1]) << 8) == 0x3C00
    decoded = O.dequantize_rows(O.Q4, scales, data, 64)[0]
    assert decoded[0] == 7.0 and decoded[1] == -8.0
    assert np.all(decoded[2:] == 0.0)


def test_zero_group(oracle_lib):
    # src/core/quant.zig:544-554
    values = np.zeros((1, 64), np.float32)
    scales, data = O.quantize_rows(O.Q4, values)
    assert O.from_f16(int(scales[0, 0]) | (int(scales[0, 1]) << 8)) == 0.0
    assert np.all(O.dequantize_rows(O.Q4, scales, data, 64) == 0.0)
    assert O.lib().orc_dot_row(O.Q4, O._u8p(scales[0]), O._u8p(data[0]), O._fp(values[0]), 64) == 0.0


def test_q5_packing(oracle_lib):
    # src/core/quant.zig:597-624
    values = np.zeros((1, 64), np.float32)
    values[0, 0], values[0, 1] = 15.0, -16.0
    scales, data = O.quantize_rows(O.Q5, values)
    decoded = O.dequantize_rows(O.Q5, scales, data, 64)[0]
    assert decoded[0] == 15.0 and decoded[1] == -16.0 and np.all(decoded[2:] == 0.0)
    assert data[0, 0] == 0x0F
    assert data[0, 32] & 0x01 and not (data[0, 32] & 0x02)
    assert np.all(data[0, 33:40] == 0xFF)


@pytest.mark.parametrize("fmt,bias", [(O.Q4, 8), (O.Q5, 16), (O.Q8, 128)])
def test_round_trip_within_step(oracle_lib, fmt, bias):
    # src/core/quant.zig:457-498
    i = np.arange(64, dtype=np.float32)
    values = (np.sin(i * np.float32(0.37)) * np.float32(3.0) + i * np.float32(0.01)).astype(np.float32)[None, :]
    scales, data = O.quantize_rows(fmt, values)
    decoded = O.dequantize_rows(fmt, scales, data, 64)[0]
    step = np.abs(values).max() / bias
    bound = step * (1.0 + bias * 0.00048828125) + 1e-6
    diff = np.abs(values[0] - decoded)
    assert np.all(diff <= bound)
    assert math.sqrt(float(np.mean(diff.astype(np.float64) ** 2))) <= step * 0.5


def test_error_shrinks_with_code_width(oracle_lib):
    # src/core/quant.zig:500-525
    i = np.arange(64, dtype=np.float32)
    values = (np.cos(i * np.float32(0.53)) * np.float32(2.5) + np.sin(i * np.float32(0.11))).astype(np.float32)[None]
    errs = []
    for fmt in (O.Q4, O.Q5, O.Q8):
        s, d = O.quantize_rows(fmt, values)
        errs.append(float(np.abs(values - O.dequantize_rows(fmt, s, d, 64)).sum()))
    assert errs[0] > errs[1] > errs[2]


def test_dot_row_matches_dense(oracle_lib):
    # src/core/quant.zig:575-595
    i = np.arange(256, dtype=np.float32)
    values = (np.cos(i * np.float32(0.11)) * np.float32(1.5)).astype(np.float32)[None]
    x = (np.sin(i * np.float32(0.07)) * np.float32(0.5)).astype(np.float32)
    s, d = O.quantize_rows(O.Q4, values)
    dense = O.dequantize_rows(O.Q4, s, d, 256)[0]
    expected = float(np.sum(dense.astype(np.float64) * x))
    actual = O.lib().orc_dot_row(O.Q4, O._u8p(s[0]), O._u8p(d[0]), O._fp(x), 256)
    assert actual == pytest.approx(expected, rel=1e-5)


def test_row_of_ones_is_56(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:932-971: scale 1/8, code 7 (clamped), 64 * 0.875 = 56 exactly.
    ones = np.ones((1, 64), np.float32)
    s, d = O.quantize_rows(O.Q4, ones)
    out = O.linear_quantized(O.Q4, s, d, np.ones(64, np.float32))
    assert out[0, 0] == 56.0


def test_quantized_linear_matches_dequantized(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:878-930
    cols, tokens, rows = 128, 3, 4
    idx = np.arange(rows * cols, dtype=np.float32)
    values = (np.cos(idx * np.float32(0.07)) * np.float32(1.25)).astype(np.float32).reshape(rows, cols)
    xi = np.arange(tokens * cols, dtype=np.float32)
    x = (np.sin(xi * np.float32(0.11)) * np.float32(0.75)).astype(np.float32).reshape(tokens, cols)
    s, d = O.quantize_rows(O.Q4, values)
    actual = O.linear_quantized(O.Q4, s, d, x)
    dense = O.dequantize_rows(O.Q4, s, d, cols)
    for t in range(tokens):
        for r in range(rows):
            expected = O.lib().orc_dot_f32(O._fp(np.ascontiguousarray(dense[r])), O._fp(np.ascontiguousarray(x[t])), cols)
            assert abs(actual[t, r] - expected) <= 1e-5


def _lcg_values(state, n, divisor):
    out = np.zeros(n, np.float32)
    for i in range(n):
        state = (state * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32(((state >> 9) % 2001) - 1000) / np.float32(divisor)
    return state, out


def test_q8_cache_attention_matches_f32(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:769-836: LCG seed 7, 4 heads / 2 kv heads / dim 64 / 5 positions.
    head_dim, kvh, heads, cached = 64, 2, 4, 5
    kvw = kvh * head_dim
    st = 7
    st, keys = _lcg_values(st, cached * kvw, 200.0)
    st, values = _lcg_values(st, cached * kvw, 400.0)
    st, query = _lcg_values(st, heads * head_dim, 500.0)
    ks, kc = O.quantize_rows(O.Q8, keys.reshape(cached, kvw))
    vs, vc = O.quantize_rows(O.Q8, values.reshape(cached, kvw))
    exact = O.decode_attention_f32(query, keys, values, cached, heads, kvh, head_dim)
    quantized = O.decode_attention_q8(query, ks, kc, vs, vc, cached, heads, kvh, head_dim)
    assert np.max(np.abs(exact - quantized)) <= 0.05


def test_rope_norm_and_position_zero(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:1080-1106
    cos, sin = O.rope_tables(2, 1000000.0, 8)
    x = np.tile(np.array([1.0, 2.0, 3.0, 4.0], np.float32), 3)
    out = O.rope(x, [0, 1, 7], 1, 4, cos, sin).reshape(3, 4)
    assert np.allclose(out[0], [1, 2, 3, 4], atol=1e-6)
    assert np.allclose((out.astype(np.float32) ** 2).sum(axis=1), 30.0, atol=1e-4)


def test_inverse_frequency(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:1108-1117
    assert O.lib().orc_inverse_frequency(0, 128, 1e6) == pytest.approx(1.0, abs=1e-6)
    assert O.lib().orc_inverse_frequency(64, 128, 1e6) == pytest.approx(1e-6, abs=1e-12)


def test_decode_attention_reads_cached_positions(oracle_lib):
    # src/core/qwen3_asr/kernels.zig:1119-1138
    q = np.array([1.0, 0.0, 0.0, 1.0], np.float32)
    keys = np.array([1.0, 0.0, 0.0, 1.0], np.float32)
    values = np.array([1.0, 1.0, 3.0, 3.0], np.float32)
    out = O.decode_attention_f32(q, keys, values, 2, 2, 1, 2)
    assert out[0] < 2.0 and out[2] > 2.0
    assert out[0] + out[2] == pytest.approx(4.0, abs=1e-5)
    assert out[1] + out[3] == pytest.approx(4.0, abs=1e-5)


def test_math_values(oracle_lib):
    # src/core/math.zig:174-214
    L = O.lib()
    assert L.orc_silu(0.0) == pytest.approx(0.0, abs=1e-7)
    assert L.orc_silu(1.0) == pytest.approx(0.7310586, abs=1e-6)
    assert L.orc_silu(-1.0) == pytest.approx(-0.26894143, abs=1e-6)
    assert L.orc_silu(30.0) == pytest.approx(30.0, abs=1e-3)
    assert L.orc_silu(-30.0) == pytest.approx(0.0, abs=1e-9)
    sm = O.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert np.allclose(sm, [0.09003057, 0.24472848, 0.66524096], atol=1e-6)
    ext = O.softmax(np.array([1000.0, -1000.0, 0.0], np.float32))
    assert ext[0] == pytest.approx(1.0, abs=1e-6) and ext[1] == 0.0
    r = O.rmsnorm(np.array([3.0, 4.0], np.float32), np.ones(2, np.float32), 2, 0.0)
    assert (r[0] * r[0] + r[1] * r[1]) / 2.0 == pytest.approx(1.0, abs=1e-6)
    z = O.rmsnorm(np.zeros(3, np.float32), np.ones(3, np.float32), 3, 1e-6)
    assert np.all(z == 0.0)


def _mulberry32(seed):
    # tests/gpu/reference.mjs:33-44
    state = seed & 0xFFFFFFFF

    def next_u32():
        nonlocal state
        state = (state + 0x6D2B79F5) & 0xFFFFFFFF
        v = state
        v = ((v ^ (v >> 15)) * (v | 1)) & 0xFFFFFFFF
        v = (v ^ ((v + (((v ^ (v >> 7)) * (v | 61)) & 0xFFFFFFFF)) & 0xFFFFFFFF)) & 0xFFFFFFFF
        return (v ^ (v >> 14)) & 0xFFFFFFFF

    return next_u32


def harness_random_vector(length, seed):
    """tests/gpu/reference.mjs:55-65 (Box-Muller over mulberry32, rounded to f32)."""
    nxt = _mulberry32(seed)
    out = np.zeros(length, np.float32)
    for i in range(length):
        first = 1 - nxt() / 4294967296
        second = nxt() / 4294967296
        out[i] = np.float32(math.sqrt(-2 * math.log(first)) * math.cos(2 * math.pi * second))
    return out


def test_argmax_ties_go_to_lowest_index(oracle_lib):
    # tests/gpu/harness.mjs:281,645-660: maximum planted at 333 and 777 -> 333.
    v = harness_random_vector(1000, 0x5EED0014)
    v[777] = 4.0
    v[333] = 4.0
    assert O.argmax(v) == 333


def test_half_float_rounding(oracle_lib):
    # src/core/half_float.zig:47-77
    for value in (0.0, -0.0, 1.0, -1.0, 0.5, 2.0, 1024.0, 0.0009765625, 65504.0):
        assert O.from_f16(O.to_f16(value)) == value
    assert O.from_f16(O.to_f16(1.0 + 1.0 / 2048.0)) == 1.0
    assert O.from_f16(O.to_f16(1.0 + 3.0 / 2048.0)) == 1.0 + 2.0 / 1024.0
    assert math.isinf(O.from_f16(O.to_f16(1e30))) and O.from_f16(O.to_f16(-1e30)) < 0
    v = 1e-4
    while v < 1.0:
        assert abs(O.from_f16(O.to_f16(v)) - v) / v < 0.0005
        v *= 1.7


def test_f16_matches_ieee_rne(oracle_lib):
    # The f16 conversion against IEEE round-to-nearest-even (numpy) on many values.
    rng = np.random.default_rng(3)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    ours = np.array([O.to_f16(float(x)) for x in v], np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(ours, v.astype(np.float16).view(np.uint16))

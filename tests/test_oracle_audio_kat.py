"""The audio-tower restatement (oracle/qw_oracle_audio.cpp) against the
reference's own known-answer tests, then against a float64 numpy
restatement of the same algorithms on random inputs.

Known answers (read from the reference's test blocks):
- src/core/math.zig:134-172: erf at ten points within 2e-7 of the C library's
  double erf, oddness and saturation, gelu(0), gelu(+-1), gelu(-10);
- src/core/qwen3_asr/kernels.zig:973-1041: the hand-computed 3x3 stride-2
  convolution (centre taps 1, 3, 7, 9) and the two-channel case (59);
- src/core/qwen3_asr/kernels.zig:1043-1078: windowed attention mixes only
  inside its window, and averages identical keys;
- src/core/qwen3_asr/model.zig:1137-1170: the sinusoidal position rows;
- src/core/model_config.zig:417-433: 390 packed steps for 3000 frames (375
  when convolved as one input), 104 for 800, 13 per chunk.
"""

import math

import numpy as np
import pytest

import oracle as O
from qwenscriber_b200 import config as qcfg

pytestmark = pytest.mark.usefixtures("oracle_lib")


def f16_bits(values):
    return np.asarray(values, np.float16).view(np.uint16)


def test_erf_and_gelu_known_answers():
    cases = [(0.0, 0.0), (0.1, 0.1124629160182849), (0.5, 0.5204998778130465), (1.0, 0.8427007929497149),
             (1.5, 0.9661051464753107), (2.0, 0.9953222650189527), (3.0, 0.9999779095030014),
             (4.0, 0.9999999845827421), (-0.75, -0.7111556336535151), (-2.5, -0.999593047982555)]
    for x, want in cases:
        assert abs(O.erf(x) - want) <= 2e-7, x
    assert O.erf(0.0) == 0.0
    assert abs(O.erf(-40.0) + 1.0) <= 1e-6 and abs(O.erf(40.0) - 1.0) <= 1e-6
    for x in np.arange(-6.0, 6.0001, 0.25, dtype=np.float32):
        assert abs(-O.erf(-float(x)) - O.erf(float(x))) <= 1e-7
    assert abs(O.gelu(0.0)) <= 1e-7
    assert abs(O.gelu(1.0) - 0.84134475) <= 1e-6
    assert abs(O.gelu(-1.0) + 0.15865525) <= 1e-6
    assert abs(O.gelu(-10.0)) <= 1e-6


def test_convolution_known_answers():
    centre = f16_bits([0, 0, 0, 0, 1, 0, 0, 0, 0]).reshape(1, 1, 3, 3)
    x = np.arange(1, 10, dtype=np.float32).reshape(1, 3, 3)
    out = O.conv3x3_stride2_gelu(x, centre, np.zeros(1, np.float32))
    assert out.shape == (1, 2, 2)
    for got, v in zip(out.reshape(-1), [1.0, 3.0, 7.0, 9.0]):
        assert abs(got - O.gelu(v)) <= 1e-5

    top_left = f16_bits([1, 0, 0, 0, 0, 0, 0, 0, 0]).reshape(1, 1, 3, 3)
    w = np.concatenate([centre, top_left], axis=1)
    x2 = np.concatenate([x, 10 * x]).astype(np.float32)
    out = O.conv3x3_stride2_gelu(x2, w, np.zeros(1, np.float32))
    for got, v in zip(out.reshape(-1), [1.0, 3.0, 7.0, 59.0]):
        assert abs(got - O.gelu(v)) <= 1e-5


def test_windowed_attention_known_answers():
    q = np.array([[1.0, 0.0], [0.0, 1.0]], np.float32)
    v = np.array([[5.0, 6.0], [7.0, 8.0]], np.float32)
    out = O.audio_attention_window(q, q, v, 0, 1, 1, 2)
    assert np.allclose(out[0], [5.0, 6.0], atol=1e-6) and np.all(out[1] == 0.0)
    out = O.audio_attention_window(q, q, v, 1, 1, 1, 2)
    assert np.all(out[0] == 0.0) and np.allclose(out[1], [7.0, 8.0], atol=1e-6)

    q = np.array([[1.0, 0.0], [1.0, 0.0]], np.float32)
    v = np.array([[2.0, 0.0], [4.0, 0.0]], np.float32)
    out = O.audio_attention_window(q, q, v, 0, 2, 1, 2)
    assert abs(out[0, 0] - 3.0) <= 1e-5 and abs(out[1, 0] - 3.0) <= 1e-5


def test_sinusoidal_position_known_answers():
    row = O.add_sinusoidal_position(np.zeros(64, np.float32), 0)
    assert np.all(row[:32] == 0.0) and np.allclose(row[32:], 1.0, atol=1e-6)
    row = O.add_sinusoidal_position(np.zeros(64, np.float32), 1)
    assert np.all(np.abs(row) <= 1.0)
    assert abs(row[0] - math.sin(1.0)) <= 1e-6 and abs(row[32] - math.cos(1.0)) <= 1e-6
    assert abs(row[1]) > abs(row[30]) and abs(row[62]) > abs(row[32])
    assert abs(row[62] - 1.0) <= 1e-4
    seeded = O.add_sinusoidal_position(np.full(64, 0.25, np.float32), 0)
    assert np.allclose(seeded[:32], 0.25, atol=1e-6) and np.allclose(seeded[32:], 1.25, atol=1e-6)


def test_packed_step_counts():
    c = qcfg.Config()  # the 0.6B geometry: n_window 50, n_window_infer 800
    a = O.OracleAudio(c.pack())
    try:
        assert a.packed_steps(3000) == 390
        assert a.packed_steps(800) == 104
        assert a.packed_steps(100) == 13
        assert a.packed_steps(150) == 13 + 7
        assert a.packed_steps(1) == 1
    finally:
        a.close()


# ---- float64 restatements on random inputs ----

def _gelu64(x):
    return 0.5 * x * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))


def test_convolution_matches_float64():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((5, 13, 10)).astype(np.float32)
    w = (rng.standard_normal((7, 5, 3, 3)) * 0.2).astype(np.float16)
    b = rng.standard_normal(7).astype(np.float32)
    got = O.conv3x3_stride2_gelu(x, w.view(np.uint16), b)
    xp = np.pad(x.astype(np.float64), ((0, 0), (1, 1), (1, 1)))
    oh, ow = (13 - 1) // 2 + 1, (10 - 1) // 2 + 1
    ref = np.zeros((7, oh, ow))
    for r in range(oh):
        for c in range(ow):
            patch = xp[:, 2 * r:2 * r + 3, 2 * c:2 * c + 3]
            ref[:, r, c] = np.tensordot(w.astype(np.float64), patch, axes=([1, 2, 3], [0, 1, 2])) + b
    np.testing.assert_allclose(got, _gelu64(ref), rtol=1e-5, atol=1e-5)


def test_attention_and_layer_norm_match_float64():
    rng = np.random.default_rng(4)
    steps, heads, hd = 30, 3, 8
    q, k, v = (rng.standard_normal((steps, heads * hd)).astype(np.float32) for _ in range(3))
    out = np.zeros_like(q)
    for start in range(0, steps, 13):  # windows of 13 steps, the last one ragged
        O.audio_attention_window(q, k, v, start, min(13, steps - start), heads, hd, out=out)
    ref = np.zeros((steps, heads * hd))
    for start in range(0, steps, 13):
        end = min(start + 13, steps)
        for h in range(heads):
            sl = slice(h * hd, (h + 1) * hd)
            s = q[start:end, sl].astype(np.float64) @ k[start:end, sl].T.astype(np.float64) / math.sqrt(hd)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            ref[start:end, sl] = p @ v[start:end, sl]
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)

    x = (rng.standard_normal((6, 96)) * 3 + 1).astype(np.float32)
    w = rng.standard_normal(96).astype(np.float32)
    b = rng.standard_normal(96).astype(np.float32)
    got = O.layer_norm(x, w, b, 1e-5)
    x64 = x.astype(np.float64)
    mu = x64.mean(axis=1, keepdims=True)
    var = ((x64 - mu) ** 2).mean(axis=1, keepdims=True)
    np.testing.assert_allclose(got, (x64 - mu) / np.sqrt(var + 1e-5) * w + b, rtol=1e-5, atol=1e-5)

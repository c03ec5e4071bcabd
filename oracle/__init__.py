"""CPU oracle for the Qwenscriber decoder token loop (TEST INFRASTRUCTURE ONLY).

A ctypes binding over ``oracle/liboracle.so``, the C++ restatement of the
reference's Zig CPU path (``src/core/{quant,half_float,math}.zig``,
``src/core/qwen3_asr/{kernels,decoder,model}.zig``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import
this package; the product (``qwenscriber_b200``) never does.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from ctypes import POINTER, c_float, c_int, c_int32, c_size_t, c_uint8, c_uint16, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

F32, F16, BF16, Q4, Q5, Q8 = 0, 1, 2, 16, 17, 18
DATA_BYTES_PER_GROUP = {Q4: 32, Q5: 40, Q8: 64}
GROUP = 64


def build() -> str:
    """Compiles liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    fp = POINTER(c_float)
    u8p = POINTER(c_uint8)
    u32p = POINTER(c_uint32)
    sig = {
        "orc_to_f16": (c_uint16, [c_float]),
        "orc_from_f16": (c_float, [c_uint16]),
        "orc_quantize_row": (None, [c_int, fp, c_size_t, u8p, u8p]),
        "orc_quantize_rows": (None, [c_int, fp, c_size_t, c_size_t, u8p, u8p, c_int]),
        "orc_dequantize_row": (None, [c_int, u8p, u8p, c_size_t, fp]),
        "orc_dot_row": (c_float, [c_int, u8p, u8p, fp, c_size_t]),
        "orc_dot_f32": (c_float, [fp, fp, c_size_t]),
        "orc_linear_quantized": (c_int32, [fp, fp, c_int, u8p, u8p, c_uint32, c_uint32, c_uint32, c_int]),
        "orc_rmsnorm": (None, [fp, fp, c_uint32, c_uint32, c_float]),
        "orc_silu_mul": (None, [fp, fp, fp, c_size_t]),
        "orc_silu": (c_float, [c_float]),
        "orc_softmax": (None, [fp, c_size_t]),
        "orc_inverse_frequency": (c_float, [c_uint32, c_uint32, c_float]),
        "orc_pow_f32": (c_float, [c_float, c_float]),
        "orc_build_rope_tables": (None, [fp, fp, c_uint32, c_float, c_uint32, c_uint32]),
        "orc_rope": (None, [fp, u32p, c_uint32, c_uint32, c_uint32, fp, fp, c_uint32]),
        "orc_decode_attention_f32": (c_int32, [fp, fp, fp, fp, c_uint32, c_uint32, c_uint32, c_uint32, fp]),
        "orc_decode_attention_q8": (
            c_int32,
            [fp, fp, u8p, u8p, u8p, u8p, c_uint32, c_uint32, c_uint32, c_uint32, fp],
        ),
        "orc_argmax": (c_uint32, [fp, c_size_t]),
        "orc_quant_hash": (c_uint64, []),
        "orc_model_new": (c_void_p, [c_void_p, c_uint32, c_uint32]),
        "orc_model_free": (None, [c_void_p]),
        "orc_model_set_threads": (None, [c_void_p, c_int]),
        "orc_model_set_tensor": (
            c_int32,
            [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_size_t],
        ),
        "orc_model_finish": (c_int32, [c_void_p]),
        "orc_decoder_reset": (None, [c_void_p]),
        "orc_decoder_position": (c_uint32, [c_void_p]),
        "orc_decoder_set_state": (c_int32, [c_void_p, c_void_p, c_void_p, c_uint64, c_uint32]),
        "orc_forward_token": (c_int32, [c_void_p, c_uint32, fp, c_int]),
        "orc_argmax_logits": (c_uint32, [c_void_p]),
        "orc_prefill": (c_int32, [c_void_p, u32p, c_uint32, fp, c_uint32, u32p]),
        "orc_step": (c_int32, [c_void_p, c_uint32, u32p]),
        "orc_logits": (fp, [c_void_p]),
        "orc_hidden": (fp, [c_void_p]),
        "orc_scratch": (fp, [c_void_p, c_int, POINTER(c_uint32)]),
        "orc_cache_keys_q8": (u8p, [c_void_p, POINTER(c_uint64)]),
        "orc_cache_values_q8": (u8p, [c_void_p, POINTER(c_uint64)]),
        "orc_rope_cos": (fp, [c_void_p]),
        "orc_rope_sin": (fp, [c_void_p]),
        "orc_erf": (c_float, [c_float]),
        "orc_gelu": (c_float, [c_float]),
        "orc_layer_norm": (None, [fp, fp, fp, c_uint32, c_uint32, c_float]),
        "orc_conv3x3_stride2_gelu": (
            c_int32,
            [fp, fp, POINTER(c_uint16), fp, c_uint32, c_uint32, c_uint32, c_uint32, c_int],
        ),
        "orc_audio_attention_window": (
            c_int32,
            [fp, c_uint32, fp, c_uint32, fp, c_uint32, fp, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32],
        ),
        "orc_add_sinusoidal_position": (None, [fp, c_uint32, c_uint32]),
        "orc_audio_new": (c_void_p, [c_void_p, c_uint32]),
        "orc_audio_free": (None, [c_void_p]),
        "orc_audio_set_threads": (None, [c_void_p, c_int]),
        "orc_audio_set_tensor": (
            c_int32,
            [c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_size_t],
        ),
        "orc_audio_finish": (c_int32, [c_void_p]),
        "orc_audio_packed_steps": (c_uint32, [c_void_p, c_uint32]),
        "orc_audio_encode_conv": (c_int32, [c_void_p, fp, c_uint32, u32p]),
        "orc_audio_encode_tower": (c_int32, [c_void_p, c_uint32]),
        "orc_audio_project_steps": (c_int32, [c_void_p, c_uint32, fp]),
        "orc_audio_project": (c_int32, [c_void_p, fp, c_uint32, fp, c_uint64, u32p]),
        "orc_audio_encoded": (fp, [c_void_p, POINTER(c_uint32)]),
    }
    for name, (restype, argtypes) in sig.items():
        fn = getattr(L, name)
        fn.restype = restype
        fn.argtypes = argtypes


def _fp(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(POINTER(c_float))


def _u8p(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(POINTER(c_uint8))


def _u32p(a: np.ndarray):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(POINTER(c_uint32))


def to_f16(value: float) -> int:
    return int(lib().orc_to_f16(value))


def from_f16(bits: int) -> float:
    return float(lib().orc_from_f16(bits))


def quantize_rows(fmt: int, values: np.ndarray, threads: int = 8) -> tuple[np.ndarray, np.ndarray]:
    """quant.zig:197-227 over each row: returns (scales u8[rows, groups*2], codes u8[rows, groups*bytes])."""
    values = np.ascontiguousarray(values, dtype=np.float32)
    rows, cols = values.shape
    groups = cols // GROUP
    scales = np.zeros((rows, groups * 2), np.uint8)
    data = np.zeros((rows, groups * DATA_BYTES_PER_GROUP[fmt]), np.uint8)
    lib().orc_quantize_rows(fmt, _fp(values), rows, cols, _u8p(scales), _u8p(data), threads)
    return scales, data


def dequantize_rows(fmt: int, scales: np.ndarray, data: np.ndarray, cols: int) -> np.ndarray:
    rows = scales.shape[0]
    out = np.zeros((rows, cols), np.float32)
    scales = np.ascontiguousarray(scales)
    data = np.ascontiguousarray(data)
    for r in range(rows):
        lib().orc_dequantize_row(fmt, _u8p(scales[r]), _u8p(data[r]), cols, _fp(out[r]))
    return out


def linear_quantized(fmt: int, scales: np.ndarray, data: np.ndarray, x: np.ndarray, threads: int = 8) -> np.ndarray:
    """kernels.zig:118-158: out[tokens, rows]."""
    scales = np.ascontiguousarray(scales)
    data = np.ascontiguousarray(data)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = x[None, :]
    tokens, cols = x.shape
    rows = scales.shape[0]
    out = np.zeros((tokens, rows), np.float32)
    st = lib().orc_linear_quantized(_fp(out), _fp(x), fmt, _u8p(scales), _u8p(data), rows, cols, tokens, threads)
    assert st == 0, st
    return out


def rmsnorm(x: np.ndarray, weight: np.ndarray, width: int, eps: float) -> np.ndarray:
    out = np.ascontiguousarray(x, dtype=np.float32).copy()
    tokens = out.size // width
    lib().orc_rmsnorm(_fp(out), _fp(np.ascontiguousarray(weight, np.float32)), width, tokens, eps)
    return out


def silu_mul(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    gate = np.ascontiguousarray(gate, np.float32)
    up = np.ascontiguousarray(up, np.float32)
    out = np.zeros_like(gate)
    lib().orc_silu_mul(_fp(out), _fp(gate), _fp(up), gate.size)
    return out


def softmax(row: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(row, np.float32).copy()
    lib().orc_softmax(_fp(out), out.size)
    return out


def rope_tables(half: int, theta: float, max_positions: int) -> tuple[np.ndarray, np.ndarray]:
    cos = np.zeros(max_positions * half, np.float32)
    sin = np.zeros(max_positions * half, np.float32)
    lib().orc_build_rope_tables(_fp(cos), _fp(sin), half, theta, max_positions, half)
    return cos, sin


def rope(x: np.ndarray, positions, heads: int, head_dim: int, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    out = np.ascontiguousarray(x, np.float32).copy()
    pos = np.ascontiguousarray(np.asarray(positions, np.uint32))
    lib().orc_rope(_fp(out), _u32p(pos), pos.size, heads, head_dim, _fp(cos), _fp(sin), head_dim // 2)
    return out


def decode_attention_q8(query, k_scales, k_codes, v_scales, v_codes, cached, heads, kv_heads, head_dim):
    out = np.zeros(heads * head_dim, np.float32)
    scores = np.zeros(max(cached, 1), np.float32)
    st = lib().orc_decode_attention_q8(
        _fp(out), _fp(np.ascontiguousarray(query, np.float32)),
        _u8p(np.ascontiguousarray(k_scales)), _u8p(np.ascontiguousarray(k_codes)),
        _u8p(np.ascontiguousarray(v_scales)), _u8p(np.ascontiguousarray(v_codes)),
        cached, heads, kv_heads, head_dim, _fp(scores),
    )
    assert st == 0, st
    return out


def decode_attention_f32(query, keys, values, cached, heads, kv_heads, head_dim):
    out = np.zeros(heads * head_dim, np.float32)
    scores = np.zeros(max(cached, 1), np.float32)
    st = lib().orc_decode_attention_f32(
        _fp(out), _fp(np.ascontiguousarray(query, np.float32)), _fp(np.ascontiguousarray(keys, np.float32)),
        _fp(np.ascontiguousarray(values, np.float32)), cached, heads, kv_heads, head_dim, _fp(scores),
    )
    assert st == 0, st
    return out


def argmax(values: np.ndarray) -> int:
    v = np.ascontiguousarray(values, np.float32)
    return int(lib().orc_argmax(_fp(v), v.size))


def quant_hash() -> int:
    return int(lib().orc_quant_hash())


class OracleModel:
    """decoder.zig's Decoder over borrowed payloads (same tensor API as the CUDA backend)."""

    def __init__(self, config_bytes: bytes, cache_format: int = 1, threads: int = 8):
        self._L = lib()
        self._cfg = ctypes.create_string_buffer(bytes(config_bytes), len(config_bytes))
        self._h = self._L.orc_model_new(self._cfg, len(config_bytes), cache_format)
        if not self._h:
            raise ValueError("orc_model_new refused the configuration")
        self._keep = []
        self._L.orc_model_set_threads(self._h, threads)
        self.config_bytes = bytes(config_bytes)

    def close(self):
        if self._h:
            self._L.orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, kind: int, layer: int, fmt: int, rows: int, cols: int, payload: np.ndarray) -> None:
        payload = np.ascontiguousarray(payload)
        self._keep.append(payload)
        st = self._L.orc_model_set_tensor(self._h, kind, layer, fmt, rows, cols, payload.ctypes.data, payload.nbytes)
        if st != 0:
            raise RuntimeError(f"orc_model_set_tensor({kind},{layer}) -> {st}")

    def finish(self) -> None:
        st = self._L.orc_model_finish(self._h)
        if st != 0:
            raise RuntimeError(f"orc_model_finish -> {st}")

    def reset(self) -> None:
        self._L.orc_decoder_reset(self._h)

    @property
    def position(self) -> int:
        return int(self._L.orc_decoder_position(self._h))

    def set_state(self, keys: np.ndarray, values: np.ndarray, position: int) -> None:
        """Loads whole q8 cache planes (the reference layout) and moves the decoder to `position`."""
        k = np.ascontiguousarray(keys, np.uint8)
        v = np.ascontiguousarray(values, np.uint8)
        st = self._L.orc_decoder_set_state(self._h, k.ctypes.data, v.ctypes.data, k.size, position)
        assert st == 0, st

    def forward_token(self, token: int, audio_row: np.ndarray | None = None, want_logits: bool = True) -> None:
        row = None
        if audio_row is not None:
            row = np.ascontiguousarray(audio_row, np.float32)
        st = self._L.orc_forward_token(self._h, token, _fp(row) if row is not None else None, 1 if want_logits else 0)
        if st != 0:
            raise RuntimeError(f"orc_forward_token -> {st}")

    def prefill(self, tokens: np.ndarray, audio: np.ndarray, audio_steps: int) -> int:
        toks = np.ascontiguousarray(tokens, np.uint32)
        aud = np.ascontiguousarray(audio, np.float32).reshape(-1)
        out = np.zeros(1, np.uint32)
        st = self._L.orc_prefill(self._h, _u32p(toks), toks.size, _fp(aud), audio_steps, _u32p(out))
        if st != 0:
            raise RuntimeError(f"orc_prefill -> {st}")
        return int(out[0])

    def step(self, token: int) -> int:
        out = np.zeros(1, np.uint32)
        st = self._L.orc_step(self._h, token, _u32p(out))
        if st != 0:
            raise RuntimeError(f"orc_step -> {st}")
        return int(out[0])

    def logits(self, vocab: int) -> np.ndarray:
        p = self._L.orc_logits(self._h)
        return np.ctypeslib.as_array(p, shape=(vocab,)).copy()

    def hidden(self, width: int) -> np.ndarray:
        p = self._L.orc_hidden(self._h)
        return np.ctypeslib.as_array(p, shape=(width,)).copy()

    def scratch(self, which: int) -> np.ndarray:
        n = c_uint32(0)
        p = self._L.orc_scratch(self._h, which, ctypes.byref(n))
        return np.ctypeslib.as_array(p, shape=(n.value,)).copy()

    def cache_q8(self) -> tuple[np.ndarray, np.ndarray]:
        n = c_uint64(0)
        pk = self._L.orc_cache_keys_q8(self._h, ctypes.byref(n))
        keys = np.ctypeslib.as_array(pk, shape=(n.value,)).copy() if n.value else np.zeros(0, np.uint8)
        pv = self._L.orc_cache_values_q8(self._h, ctypes.byref(n))
        values = np.ctypeslib.as_array(pv, shape=(n.value,)).copy() if n.value else np.zeros(0, np.uint8)
        return keys, values

    def rope_tables(self, max_positions: int, half: int) -> tuple[np.ndarray, np.ndarray]:
        c = np.ctypeslib.as_array(self._L.orc_rope_cos(self._h), shape=(max_positions * half,)).copy()
        s = np.ctypeslib.as_array(self._L.orc_rope_sin(self._h), shape=(max_positions * half,)).copy()
        return c, s


# ---- the audio tower and projector (qw_oracle_audio.cpp) ----


def erf(x: float) -> float:
    return float(lib().orc_erf(x))


def gelu(x: float) -> float:
    return float(lib().orc_gelu(x))


def layer_norm(x: np.ndarray, weight: np.ndarray, bias: np.ndarray, eps: float) -> np.ndarray:
    """math.zig:99-116 over every row of x [tokens][width]."""
    out = np.ascontiguousarray(x, np.float32).copy()
    tokens, width = out.reshape(-1, x.shape[-1]).shape
    lib().orc_layer_norm(_fp(out), _fp(np.ascontiguousarray(weight, np.float32)),
                         _fp(np.ascontiguousarray(bias, np.float32)), width, tokens, eps)
    return out


def conv3x3_stride2_gelu(x: np.ndarray, weights_f16: np.ndarray, bias: np.ndarray, threads: int = 8) -> np.ndarray:
    """kernels.zig:332-362: x [in_ch][h][w] f32, weights [out][in][3][3] as f16 bits (uint16)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weights_f16, np.uint16)
    in_ch, h, wd = x.shape
    out_ch = w.shape[0]
    out = np.zeros((out_ch, (h - 1) // 2 + 1, (wd - 1) // 2 + 1), np.float32)
    st = lib().orc_conv3x3_stride2_gelu(_fp(out), _fp(x), w.ctypes.data_as(POINTER(c_uint16)),
                                        _fp(np.ascontiguousarray(bias, np.float32)), out_ch, in_ch, h, wd, threads)
    assert st == 0, st
    return out


def audio_attention_window(q: np.ndarray, k: np.ndarray, v: np.ndarray, start: int, length: int, heads: int,
                           head_dim: int, out: np.ndarray | None = None) -> np.ndarray:
    """kernels.zig:435-487 on [steps][heads * head_dim] rows (stride = the row width)."""
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    width = heads * head_dim
    if out is None:
        out = np.zeros_like(q)
    st = lib().orc_audio_attention_window(_fp(out), width, _fp(q), width, _fp(k), width, _fp(v), width, start, length,
                                          heads, head_dim)
    assert st == 0, st
    return out


def add_sinusoidal_position(row: np.ndarray, step: int) -> np.ndarray:
    out = np.ascontiguousarray(row, np.float32).copy()
    lib().orc_add_sinusoidal_position(_fp(out), step, out.size)
    return out


class OracleAudio:
    """model.zig's audio tower and projector over borrowed payloads."""

    def __init__(self, config_bytes: bytes, threads: int = 8):
        self._L = lib()
        self._cfg = ctypes.create_string_buffer(bytes(config_bytes), len(config_bytes))
        self._h = self._L.orc_audio_new(self._cfg, len(config_bytes))
        if not self._h:
            raise ValueError("orc_audio_new refused the configuration")
        self._keep = []
        self._L.orc_audio_set_threads(self._h, threads)
        self.steps = 0

    def close(self):
        if self._h:
            self._L.orc_audio_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_tensor(self, kind: int, layer: int, fmt: int, rows: int, cols: int, payload: np.ndarray) -> int:
        payload = np.ascontiguousarray(payload)
        self._keep.append(payload)
        return int(self._L.orc_audio_set_tensor(self._h, kind, layer, fmt, rows, cols, payload.ctypes.data,
                                                payload.nbytes))

    def finish(self) -> int:
        return int(self._L.orc_audio_finish(self._h))

    def packed_steps(self, frames: int) -> int:
        return int(self._L.orc_audio_packed_steps(self._h, frames))

    def encode_conv(self, log_mel: np.ndarray) -> int:
        mel = np.ascontiguousarray(log_mel, np.float32)
        steps = np.zeros(1, np.uint32)
        st = self._L.orc_audio_encode_conv(self._h, _fp(mel), mel.shape[1], _u32p(steps))
        if st != 0:
            raise RuntimeError(f"orc_audio_encode_conv -> {st}")
        self.steps = int(steps[0])
        return self.steps

    def encode_tower(self) -> None:
        st = self._L.orc_audio_encode_tower(self._h, self.steps)
        if st != 0:
            raise RuntimeError(f"orc_audio_encode_tower -> {st}")

    def encoded(self, width: int) -> np.ndarray:
        n = c_uint32(0)
        p = self._L.orc_audio_encoded(self._h, ctypes.byref(n))
        return np.ctypeslib.as_array(p, shape=(n.value,)).copy().reshape(-1, width)

    def project_steps(self, out_dim: int) -> np.ndarray:
        out = np.zeros((self.steps, out_dim), np.float32)
        st = self._L.orc_audio_project_steps(self._h, self.steps, _fp(out))
        if st != 0:
            raise RuntimeError(f"orc_audio_project_steps -> {st}")
        return out

    def project(self, log_mel: np.ndarray, out_dim: int) -> np.ndarray:
        """model.zig:451-460: conv stage, tower, projector."""
        self.encode_conv(log_mel)
        self.encode_tower()
        return self.project_steps(out_dim)

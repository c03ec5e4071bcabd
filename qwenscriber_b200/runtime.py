"""Python host binding of libqwenscriber_cuda (the CUDA decoder backend).

`CudaModel` mirrors the reference runtime's model and decode families
(src/wasm/exports.zig `qw_model_*` / `qw_decode_*`, src/wasm/model.zig) with
the same argument meaning, state machine and error codes: a negative status
raises `QwcError` carrying the reference's status number (src/wasm/abi.zig:50-84).

The library must have been built for sm_100a (`qwenscriber_b200.build`); there
is no CPU fallback: without the shared library or a CUDA device every call
fails loudly.
"""

from __future__ import annotations

import ctypes
import os
import struct
from ctypes import POINTER, c_char_p, c_float, c_int32, c_int64, c_uint32, c_uint64, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwenscriber_cuda.so")

STATUS = {
    0: "ok", -1: "invalid_argument", -2: "out_of_memory", -3: "unsupported", -4: "bad_magic", -5: "bad_version",
    -6: "checksum_mismatch", -7: "shape_mismatch", -8: "invalid_state", -9: "limit_exceeded", -10: "not_found",
    -11: "truncated", -12: "invalid_encoding", -13: "unsupported_model", -14: "audio_too_long",
}

STATUS_CODE = {name: code for code, name in STATUS.items()}

CACHE_F32, CACHE_Q8 = 0, 1
OPTION_IGNORE_EOS, OPTION_KEEP_LOGITS, OPTION_STEP_CHUNK, OPTION_TRACE, OPTION_PREFILL_SERIAL = 1, 2, 3, 4, 5
OPTION_EXACT, OPTION_WAIT_LIMIT_US, OPTION_TEST_STALL = 6, 7, 8
FEATURE_MODEL, FEATURE_DECODE, FEATURE_STREAMS = 1 << 3, 1 << 4, 1 << 8
LIMIT_EXCEEDED = -9
UNSUPPORTED_MODEL = -13
ARGMAX_NOALLOC_MAX_COUNT = 4194304  # QWC_ARGMAX_NOALLOC_MAX_COUNT

# Every symbol include/qwenscriber_cuda.h declares: (restype, argtypes).
SIGNATURES = {
    "qwc_abi_version": (c_uint32, []),
    "qwc_features": (c_uint32, []),
    "qwc_create": (c_uint32, [c_int32]),
    "qwc_destroy": (c_int32, [c_uint32]),
    "qwc_status_message": (c_char_p, [c_int32]),
    "qwc_set_option": (c_int32, [c_uint32, c_uint32, c_uint32]),
    "qwc_model_begin": (c_int32, [c_uint32]),
    "qwc_model_add_shard": (c_int32, [c_uint32, c_void_p, c_uint64]),
    "qwc_shard_validate": (c_int32, [c_void_p, c_uint64, c_void_p]),
    "qwc_shard_checksum": (c_uint32, [c_void_p, c_uint64]),
    "qwc_model_add_tensor": (c_int32, [c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_uint64]),
    "qwc_model_set_cache_format": (c_int32, [c_uint32, c_uint32]),
    "qwc_model_set_streams": (c_int32, [c_uint32, c_uint32]),
    "qwc_model_finish": (c_int32, [c_uint32, c_void_p, c_uint32]),
    "qwc_model_requirements": (c_int32, [c_uint32, c_void_p]),
    "qwc_model_tensor_count": (c_int32, [c_uint32, POINTER(c_uint32)]),
    "qwc_model_tensor_descriptor": (c_int32, [c_uint32, c_uint32, c_void_p]),
    "qwc_decode_begin": (c_int32, [c_uint32, c_void_p, c_uint32, c_void_p, c_uint32, c_uint32]),
    "qwc_decode_step": (c_int32, [c_uint32, POINTER(c_uint32)]),
    "qwc_decode_tokens": (c_int32, [c_uint32, c_void_p, c_uint32]),
    "qwc_decode_end": (c_int32, [c_uint32]),
    "qwc_stream_begin": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint32, c_void_p, c_uint32, c_uint32]),
    "qwc_streams_step": (c_int32, [c_uint32, c_void_p, c_void_p]),
    "qwc_stream_tokens": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint32]),
    "qwc_stream_end": (c_int32, [c_uint32, c_uint32]),
    "qwc_streams_run_timed": (c_int32, [c_uint32, c_uint32, c_void_p]),
    "qwc_decode_run_timed": (c_int32, [c_uint32, c_uint32, POINTER(c_float)]),
    "qwc_debug_logits": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint32]),
    "qwc_debug_hold": (c_int32, [c_uint32, c_uint32, c_int64, POINTER(c_uint32)]),
    "qwc_debug_scratch": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint32]),
    "qwc_debug_trace": (c_int32, [c_uint32, c_void_p, c_uint32]),
    "qwc_debug_cache": (c_int32, [c_uint32, c_uint32, c_uint32, c_void_p, c_uint64]),
    "qwc_kernel_launches": (c_uint64, [c_uint32]),
    "qwc_model_audio_config": (c_int32, [c_uint32, c_void_p]),
    "qwc_audio_project": (c_int32, [c_uint32, c_void_p, c_uint32, c_void_p, c_uint64, POINTER(c_uint32)]),
    "qwc_decode_begin_features": (c_int32, [c_uint32, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32]),
    "qwc_stream_begin_features": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32]),
    "qwc_debug_audio": (c_int32, [c_uint32, c_uint32, c_void_p, c_uint64]),
    "qwc_audio_run_timed": (c_int32, [c_uint32, c_void_p, c_uint32, c_uint32, POINTER(c_float), POINTER(c_uint32)]),
    "qwc_rope_tables": (c_int32, [c_float, c_uint32, c_uint32, c_void_p, c_void_p]),
    "qwc_op_dequantize": (c_int32, [c_uint32, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_void_p]),
    "qwc_op_quantize_q8": (c_int32, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    "qwc_op_gemv": (c_int32, [c_uint32, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    "qwc_op_attention_q8": (
        c_int32,
        [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p],
    ),
    "qwc_op_argmax": (c_int32, [c_void_p, c_uint32, c_void_p, c_void_p]),
    "qwc_op_argmax_noalloc": (c_int32, [c_void_p, c_uint32, c_void_p, c_void_p]),
    "qwc_op_gemm_streams": (c_int32, [c_uint32, c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_uint32,
                                      c_void_p, c_void_p]),
    "qwc_op_rmsnorm": (c_int32, [c_void_p, c_void_p, c_uint32, c_uint32, c_float, c_void_p, c_void_p]),
    "qwc_op_rope": (c_int32, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p]),
    "qwc_op_silu_mul": (c_int32, [c_void_p, c_void_p, c_uint32, c_void_p, c_void_p]),
}


class QwcError(RuntimeError):
    def __init__(self, status: int, call: str):
        self.status = status
        self.name = STATUS.get(status, "unknown")
        super().__init__(f"{call} failed: {self.name} ({status})")


_lib = None


def lib() -> ctypes.CDLL:
    """Loads the in-tree shared library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} is missing: run qwenscriber_b200.build.build() first")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def aligned_copy(data: bytes | np.ndarray, alignment: int = 16) -> np.ndarray:
    """The bytes of `data` in a fresh uint8 array whose first byte is
    `alignment`-aligned."""
    raw = np.frombuffer(bytes(data), np.uint8) if not isinstance(data, np.ndarray) else data.view(np.uint8).ravel()
    store = np.empty(raw.nbytes + alignment, np.uint8)
    start = (-store.ctypes.data) % alignment
    out = store[start:start + raw.nbytes]
    out[:] = raw
    return out


def shard_validate(shard: bytes | np.ndarray) -> tuple[int, int]:
    """qwc_shard_validate: (status, tensor count); needs no GPU."""
    buf = aligned_copy(shard)
    count = ctypes.c_uint32(0)
    status = lib().qwc_shard_validate(buf.ctypes.data, buf.nbytes, ctypes.byref(count))
    return status, count.value


def check(status: int, call: str) -> int:
    if status < 0:
        raise QwcError(status, call)
    return status


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class Requirements(ctypes.Structure):
    _fields_ = [
        ("weight_bytes", c_uint64), ("cache_bytes", c_uint64), ("scratch_bytes", c_uint64), ("total_bytes", c_uint64),
        ("max_positions", c_uint32), ("max_audio_frames", c_uint32), ("max_decode_tokens", c_uint32),
        ("reserved", c_uint32),
    ]


assert ctypes.sizeof(Requirements) == 48


class CudaModel:
    """One handle bound to one CUDA device: a loaded decoder and its streams."""

    def __init__(self, device: int = 0):
        self._L = lib()
        self.handle = self._L.qwc_create(device)
        if self.handle == 0:
            raise QwcError(-1, f"qwc_create({device})")
        self.vocab = 0

    def close(self) -> None:
        if self.handle:
            self._L.qwc_destroy(self.handle)
            self.handle = 0

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- model family ----
    def begin(self) -> None:
        check(self._L.qwc_model_begin(self.handle), "qwc_model_begin")

    def add_tensor(self, kind: int, layer: int, fmt: int, rows: int, cols: int, payload: np.ndarray) -> None:
        p = np.ascontiguousarray(payload)
        check(self._L.qwc_model_add_tensor(self.handle, kind, layer, fmt, rows, cols, p.ctypes.data, p.nbytes),
              f"qwc_model_add_tensor(kind={kind}, layer={layer})")

    def add_shard(self, shard: bytes | np.ndarray) -> None:
        """qwc_model_add_shard on a whole `.qw` shard (copied into a 16-byte
        aligned buffer first, as the ABI requires)."""
        buf = aligned_copy(shard)
        check(self._L.qwc_model_add_shard(self.handle, buf.ctypes.data, buf.nbytes), "qwc_model_add_shard")

    def set_cache_format(self, fmt: int) -> None:
        check(self._L.qwc_model_set_cache_format(self.handle, fmt), "qwc_model_set_cache_format")

    def set_streams(self, n: int) -> None:
        check(self._L.qwc_model_set_streams(self.handle, n), "qwc_model_set_streams")

    def finish(self, config_bytes: bytes) -> None:
        buf = ctypes.create_string_buffer(bytes(config_bytes), len(config_bytes))
        check(self._L.qwc_model_finish(self.handle, buf, len(config_bytes)), "qwc_model_finish")
        from .config import Config
        self.vocab = Config.unpack(bytes(config_bytes)).vocab_size

    def requirements(self) -> dict:
        r = Requirements()
        check(self._L.qwc_model_requirements(self.handle, ctypes.byref(r)), "qwc_model_requirements")
        return {name: getattr(r, name) for name, _ in Requirements._fields_}

    def tensor_count(self) -> int:
        n = c_uint32(0)
        check(self._L.qwc_model_tensor_count(self.handle, ctypes.byref(n)), "qwc_model_tensor_count")
        return n.value

    def tensor_descriptor(self, index: int) -> dict:
        """qwc_model_tensor_descriptor: the 64-byte descriptor as a dict."""
        raw = (ctypes.c_uint8 * 64)()
        check(self._L.qwc_model_tensor_descriptor(self.handle, index, ctypes.addressof(raw)),
              "qwc_model_tensor_descriptor")
        b = bytes(raw)
        off, length = struct.unpack_from("<QQ", b, 0)
        kind, layer, fmt, rank, d0, d1, d2, d3, shard_index = struct.unpack_from("<9I", b, 16)
        return {"offset_bytes": off, "len_bytes": length, "kind": kind, "layer": layer, "format": fmt,
                "rank": rank, "dims": (d0, d1, d2, d3), "shard_index": shard_index}

    def set_option(self, option: int, value: int) -> None:
        check(self._L.qwc_set_option(self.handle, option, value), "qwc_set_option")

    # ---- decode family (stream 0) ----
    def decode_begin(self, prompt, audio: np.ndarray | None, max_tokens: int) -> None:
        ids = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        rows = None if audio is None else np.ascontiguousarray(audio, dtype=np.float32)
        steps = 0 if rows is None else rows.shape[0]
        check(self._L.qwc_decode_begin(self.handle, ids.ctypes.data, ids.size, _ptr(rows), steps, max_tokens),
              "qwc_decode_begin")

    def decode_step(self) -> int | None:
        """The next token, or None once the sequence has finished (qw_decode_step's 1 / 0)."""
        out = c_uint32(0)
        r = check(self._L.qwc_decode_step(self.handle, ctypes.byref(out)), "qwc_decode_step")
        return out.value if r == 1 else None

    def decode_tokens(self, capacity: int = 8192) -> list[int]:
        out = np.zeros(capacity, np.uint32)
        n = check(self._L.qwc_decode_tokens(self.handle, out.ctypes.data, capacity), "qwc_decode_tokens")
        return out[:n].tolist()

    def decode_end(self) -> None:
        check(self._L.qwc_decode_end(self.handle), "qwc_decode_end")

    def run_timed(self, steps: int) -> float:
        ms = c_float(0.0)
        check(self._L.qwc_decode_run_timed(self.handle, steps, ctypes.byref(ms)), "qwc_decode_run_timed")
        return ms.value

    # ---- multi-stream family (handles with set_streams(n), n >= 2) ----
    def stream_begin(self, slot: int, prompt, audio: np.ndarray | None, max_tokens: int) -> None:
        ids = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        rows = None if audio is None or len(audio) == 0 else np.ascontiguousarray(audio, dtype=np.float32)
        steps = 0 if rows is None else rows.shape[0]
        check(self._L.qwc_stream_begin(self.handle, slot, ids.ctypes.data, ids.size, _ptr(rows), steps, max_tokens),
              "qwc_stream_begin")

    def streams_step(self, slots: int) -> tuple[np.ndarray, np.ndarray, int]:
        """One batched step: (tokens, results, produced); results 1 = token, 2 = prompt position, 0 = idle/done."""
        tokens = np.zeros(max(slots, 64), np.uint32)
        results = np.zeros(max(slots, 64), np.int32)
        n = check(self._L.qwc_streams_step(self.handle, tokens.ctypes.data, results.ctypes.data), "qwc_streams_step")
        return tokens[:slots], results[:slots], n

    def stream_tokens(self, slot: int, capacity: int = 8192) -> list[int]:
        out = np.zeros(capacity, np.uint32)
        n = check(self._L.qwc_stream_tokens(self.handle, slot, out.ctypes.data, capacity), "qwc_stream_tokens")
        return out[:n].tolist()

    def stream_end(self, slot: int) -> None:
        check(self._L.qwc_stream_end(self.handle, slot), "qwc_stream_end")

    def streams_run_timed(self, steps: int) -> float:
        ms = c_float(0.0)
        check(self._L.qwc_streams_run_timed(self.handle, steps, ctypes.byref(ms)), "qwc_streams_run_timed")
        return ms.value

    # ---- parity hooks ----
    def debug_logits(self, slot: int = 0) -> np.ndarray:
        out = np.zeros(self.vocab, np.float32)
        check(self._L.qwc_debug_logits(self.handle, slot, out.ctypes.data, out.size), "qwc_debug_logits")
        return out

    def debug_hold(self, force: int = -1, slot: int = 0) -> int:
        """The token held for the next decode step; `force` >= 0 replaces it first."""
        out = c_uint32(0)
        check(self._L.qwc_debug_hold(self.handle, slot, force, ctypes.byref(out)), "qwc_debug_hold")
        return out.value

    def debug_scratch(self, which: int, count: int = 16384) -> np.ndarray:
        out = np.zeros(count, np.float32)
        n = check(self._L.qwc_debug_scratch(self.handle, which, out.ctypes.data, count), "qwc_debug_scratch")
        return out[:n]

    def debug_trace(self, count: int = 148 * 512 * 2) -> np.ndarray:
        out = np.zeros(count, np.uint64)
        n = check(self._L.qwc_debug_trace(self.handle, out.ctypes.data, count), "qwc_debug_trace")
        return out[:n]

    def debug_cache(self, which: int, nbytes: int, slot: int = 0) -> np.ndarray:
        out = np.zeros(nbytes, np.uint8)
        check(self._L.qwc_debug_cache(self.handle, slot, which, out.ctypes.data, nbytes), "qwc_debug_cache")
        return out

    def launches(self) -> int:
        return int(self._L.qwc_kernel_launches(self.handle))

    # ---- audio family: the tower and projector ----
    AUDIO_CONFIG_FIELDS = ("d_model", "layers", "attention_heads", "head_dim", "ffn_dim", "downsample_hidden_size",
                           "n_window", "n_window_infer", "chunk_frames", "frequency_bins", "conv_out_input_features",
                           "chunk_steps", "max_position_steps", "output_dim", "mel_bins", "layer_norm_eps",
                           "reserved_0", "reserved_1")

    def audio_config(self) -> dict:
        """qwc_model_audio_config: the 72-byte qwc_audio_config as a dict."""
        buf = ctypes.create_string_buffer(72)
        check(self._L.qwc_model_audio_config(self.handle, buf), "qwc_model_audio_config")
        return dict(zip(self.AUDIO_CONFIG_FIELDS, struct.unpack("<15If2I", buf.raw)))

    def audio_project(self, log_mel: np.ndarray, out_dim: int, capacity: int | None = None) -> np.ndarray:
        """qwc_audio_project on a [mel_bins][frames] log-mel: [steps][out_dim] projected rows."""
        mel = np.ascontiguousarray(log_mel, dtype=np.float32)
        frames = mel.shape[1] if mel.ndim == 2 else 0
        cap = capacity if capacity is not None else max(1, 4 * frames) * out_dim
        out = np.zeros(cap, np.float32)
        steps = c_uint32(0)
        check(self._L.qwc_audio_project(self.handle, mel.ctypes.data, frames, out.ctypes.data, cap,
                                        ctypes.byref(steps)), "qwc_audio_project")
        return out[:steps.value * out_dim].reshape(steps.value, out_dim)

    def decode_begin_features(self, prompt, log_mel: np.ndarray, max_tokens: int) -> None:
        ids = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        mel = np.ascontiguousarray(log_mel, dtype=np.float32)
        check(self._L.qwc_decode_begin_features(self.handle, ids.ctypes.data, ids.size, mel.ctypes.data, mel.nbytes,
                                                max_tokens), "qwc_decode_begin_features")

    def stream_begin_features(self, slot: int, prompt, log_mel: np.ndarray, max_tokens: int) -> None:
        ids = np.ascontiguousarray(np.asarray(prompt, dtype=np.uint32))
        mel = np.ascontiguousarray(log_mel, dtype=np.float32)
        check(self._L.qwc_stream_begin_features(self.handle, slot, ids.ctypes.data, ids.size, mel.ctypes.data,
                                                mel.nbytes, max_tokens), "qwc_stream_begin_features")

    def debug_audio(self, which: int, steps: int, width: int) -> np.ndarray:
        out = np.zeros(steps * width, np.float32)
        n = check(self._L.qwc_debug_audio(self.handle, which, out.ctypes.data, out.size), "qwc_debug_audio")
        return out[:n].reshape(steps, width)

    def audio_run_timed(self, log_mel: np.ndarray, reps: int) -> tuple[float, int]:
        """(device ms of `reps` clips, kernels one clip launches)."""
        mel = np.ascontiguousarray(log_mel, dtype=np.float32)
        ms, launches = c_float(0.0), c_uint32(0)
        check(self._L.qwc_audio_run_timed(self.handle, mel.ctypes.data, mel.shape[1], reps, ctypes.byref(ms),
                                          ctypes.byref(launches)), "qwc_audio_run_timed")
        return ms.value, launches.value


def rope_tables(theta: float, head_dim: int, max_positions: int) -> tuple[np.ndarray, np.ndarray]:
    half = head_dim // 2
    c = np.zeros(max_positions * half, np.float32)
    s = np.zeros(max_positions * half, np.float32)
    check(lib().qwc_rope_tables(theta, head_dim, max_positions, c.ctypes.data, s.ctypes.data), "qwc_rope_tables")
    return c, s

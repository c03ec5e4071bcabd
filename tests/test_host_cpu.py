"""Host-side logic of the CUDA backend, checked on CPU (no GPU needed).

* the numpy quantizer the synthetic models use equals the oracle bit for bit;
* the tensor payload layout follows quant.zig's plane layout tests;
* the 160-byte Config round-trips with the reference's field offsets;
* libqwenscriber_cuda.so loads and exports every symbol the header declares,
  and its host-only calls (status text, rope tables, ABI version) behave;
* header constants match the reference's (the drift gate of
  tests/gpu/layout_drift.mjs, for this backend).
"""

import os
import re
import struct

import numpy as np
import pytest

import oracle as O
from qwenscriber_b200 import config as cfgmod
from qwenscriber_b200 import quant, synthetic
from qwenscriber_b200 import runtime as rt

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "qwenscriber_cuda.h")


@pytest.mark.parametrize("fmt", [quant.Q4, quant.Q5, quant.Q8])
def test_numpy_quantizer_is_bit_exact(oracle_lib, fmt):
    rng = np.random.default_rng(11)
    v = (rng.standard_normal((64, 512)) * rng.choice([1e-3, 0.02, 1.0, 40.0], size=(64, 1))).astype(np.float32)
    v[3, :64] = 0.0                                    # an all-zero group stores scale 0
    v[4, :64] = np.float32(0.5) * np.arange(64) / 64   # values landing on half steps
    v[5, 5] = 1e-30                                    # subnormal-scale group
    s_np, c_np = quant.quantize(fmt, v)
    s_or, c_or = O.quantize_rows(fmt, v)
    assert np.array_equal(s_np.view(np.uint8).reshape(s_or.shape), s_or)
    assert np.array_equal(c_np, c_or)
    # and the numpy decode equals the oracle's dequantizeRow
    assert np.array_equal(quant.dequantize(fmt, s_np, c_np, 512), O.dequantize_rows(fmt, s_or, c_or, 512))


def test_q5_packing_round_trips_every_code():
    # quant.zig:253-269: low nibbles in the q4 layout, then the fifth-bit plane.
    rng = np.random.default_rng(5)
    u = rng.integers(0, 32, size=(7, 256)).astype(np.uint8)
    u[0, :64] = np.arange(64) % 32          # every code, every bit position of a group
    packed = quant.pack_q5(u)
    assert packed.shape == (7, 4 * 40)
    assert np.array_equal(quant.unpack_q5(packed, 256), u.astype(np.int32))
    g0 = packed[0, :40]
    assert g0[0] == (0 | (1 << 4)) and g0[15] == ((30 & 15) | ((31 & 15) << 4))  # low nibbles of 0, 1 / 30, 31
    assert g0[32 + 2] == 0xFF and g0[32] == 0x00                     # weights 16..23 have the fifth bit


def test_plane_layout_matches_reference_cases():
    # quant.zig:423-435: 896 x 896 q4 at base 0, alignment 16.
    so, sl, do, dl = quant.plane_layout(quant.Q4, 896, 896)
    assert (so, sl, dl) == (0, 14 * 896 * 2, 14 * 896 * 32)
    assert do % 16 == 0 and do >= sl
    with pytest.raises(ValueError):
        quant.plane_layout(quant.Q4, 1, 100)  # RowNotGroupAligned (quant.zig:395-400)


def test_kv_cache_bytes_formula():
    # quant.zig:402-421: 28 layers, 8 kv heads x 128, 8192 positions.
    layers, kvw, positions = 28, 1024, 8192
    f32_bytes = 2 * layers * positions * kvw * 4
    q8_plane = positions * (kvw + kvw // 64 * 2)
    assert f32_bytes == 1879048192
    assert 2 * layers * q8_plane < f32_bytes / 3


def test_config_pack_layout():
    c = cfgmod.qwen3_asr_0p6b()
    b = c.pack()
    assert len(b) == 160 and b[:8] == b"QWCFG001"
    # model_config.zig:366-375 offsets
    assert struct.unpack_from("<I", b, 8)[0] == 1
    assert struct.unpack_from("<I", b, 16)[0] == c.audio_d_model
    assert struct.unpack_from("<I", b, 60)[0] == c.text_hidden_size
    assert struct.unpack_from("<I", b, 104)[0] == c.token_audio_start
    assert struct.unpack_from("<I", b, 144)[0] == c.flags
    assert cfgmod.Config.unpack(b).pack() == b
    big = cfgmod.qwen3_asr_1p7b()
    assert big.text_hidden_size == 2048 and big.text_ffn_dim == 6144 and big.q_width == 2048


def _declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(qwc_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(cuda_lib):
    declared = _declared_symbols()
    assert len(declared) >= 30
    for name in declared:
        assert hasattr(cuda_lib, name), name
        assert name in rt.SIGNATURES, f"{name} has no binding"
    assert set(rt.SIGNATURES) == set(declared)


def test_host_only_calls(cuda_lib):
    assert cuda_lib.qwc_abi_version() == 0x00010000  # abi.zig:439-442
    assert cuda_lib.qwc_features() & rt.FEATURE_MODEL and cuda_lib.qwc_features() & rt.FEATURE_DECODE
    for code, name in rt.STATUS.items():
        assert cuda_lib.qwc_status_message(code).decode().replace(" ", "_").startswith(name.split("_")[0])
    assert cuda_lib.qwc_status_message(-99) == b"unknown status"


def test_operators_refuse_misaligned_pointers(cuda_lib):
    # The checks run before any CUDA call, so fake device addresses are safe
    # here: a pointer the GEMV's vector loads would fault on is refused.
    A = 1 << 20  # an address aligned to everything the operators ask for
    out = A + 4096
    gemv = cuda_lib.qwc_op_gemv
    bad = rt.STATUS_CODE["invalid_argument"]
    for fmt in (quant.Q4, quant.Q8):
        assert gemv(fmt, A, A + 8, 4, 1024, A, out, None) == bad      # codes 8-byte aligned only
        assert gemv(fmt, A, A, 4, 1024, A + 4, out, None) == bad      # x 4-byte aligned only
        assert gemv(fmt, A + 1, A, 4, 1024, A, out, None) == bad      # scales odd
    assert gemv(quant.Q5, A, A + 4, 4, 1024, A, out, None) == bad     # q5 codes need 8 bytes
    assert gemv(quant.Q5, A, A, 4, 1024, A + 2, out, None) == bad     # q5 x needs 4 bytes
    assert cuda_lib.qwc_op_dequantize(quant.Q4, A + 1, A, 4, 1024, out, None) == bad
    assert gemv(quant.Q4, A, A, 4, 100, A, out, None) == rt.STATUS_CODE["shape_mismatch"]  # cols not whole groups
    assert gemv(7, A, A, 4, 1024, A, out, None) == rt.STATUS_CODE["unsupported"]


def test_tensor_descriptor_refuses_bad_handles(cuda_lib):
    # A handle needs a device; without one the lookup fails before anything else.
    import ctypes

    buf = (ctypes.c_uint8 * 64)()
    bad = rt.STATUS_CODE["invalid_argument"]
    assert cuda_lib.qwc_model_tensor_descriptor(0, 0, ctypes.addressof(buf)) == bad
    assert cuda_lib.qwc_model_tensor_descriptor(12345, 0, None) == bad


def test_rope_tables_match_oracle_bit_for_bit(cuda_lib, oracle_lib):
    # kernels.zig:534-564: the tables the CUDA backend uploads equal the oracle's.
    cos_p, sin_p = rt.rope_tables(1000000.0, 128, 4096)
    cos_o, sin_o = O.rope_tables(64, 1000000.0, 4096)
    assert np.array_equal(cos_p.view(np.uint32), cos_o.view(np.uint32))
    assert np.array_equal(sin_p.view(np.uint32), sin_o.view(np.uint32))


def test_header_constants_match_reference():
    text = open(HEADER).read()

    def const(name):
        return int(re.search(rf"\b{name}\s*=\s*(-?\d+)", text).group(1))

    # abi.zig:50-84
    expected_status = {"QWC_OK": 0, "QWC_INVALID_ARGUMENT": -1, "QWC_OUT_OF_MEMORY": -2, "QWC_UNSUPPORTED": -3,
                       "QWC_BAD_MAGIC": -4, "QWC_BAD_VERSION": -5, "QWC_CHECKSUM_MISMATCH": -6,
                       "QWC_SHAPE_MISMATCH": -7, "QWC_INVALID_STATE": -8, "QWC_LIMIT_EXCEEDED": -9,
                       "QWC_NOT_FOUND": -10, "QWC_TRUNCATED": -11, "QWC_INVALID_ENCODING": -12,
                       "QWC_UNSUPPORTED_MODEL": -13, "QWC_AUDIO_TOO_LONG": -14}
    for k, v in expected_status.items():
        assert const(k) == v, k
    # dtype.zig:17-24, container.zig:333-376
    assert (const("QWC_FORMAT_Q4"), const("QWC_FORMAT_Q5"), const("QWC_FORMAT_Q8")) == (16, 17, 18)
    assert const("QWC_KIND_DECODER_EMBED_TOKENS") == 30 and const("QWC_KIND_DECODER_DOWN") == 43
    # quant constants used by the kernels (quant.zig:49-59)
    internal = open(os.path.join(ROOT, "qwenscriber_b200", "csrc", "qwc_internal.h")).read()
    assert re.search(r"kGroup = 64;", internal)
    assert ("return format == kFormatQ4 ? 32u : format == kFormatQ5 ? 40u : (format == kFormatQ8 ? 64u : 0u);"
            in internal)
    assert re.search(r"kFormatQ5 = 17;", internal)


def test_qwc_create_without_device_returns_zero(cuda_lib):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a device is present")
    assert cuda_lib.qwc_create(0) == 0


def test_synthetic_prompt_shapes():
    c = cfgmod.qwen3_asr_0p6b()
    p = synthetic.make_prompt(c, 188, 8, seed=0)
    assert p.tokens.shape == (196,) and p.audio.shape == (188, 1024)
    assert np.all(p.tokens[:188] == c.token_audio_pad) and not np.any(p.tokens[188:] == c.token_audio_pad)
    assert p.tokens.max() < c.vocab_size

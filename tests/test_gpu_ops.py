"""Per-operator parity of the CUDA kernels against the CPU oracle, through the C ABI.

Device memory comes from torch (plumbing only); every compute call goes
through libqwenscriber_cuda's `qwc_op_*` entry points. Tolerances are the
reference's own CPU-vs-GPU bounds (tests/gpu/harness.mjs:54-104): dequant and
quantize bit exact, matmul atol 1e-3 / rtol 1e-4, rmsnorm 1e-4, rope
atol 2e-3 / rtol 1e-3, attention 1e-4, silu_mul 1e-5, argmax exact.
"""

import numpy as np
import pytest

import oracle as O
from qwenscriber_b200 import quant
from qwenscriber_b200 import runtime as rt

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _call(name, *args):
    st = getattr(rt.lib(), name)(*args)
    assert st == 0, f"{name} -> {rt.STATUS.get(st, st)}"


def _random_planes(rng, fmt, rows, cols):
    groups = cols // 64
    scales = (np.abs(rng.standard_normal((rows, groups))) * 0.01).astype(np.float16).view(np.uint16)
    scales[0, 0] = 0x0001  # subnormal f16 scale (harness.mjs:99-103)
    scales[1, 1] = 0
    codes = rng.integers(0, 256, size=(rows, groups * quant.DATA_BYTES[fmt]), dtype=np.uint8)
    return scales, codes


@pytest.mark.parametrize("fmt", [quant.Q4, quant.Q5, quant.Q8])
def test_dequantize_is_bit_exact(gpu, cuda_lib, oracle_lib, fmt):
    import torch

    rng = np.random.default_rng(1)
    rows, cols = 257, 2048
    scales, codes = _random_planes(rng, fmt, rows, cols)
    out = torch.zeros(rows * cols, dtype=torch.float32, device=gpu)
    ds, dc = _dev(torch, scales), _dev(torch, codes)
    _call("qwc_op_dequantize", fmt, ds.data_ptr(), dc.data_ptr(), rows, cols, out.data_ptr(), None)
    torch.cuda.synchronize()
    expected = O.dequantize_rows(fmt, scales.view(np.uint8).reshape(rows, -1), codes, cols)
    got = out.cpu().numpy().reshape(rows, cols)
    assert np.array_equal(got.view(np.uint32), expected.view(np.uint32))


def test_quantize_q8_is_bit_exact(gpu, cuda_lib, oracle_lib):
    import torch

    rng = np.random.default_rng(2)
    rows, cols = 300, 1024
    v = (rng.standard_normal((rows, cols)) * rng.choice([1e-4, 0.03, 1.0, 77.0], size=(rows, 1))).astype(np.float32)
    v[0, :64] = 0.0                                   # zero group -> scale 0, code 128
    v[1, :64] = np.arange(64, dtype=np.float32) - 31.5  # halves land on ties
    v[2, 3] = 1e-38
    ds = torch.zeros(rows * cols // 64 * 2, dtype=torch.uint8, device=gpu)
    dc = torch.zeros(rows * cols, dtype=torch.uint8, device=gpu)
    dv = _dev(torch, v)
    _call("qwc_op_quantize_q8", dv.data_ptr(), rows, cols, ds.data_ptr(), dc.data_ptr(), None)
    torch.cuda.synchronize()
    es, ec = O.quantize_rows(O.Q8, v)
    assert np.array_equal(ds.cpu().numpy().reshape(es.shape), es)
    assert np.array_equal(dc.cpu().numpy().reshape(ec.shape), ec)


@pytest.mark.parametrize("fmt,cols", [(quant.Q4, 1024), (quant.Q4, 2048), (quant.Q4, 3072), (quant.Q4, 6144),
                                      (quant.Q8, 1024), (quant.Q8, 3072),
                                      (quant.Q5, 128), (quant.Q5, 1024), (quant.Q5, 2048), (quant.Q5, 6144)])
def test_gemv_matches_linear_quantized(gpu, cuda_lib, oracle_lib, fmt, cols):
    import torch

    rng = np.random.default_rng(cols + fmt)
    rows = 389
    scales, codes = _random_planes(rng, fmt, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    out = torch.zeros(rows, dtype=torch.float32, device=gpu)
    ds, dc, dx = _dev(torch, scales), _dev(torch, codes), _dev(torch, x)
    _call("qwc_op_gemv", fmt, ds.data_ptr(), dc.data_ptr(), rows, cols, dx.data_ptr(), out.data_ptr(), None)
    torch.cuda.synchronize()
    expected = O.linear_quantized(fmt, scales.view(np.uint8).reshape(rows, -1), codes, x)[0]
    got = out.cpu().numpy()
    np.testing.assert_allclose(got, expected, atol=1e-3, rtol=1e-4)


def test_attention_q8_matches_oracle(gpu, cuda_lib, oracle_lib):
    import torch

    rng = np.random.default_rng(4)
    heads, kvh, hd, cached = 16, 8, 128, 301
    kvw = kvh * hd
    keys = rng.standard_normal((cached, kvw)).astype(np.float32)
    values = rng.standard_normal((cached, kvw)).astype(np.float32)
    q = (rng.standard_normal(heads * hd) * 0.3).astype(np.float32)
    ks, kc = O.quantize_rows(O.Q8, keys)
    vs, vc = O.quantize_rows(O.Q8, values)
    expected = O.decode_attention_q8(q, ks, kc, vs, vc, cached, heads, kvh, hd)
    out = torch.zeros(heads * hd, dtype=torch.float32, device=gpu)
    t = [_dev(torch, a) for a in (q, ks, kc, vs, vc)]
    _call("qwc_op_attention_q8", *[a.data_ptr() for a in t], cached, heads, kvh, hd, out.data_ptr(), None)
    torch.cuda.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), expected, atol=1e-4, rtol=1e-4)


def test_argmax_first_index_of_maximum(gpu, cuda_lib):
    import torch

    from tests.test_oracle_kat import harness_random_vector

    v = harness_random_vector(1000, 0x5EED0014)
    v[777] = 4.0
    v[333] = 4.0
    out = torch.zeros(1, dtype=torch.int32, device=gpu)
    dv = _dev(torch, v)
    _call("qwc_op_argmax", dv.data_ptr(), v.size, out.data_ptr(), None)
    torch.cuda.synchronize()
    assert int(out.item()) == 333
    rng = np.random.default_rng(9)
    big = rng.standard_normal(151936).astype(np.float32)
    big[100000] = big[5] = 10.0
    dv = _dev(torch, big)
    _call("qwc_op_argmax", dv.data_ptr(), big.size, out.data_ptr(), None)
    torch.cuda.synchronize()
    assert int(out.item()) == 5 == O.argmax(big)


def test_argmax_nan_and_infinity_follow_the_reference(gpu, cuda_lib, oracle_lib):
    """decoder.zig:290-301 seeds the maximum with values[0] and replaces it on
    a strict `>` only: a NaN at index 0 is the answer, a NaN elsewhere never
    wins, and rows of equal infinities give their first index. Both argmax
    entry points, against the oracle's sequential scan."""
    import torch

    rng = np.random.default_rng(31)
    n = 151936
    cases = []
    v = rng.standard_normal(n).astype(np.float32)
    v[0] = np.nan
    v[9] = 50.0
    cases.append(v)  # NaN at index 0 -> 0
    v = rng.standard_normal(n).astype(np.float32)
    v[[3, 70000, 150000]] = np.nan
    v[12345] = 20.0
    cases.append(v)  # NaNs elsewhere are skipped
    cases.append(np.full(n, np.inf, np.float32))  # all +inf -> 0
    cases.append(np.full(n, -np.inf, np.float32))  # all -inf -> 0
    v = np.full(n, -np.inf, np.float32)
    v[99999] = np.inf
    v[140000] = np.inf
    cases.append(v)  # first +inf
    v = np.full(n, np.nan, np.float32)
    cases.append(v)  # all NaN -> 0
    v = np.full(n, np.nan, np.float32)
    v[0] = -np.inf
    cases.append(v)  # -inf then NaNs -> 0
    v = np.full(n, np.nan, np.float32)
    v[77] = 1.0
    v[0] = 0.5
    cases.append(v)  # finite values among NaNs
    out = torch.zeros(1, dtype=torch.int32, device=gpu)
    for v in cases:
        expected = O.argmax(v)
        dv = _dev(torch, v)
        for name in ("qwc_op_argmax", "qwc_op_argmax_noalloc"):
            out.zero_()
            _call(name, dv.data_ptr(), v.size, out.data_ptr(), None)
            torch.cuda.synchronize()
            assert int(out.item()) == expected, (name, expected, int(out.item()))


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_rmsnorm_rope_silu_bit_exact(gpu, cuda_lib, oracle_lib):
    """The per-operator kernels follow the reference's own order (sequential
    sum of squares, each product rounded, exp as the host expf), so they equal
    the oracle bit for bit rather than within the harness tolerances."""
    import torch

    rng = np.random.default_rng(5)
    x = (rng.standard_normal((3, 2048)) * 3).astype(np.float32)
    w = rng.standard_normal(2048).astype(np.float32)
    out = torch.zeros(3 * 2048, dtype=torch.float32, device=gpu)
    dx, dw = _dev(torch, x), _dev(torch, w)
    _call("qwc_op_rmsnorm", dx.data_ptr(), dw.data_ptr(), 2048, 3, 1e-6, out.data_ptr(), None)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out.cpu().numpy()), _bits(O.rmsnorm(x, w, 2048, 1e-6).reshape(-1)))

    cos, sin = rt.rope_tables(1000000.0, 128, 512)
    q = rng.standard_normal(16 * 128).astype(np.float32)
    dq, dc, ds = _dev(torch, q), _dev(torch, cos), _dev(torch, sin)
    _call("qwc_op_rope", dq.data_ptr(), 16, 128, dc.data_ptr(), ds.data_ptr(), 437, None)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(dq.cpu().numpy()), _bits(O.rope(q, [437], 16, 128, cos, sin)))

    # silu over the whole f32 range exp meets: every 1021st bit pattern of
    # [-110, 110] plus the edges of its overflow and underflow branches.
    lo = np.frombuffer(np.float32(-110.0).tobytes(), np.uint32)[0]
    hi = np.frombuffer(np.float32(110.0).tobytes(), np.uint32)[0]
    pos = np.arange(0, hi, 1021, dtype=np.uint32).view(np.float32)
    neg = np.arange(0x80000000, lo, 1021, dtype=np.uint32).view(np.float32)
    edges = np.array([0.0, -0.0, 88.0, -88.0, 88.72283, -88.72283, 103.97, -103.97, 103.28, -103.28, 1e-30, -1e-30,
                      np.inf, -np.inf], np.float32)
    g = np.concatenate([pos, neg, edges]).astype(np.float32)
    u = rng.standard_normal(g.size).astype(np.float32)
    o = torch.zeros(g.size, dtype=torch.float32, device=gpu)
    dg, du = _dev(torch, g), _dev(torch, u)
    _call("qwc_op_silu_mul", dg.data_ptr(), du.data_ptr(), g.size, o.data_ptr(), None)
    torch.cuda.synchronize()
    got, want = o.cpu().numpy(), O.silu_mul(g, u)
    same = (_bits(got) == _bits(want)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), (g[~same][:5], got[~same][:5], want[~same][:5], int((~same).sum()))

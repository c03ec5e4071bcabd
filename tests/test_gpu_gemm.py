"""The tensor-core stream GEMM (qwc_op_gemm_streams) against exact references.

The kernel feeds each dequantized weight as an exact f16 pair (hi + lo) and
each activation as f16 hi + lo, so the first check is against the f64
product of the exact weights with those 22-bit activations, where only the
f32 accumulation order differs (relative 1e-5 of sum |w x|). The second
check compares with the reference's f32 linearQuantized (kernels.zig:118-158,
the oracle) at the same bound.
"""

import numpy as np
import pytest

import oracle as O
from qwenscriber_b200 import quant
from qwenscriber_b200 import runtime as rt

pytestmark = pytest.mark.gpu


def _planes(rng, fmt, rows, cols):
    groups = cols // 64
    scales = (np.abs(rng.standard_normal((rows, groups))) * 0.003 + 1e-4).astype(np.float16)
    scales[0, 0] = np.float16(0.0)
    codes = rng.integers(0, 256, size=(rows, groups * quant.DATA_BYTES[fmt]), dtype=np.uint8)
    return scales, codes


def _weights(fmt, scales, codes):
    rows = codes.shape[0]
    if fmt == quant.Q4:
        lo = (codes & 0x0F).astype(np.int32)
        hi = (codes >> 4).astype(np.int32)
        q = np.empty((rows, codes.shape[1] * 2), np.int32)
        q[:, 0::2], q[:, 1::2] = lo, hi
        q -= 8
    elif fmt == quant.Q5:
        q = quant.unpack_q5(codes, codes.shape[1] // 40 * 64) - 16
    else:
        q = codes.astype(np.int32) - 128
    s = np.repeat(scales.astype(np.float32), 64, axis=1)
    return q.astype(np.float32) * s  # exact: a <= 8-bit integer times an f16


@pytest.mark.parametrize("fmt,rows,cols,streams", [
    (quant.Q4, 256, 1024, 64), (quant.Q4, 300, 2048, 7), (quant.Q8, 384, 2048, 64),
    (quant.Q4, 128, 6144, 64), (quant.Q8, 200, 1024, 33), (quant.Q5, 256, 1024, 64), (quant.Q5, 300, 2048, 19)])
def test_gemm_streams(gpu, cuda_lib, oracle_lib, fmt, rows, cols, streams):
    import torch

    rng = np.random.default_rng(rows * 7 + cols + streams)
    scales, codes = _planes(rng, fmt, rows, cols)
    x = rng.standard_normal((streams, cols)).astype(np.float32)
    ds = torch.from_numpy(scales.view(np.uint16).copy()).cuda()
    dc = torch.from_numpy(codes).cuda()
    dx = torch.from_numpy(x).cuda()
    out = torch.zeros((streams, rows), dtype=torch.float32, device=gpu)
    st = cuda_lib.qwc_op_gemm_streams(fmt, ds.data_ptr(), dc.data_ptr(), rows, cols, dx.data_ptr(), streams,
                                      out.data_ptr(), None)
    torch.cuda.synchronize()
    assert st == 0, rt.STATUS.get(st, st)
    got = out.cpu().numpy()

    w = _weights(fmt, scales, codes).astype(np.float64)
    xh = x.astype(np.float16)
    xl = (x - xh.astype(np.float32)).astype(np.float16)
    x22 = xh.astype(np.float64) + xl.astype(np.float64)
    exact = x22 @ w.T
    mag = np.abs(x22) @ np.abs(w).T
    err = np.abs(got - exact)
    assert np.all(err <= 1e-5 * mag + 1e-30), float(np.max(err / (mag + 1e-30)))

    # Against the reference's f32 path.
    ref = O.linear_quantized(fmt, scales.view(np.uint8), codes, x)
    assert np.all(np.abs(got - ref) <= 1e-5 * mag + 1e-6), float(np.max(np.abs(got - ref) / (mag + 1e-30)))

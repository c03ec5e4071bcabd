"""qwc_op_argmax_noalloc against qwc_op_argmax, both through the C ABI.

The no-allocation variant keeps its block partials in a fixed array compiled
into the library; it must return exactly what the allocating entry point
returns, on consecutive calls (the second call reuses the scratch the first
one wrote), and refuse counts beyond its stated maximum.
"""

import ctypes

import numpy as np
import pytest

from qwenscriber_b200 import runtime as rt

pytestmark = pytest.mark.gpu


def _argmax_both(torch, lib, values, out_ref, out_new):
    dv = torch.from_numpy(np.ascontiguousarray(values)).cuda()
    st_ref = lib.qwc_op_argmax(dv.data_ptr(), values.size, out_ref.data_ptr(), None)
    st_new = lib.qwc_op_argmax_noalloc(dv.data_ptr(), values.size, out_new.data_ptr(), None)
    torch.cuda.synchronize()
    assert st_ref == 0 and st_new == 0, (rt.STATUS.get(st_ref), rt.STATUS.get(st_new))
    return int(out_ref.item()), int(out_new.item())


def test_noalloc_argmax_matches_allocating_argmax_on_consecutive_calls(gpu, cuda_lib):
    import torch

    rng = np.random.default_rng(20261201)
    out_ref = torch.full((1,), -1, dtype=torch.int32, device=gpu)
    out_new = torch.full((1,), -1, dtype=torch.int32, device=gpu)

    # First call: a vocabulary-sized row with a tie; the lowest index must win.
    first = rng.standard_normal(151936).astype(np.float32)
    first[120000] = first[4321] = 9.5
    ref1, new1 = _argmax_both(torch, cuda_lib, first, out_ref, out_new)
    assert ref1 == new1 == 4321

    # Second call in a row, smaller and with its maximum late in the row, so
    # stale partials from the first call would show up as a wrong index.
    second = rng.standard_normal(3000).astype(np.float32)
    second[2999] = 50.0
    ref2, new2 = _argmax_both(torch, cuda_lib, second, out_ref, out_new)
    assert ref2 == new2 == 2999

    # The largest accepted count (every scratch partial in use), then one more value.
    top = rt.ARGMAX_NOALLOC_MAX_COUNT
    big = torch.randn(top, device=gpu, dtype=torch.float32)
    big[top - 7] = 100.0
    st = cuda_lib.qwc_op_argmax_noalloc(big.data_ptr(), top, out_new.data_ptr(), None)
    st_ref = cuda_lib.qwc_op_argmax(big.data_ptr(), top, out_ref.data_ptr(), None)
    torch.cuda.synchronize()
    assert st == 0 and st_ref == 0
    assert int(out_new.item()) == int(out_ref.item()) == top - 7
    too_big = ctypes.c_uint32(top + 1)
    assert cuda_lib.qwc_op_argmax_noalloc(big.data_ptr(), too_big, out_new.data_ptr(), None) == rt.LIMIT_EXCEEDED

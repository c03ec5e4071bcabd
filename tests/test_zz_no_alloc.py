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

    # First call: every one of the 512 partials in use, a tie (the lowest index
    # must win) and the row's maximum in one of the last partials.
    first = rng.standard_normal(512 * 8192 // 4).astype(np.float32)
    first[1000000] = first[900000] = 100.0
    ref1, new1 = _argmax_both(torch, cuda_lib, first, out_ref, out_new)
    assert ref1 == new1 == 900000

    # Second call in a row, with 12 partials and a smaller maximum: a pass
    # that read the first call's partials left in the scratch would return
    # 900000 instead.
    second = rng.standard_normal(3000).astype(np.float32)
    second[2999] = 50.0
    ref2, new2 = _argmax_both(torch, cuda_lib, second, out_ref, out_new)
    assert ref2 == new2 == 2999

    # Third call, as many partials as the first again, maximum near the end.
    third = rng.standard_normal(first.size).astype(np.float32)
    third[first.size - 3] = 60.0
    ref3, new3 = _argmax_both(torch, cuda_lib, third, out_ref, out_new)
    assert ref3 == new3 == first.size - 3

    # The call allocates nothing: device-wide free memory and torch's pool
    # are unchanged across it (its set-up ran in the calls above).
    dv = torch.from_numpy(third).cuda()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    torch_bytes0 = torch.cuda.memory_allocated()
    assert cuda_lib.qwc_op_argmax_noalloc(dv.data_ptr(), third.size, out_new.data_ptr(), None) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0 and torch.cuda.memory_allocated() == torch_bytes0
    assert int(out_new.item()) == first.size - 3

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

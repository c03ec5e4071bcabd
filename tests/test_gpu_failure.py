"""Failure detection without a GPU fault: every device-side wait of the
persistent decode kernel is bounded, and a wait that runs out comes back to
the host as a status code, never a trap or a hang (the reference's contract:
src/wasm/exports.zig:3-6, the error-to-status map of src/wasm/abi.zig:91-147).

QWC_OPTION_TEST_STALL makes the next launch's grid barriers wait for one CTA
more than the launch has: a wait on a count nothing completes, which ends only
when its bound (QWC_OPTION_WAIT_LIMIT_US, here one millisecond) runs out. The
call must return QWC_INVALID_STATE promptly, the following launch must run
normally (the stall is one-shot), and the same handle must then decode the
oracle's greedy chain. Only the single-stream kernel runs with the short bound.
"""

import time

import pytest

from qwenscriber_b200 import quant, synthetic
from qwenscriber_b200 import runtime as rt

from .parity import oracle_model, small_config

pytestmark = pytest.mark.gpu


def test_expired_wait_returns_invalid_state_and_handle_recovers(gpu, cuda_lib, oracle_lib):
    c = small_config(quant.Q8, layers=2, max_positions=256)
    model = synthetic.make_model(c, quant.Q8, seed=13)
    prompt = synthetic.make_prompt(c, 24, 4, seed=13)
    gm = rt.CudaModel(0)
    om = oracle_model(model)
    try:
        synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8)
        gm.set_option(rt.OPTION_IGNORE_EOS, 1)
        gm.set_option(rt.OPTION_STEP_CHUNK, 4)
        gm.decode_begin(prompt.tokens, prompt.audio, 32)  # default bounds: the prefill succeeds
        gm.set_option(rt.OPTION_WAIT_LIMIT_US, 1000)
        gm.set_option(rt.OPTION_TEST_STALL, 1)
        t0 = time.perf_counter()
        with pytest.raises(rt.QwcError) as e:
            gm.decode_step()
        elapsed = time.perf_counter() - t0
        assert e.value.status == rt.STATUS_CODE["invalid_state"]
        assert elapsed < 2.0, elapsed  # the bound, not a hang or the 4 s default
        # One-shot: the next launch, still with the 1 ms bound, runs to completion.
        assert isinstance(gm.decode_step(), int)
        gm.decode_end()

        # The same handle, default bounds again: a fresh session decodes the oracle's chain.
        gm.set_option(rt.OPTION_WAIT_LIMIT_US, 0)
        nxt = om.prefill(prompt.tokens, prompt.audio, prompt.audio.shape[0])
        gm.decode_begin(prompt.tokens, prompt.audio, 12)
        for _ in range(12):
            assert gm.decode_step() == nxt
            nxt = om.step(nxt)
        gm.decode_end()
    finally:
        gm.close()
        om.close()

"""Failure detection without a GPU fault: every device-side wait of the
persistent decode kernel is bounded, and a wait that runs out comes back to
the host as a status code, never a trap or a hang (the reference's contract:
src/wasm/exports.zig:3-6, the error-to-status map of src/wasm/abi.zig:91-147).

QWC_OPTION_WAIT_LIMIT_US bounds the waits at one microsecond, far below the
time a launch's first weight tiles take to arrive from HBM, so the first
bounded wait of the next launch gives up. The call must return
QWC_INVALID_STATE, and the same handle must then decode the oracle's greedy
chain once the default bound is restored. Only the single-stream kernel runs
with the short bound here.
"""

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
        gm.set_option(rt.OPTION_WAIT_LIMIT_US, 1)
        statuses = []
        for _ in range(3):
            try:
                gm.decode_step()
                statuses.append(rt.STATUS_CODE["ok"])
            except rt.QwcError as e:
                statuses.append(e.status)
        assert rt.STATUS_CODE["invalid_state"] in statuses, statuses
        assert all(s in (0, rt.STATUS_CODE["invalid_state"]) for s in statuses), statuses
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

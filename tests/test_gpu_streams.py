"""Parity of the batched multi-stream step (qwc_model_set_streams > 1) against
the CPU oracle, one oracle decoder per slot, through the stream family of the
C ABI.

Every slot has its own prompt (ragged lengths, some spanning several
64-position attention chunks). After each qwc_streams_step, every slot that
emitted a token is compared with its oracle: the logits within the north
star's bounds (2e-2 max-abs, cosine >= 0.9999), the token identical or a
near tie (oracle margin <= 2 x the measured logit error), in which case the
oracle's token is forced so later steps compare on identical inputs.

The batched projections feed exact weights and 22-bit activations to the
tensor cores (documented in the header), so the q8 cache rows are held to the
single-stream path's bound: codes within one, scales within one f16 ulp.
"""

import numpy as np
import pytest

from qwenscriber_b200 import quant, synthetic
from qwenscriber_b200 import runtime as rt

from .parity import cosine, kv_compare, oracle_model, small_config

pytestmark = pytest.mark.gpu

LOGIT_ATOL = 2e-2
COSINE_MIN = 0.9999


def _prompts(config, slots, seed, lengths):
    out = []
    for s in range(slots):
        rows, ids = lengths[s % len(lengths)]
        out.append(synthetic.make_prompt(config, rows, ids, seed, stream=s))
    return out


def _run(model, slots, lengths, tokens_per_slot, max_near_ties, seed=5):
    c = model.config
    prompts = _prompts(c, slots, seed, lengths)
    gm = rt.CudaModel(0)
    oms = []
    try:
        synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8, streams=slots)
        gm.set_option(rt.OPTION_IGNORE_EOS, 1)
        expect, logits = [], []
        for s, p in enumerate(prompts):
            om = oracle_model(model, threads=4)
            oms.append(om)
            expect.append(om.prefill(p.tokens, p.audio, p.audio.shape[0]))
            logits.append(om.logits(c.vocab_size))
            gm.stream_begin(s, p.tokens, p.audio, tokens_per_slot)
        emitted = [0] * slots
        worst_abs, worst_cos, ties = 0.0, 1.0, []
        for _ in range(max(len(p.tokens) for p in prompts) + tokens_per_slot + 2):
            toks, res, _ = gm.streams_step(slots)
            for s in range(slots):
                if res[s] != 1:
                    assert res[s] in (0, 2), res[s]
                    continue
                lg = gm.debug_logits(s)
                lo = logits[s]
                err = float(np.max(np.abs(lo - lg)))
                worst_abs = max(worst_abs, err)
                worst_cos = min(worst_cos, cosine(lo, lg))
                tok = int(toks[s])
                if tok != expect[s]:
                    ties.append({"slot": s, "step": emitted[s], "oracle": expect[s], "gpu": tok,
                                 "margin": float(lo[expect[s]] - lo[tok]), "logit_err": err})
                    assert lo[expect[s]] - lo[tok] <= 2 * err
                    gm.debug_hold(force=expect[s], slot=s)
                emitted[s] += 1
                if emitted[s] < tokens_per_slot:
                    expect[s] = oms[s].step(expect[s])
                    logits[s] = oms[s].logits(c.vocab_size)
            if all(e >= tokens_per_slot for e in emitted):
                break
        print(f"streams parity: {slots} slots, max |dlogit| {worst_abs:.3e}, min cosine {worst_cos:.9f}, "
              f"near ties {len(ties)} {ties[:4]}")
        assert all(e == tokens_per_slot for e in emitted), emitted
        assert worst_abs <= LOGIT_ATOL, worst_abs
        assert worst_cos >= COSINE_MIN, worst_cos
        assert len(ties) <= max_near_ties, ties
        # The q8 cache rows of a few slots against their oracles.
        for s in range(min(slots, 3)):
            ok_, ov = oms[s].cache_q8()
            for which, ora in ((0, ok_), (1, ov)):
                r = kv_compare(gm.debug_cache(which, ora.size, slot=s), ora, c, oms[s].position)
                print(f"slot {s} kv {'kv'[which]}: {r}")
                assert r["codes_max"] <= 1 and r["scale_ulps_max"] <= 1, r
                assert r["codes_exact"] >= 0.99 and r["scales_exact"] >= 0.95, r
        return gm, prompts
    finally:
        gm.close()
        for om in oms:
            om.close()


@pytest.mark.parametrize("fmt", [quant.Q8, quant.Q4])
def test_streams_match_oracle(gpu, cuda_lib, oracle_lib, fmt):
    config = small_config(fmt, layers=2, vocab=8192, max_positions=512)
    model = synthetic.make_model(config, fmt, seed=21)
    _run(model, slots=6, lengths=[(10, 4), (60, 8), (3, 2), (120, 10), (0, 5), (70, 1)], tokens_per_slot=12,
         max_near_ties=3)


def test_sixty_four_streams(gpu, cuda_lib, oracle_lib):
    config = small_config(quant.Q4, layers=2, vocab=8192, max_positions=256)
    model = synthetic.make_model(config, quant.Q4, seed=22)
    _run(model, slots=64, lengths=[(5, 3), (20, 4), (1, 2), (66, 3)], tokens_per_slot=4, max_near_ties=6)


def test_device_chained_steps_match_host_steps(gpu, cuda_lib, oracle_lib):
    """qwc_streams_run_timed (greedy chain on the device) emits the same tokens
    as host-driven qwc_streams_step calls from the same state."""
    config = small_config(quant.Q4, layers=2, vocab=8192, max_positions=256)
    model = synthetic.make_model(config, quant.Q4, seed=23)
    prompts = _prompts(config, 5, 9, [(8, 3), (30, 2), (2, 6)])
    runs = []
    for timed in (False, True):
        gm = rt.CudaModel(0)
        synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8, streams=5)
        gm.set_option(rt.OPTION_IGNORE_EOS, 1)
        for s, p in enumerate(prompts):
            gm.stream_begin(s, p.tokens, p.audio, 64)
        while True:  # consume every prompt; each slot then holds its first token
            _, res, _ = gm.streams_step(5)
            if not np.any(res == 2):
                break
        # Align: every slot has emitted exactly one token once all prompts are done.
        while min(len(gm.stream_tokens(s)) for s in range(5)) < 2:
            gm.streams_step(5)
        base = [len(gm.stream_tokens(s)) for s in range(5)]
        if timed:
            ms = gm.streams_run_timed(8)
            assert ms > 0
        else:
            for _ in range(8):
                gm.streams_step(5)
        runs.append([gm.stream_tokens(s)[base[s]:base[s] + 8] for s in range(5)])
        gm.close()
    assert runs[0] == runs[1]

"""Model loading through `.qw` shards (qwc_model_add_shard) on the GPU.

The same synthetic model is loaded twice, once as shards (the reference's
qw_model_add_shard path, src/wasm/model.zig:156-178) and once tensor by
tensor; both handles must decode the same greedy tokens with bit-identical
logits, because the device holds the same bytes either way. The model
family's refusals for shards follow the reference: a repeated shard, a
tensor added twice, and a call outside the ready state.
"""

import numpy as np
import pytest

from qwenscriber_b200 import quant, shard, synthetic
from qwenscriber_b200 import runtime as rt

from .parity import small_config

pytestmark = pytest.mark.gpu

CODE = {name: code for code, name in rt.STATUS.items()}


def _decode(gm, prompt, steps):
    gm.set_option(rt.OPTION_KEEP_LOGITS, 1)
    gm.set_option(rt.OPTION_IGNORE_EOS, 1)
    gm.decode_begin(prompt.tokens, prompt.audio, steps + 1)
    tokens, logits = [], [gm.debug_logits()]
    for _ in range(steps):
        tokens.append(gm.decode_step())
        logits.append(gm.debug_logits())
    return tokens, logits


@pytest.mark.parametrize("fmt", [quant.Q8, quant.Q4, quant.Q5])
def test_shards_load_the_same_model_as_tensors(gpu, cuda_lib, fmt):
    config = small_config(fmt, layers=3)
    model = synthetic.make_model(config, fmt, seed=17)
    prompt = synthetic.make_prompt(config, 12, 4, seed=17)
    parts = shard.write_model_shards(model, shards=3)

    a = rt.CudaModel(0)
    b = rt.CudaModel(0)
    try:
        a.begin()
        for p in parts:
            a.add_shard(p)
        a.set_cache_format(rt.CACHE_Q8)
        a.finish(config.pack())
        synthetic.load_into(model, b, cache_format=rt.CACHE_Q8)
        ta, la = _decode(a, prompt, 8)
        tb, lb = _decode(b, prompt, 8)
        assert ta == tb
        for x, y in zip(la, lb):
            assert np.array_equal(x, y)
    finally:
        a.close()
        b.close()


def test_shard_refusals(gpu, cuda_lib):
    config = small_config(quant.Q8, layers=2)
    model = synthetic.make_model(config, quant.Q8, seed=3)
    parts = shard.write_model_shards(model, shards=2)
    gm = rt.CudaModel(0)
    try:
        with pytest.raises(rt.QwcError) as e:
            gm.add_shard(parts[0])  # idle: no qwc_model_begin yet
        assert e.value.status == CODE["invalid_state"]
        gm.begin()
        gm.add_shard(parts[0])
        with pytest.raises(rt.QwcError) as e:
            gm.add_shard(parts[0])  # the same payload again (DuplicateShard)
        assert e.value.status == CODE["invalid_argument"]
        # A shard that repeats one tensor of the first (DuplicateTensor) is
        # refused whole: the handle keeps only the first shard's tensors.
        t = next(t for t in model.tensors if t.layer == 1 and t.kind == synthetic.Q)
        with pytest.raises(rt.QwcError) as e:
            gm.add_shard(shard.build([shard.tensor_entry(t)]))
        assert e.value.status == CODE["invalid_argument"]
        # A decoder matrix in f16 (valid container, no kernel for it).
        f16 = shard.build([(synthetic.Q, 9, 1, (64, 64), bytes(64 * 64 * 2))])
        with pytest.raises(rt.QwcError) as e:
            gm.add_shard(f16)
        assert e.value.status == CODE["unsupported_model"]
        gm.add_shard(parts[1])
        gm.set_cache_format(rt.CACHE_Q8)
        gm.finish(config.pack())
        assert gm.tensor_count() == len(model.tensors)
    finally:
        gm.close()

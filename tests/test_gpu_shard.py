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

from .parity import audio_config, small_config

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


def _index(shard_bytes: bytes, shard_index: int) -> list[dict]:
    """The descriptors src/wasm/model.zig:281-319 reports for one shard: its
    entries in index order, offsets absolute within the shard's bytes."""
    import struct

    _, _, index_len, payload_offset, _, count, _ = struct.unpack_from("<8sIIIIII", shard_bytes, 0)
    out = []
    for i in range(count):
        kind, layer, fmt, rank, _, d0, d1, d2, d3, off, length = struct.unpack_from("<HHBBH4IQQ", shard_bytes,
                                                                                    32 + 40 * i)
        out.append({"offset_bytes": payload_offset + off, "len_bytes": length, "kind": kind, "layer": layer,
                    "format": fmt, "rank": rank, "dims": (d0, d1, d2, d3), "shard_index": shard_index})
    return out


def test_tensor_descriptors_enumerate_every_shard_entry(gpu, cuda_lib):
    """qw_model_tensor_count/descriptor over shards that also hold the audio
    tower and projector (rank-4 f16 convolutions, biases, norms, matrices of
    audio layers 1024+), and over a model added tensor by tensor."""
    config = audio_config(quant.Q4)
    model = synthetic.make_model(config, quant.Q4, seed=29, audio=True)
    first = [shard.tensor_entry(t) for t in model.tensors if t.layer <= 1 or t.layer >= 1024]
    second = [shard.tensor_entry(t) for t in model.tensors if t.layer == 2]
    parts = [shard.build(first), shard.build(second)]
    expected = _index(parts[0], 0) + _index(parts[1], 1)
    assert len(expected) == len(model.tensors)
    assert any(e["rank"] == 4 and e["format"] == quant.F16 for e in expected)
    a = rt.CudaModel(0)
    b = rt.CudaModel(0)
    try:
        a.begin()
        for p in parts:
            a.add_shard(p)
        a.set_cache_format(rt.CACHE_Q8)
        a.finish(config.pack())
        assert a.tensor_count() == len(expected)
        for i, want in enumerate(expected):
            assert a.tensor_descriptor(i) == want, i
        with pytest.raises(rt.QwcError) as e:
            a.tensor_descriptor(len(expected))
        assert e.value.status == CODE["not_found"]

        synthetic.load_into(model, b, cache_format=rt.CACHE_Q8)
        assert b.tensor_count() == len(model.tensors)
        for i, t in enumerate(model.tensors):
            d = b.tensor_descriptor(i)
            vec = t.fmt == quant.F32 and t.rows == 1  # added alone, a convolution is described as rows x in*9
            assert d == {"offset_bytes": 0, "len_bytes": t.payload.nbytes, "kind": t.kind, "layer": t.layer,
                         "format": t.fmt, "rank": 1 if vec else 2,
                         "dims": (t.cols, 1, 1, 1) if vec else (t.rows, t.cols, 1, 1), "shard_index": 0xFFFFFFFF}, i

        # The shard-loaded handle decodes and projects audio like the tensor-loaded one.
        prompt = synthetic.make_prompt(config, 10, 3, seed=29)
        ta, la = _decode(a, prompt, 4)
        tb, lb = _decode(b, prompt, 4)
        assert ta == tb and all(np.array_equal(x, y) for x, y in zip(la, lb))
        mel = synthetic.make_log_mel(config, 260, seed=29)
        assert np.array_equal(a.audio_project(mel, config.audio_output_dim),
                              b.audio_project(mel, config.audio_output_dim))
    finally:
        a.close()
        b.close()

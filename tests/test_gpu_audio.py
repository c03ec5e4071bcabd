"""The audio tower and projector on the GPU (qwc_audio_project,
qwc_decode_begin_features) against the CPU restatement of Model.projectAudio
(oracle/qw_oracle_audio.cpp; src/core/qwen3_asr/model.zig:445-744), stage
by stage as the reference's own bring-up compares them (encodeConvStage,
encodeTowerStage, projectSteps: model.zig:462-499).

Tolerances: the first convolution and GELU are the reference's arithmetic,
but convolutions 2 and 3 and every projection run on the tensor cores with
22-bit activations (f16 hi + lo) and another summation order, and the
LayerNorm and attention reductions are trees. Each stage is compared by its
largest absolute difference relative to the stage's largest magnitude
(`rel`) and by cosine similarity.
"""

import numpy as np
import pytest

from qwenscriber_b200 import quant, synthetic
from qwenscriber_b200 import runtime as rt

from .parity import audio_config, cosine, oracle_audio, oracle_model, small_config

pytestmark = pytest.mark.gpu

REL_SMALL = 2e-5   # 2-layer towers
REL_DEEP = 2e-4    # the released 18-layer geometry


def rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _load(model, streams=None):
    gm = rt.CudaModel(0)
    synthetic.load_into(model, gm, cache_format=rt.CACHE_Q8, streams=streams)
    return gm


def test_audio_config_is_the_reference_geometry(gpu, cuda_lib):
    """qw_model_audio_config's derived values (model_config.zig:417-433 known answers)."""
    for big, d, layers, heads, ffn in ((False, 896, 18, 14, 3584), (True, 1024, 24, 16, 4096)):
        c = small_config(quant.Q4, layers=1, vocab=4096, max_positions=256, big=big)
        model = synthetic.make_model(c, quant.Q4, seed=1)
        gm = _load(model)
        try:
            a = gm.audio_config()
            assert (a["d_model"], a["layers"], a["attention_heads"], a["ffn_dim"]) == (d, layers, heads, ffn)
            assert a["head_dim"] == 64 and a["chunk_frames"] == 100 and a["frequency_bins"] == 16
            assert a["conv_out_input_features"] == 7680 and a["chunk_steps"] == 13 and a["mel_bins"] == 128
            assert a["n_window"] == 50 and a["n_window_infer"] == 800 and a["max_position_steps"] == 13
            assert a["output_dim"] == c.text_hidden_size and a["downsample_hidden_size"] == 480
            assert abs(a["layer_norm_eps"] - 1e-5) < 1e-12 and a["reserved_0"] == a["reserved_1"] == 0
            # This model carries no tower: the audio calls report the missing tensors.
            with pytest.raises(rt.QwcError) as e:
                gm.audio_project(np.zeros((128, 100), np.float32), c.text_hidden_size)
            assert e.value.status == rt.STATUS_CODE["not_found"]
        finally:
            gm.close()


@pytest.mark.parametrize("fmt,frames", [(quant.Q8, 350), (quant.Q4, 1000), (quant.Q5, 260), (quant.Q4, 1)])
def test_tower_stages_match_oracle(gpu, cuda_lib, oracle_lib, fmt, frames):
    """Two-layer towers; 350 and 1000 frames span several attention windows
    (26 steps each here) and a partial last chunk; 1 frame is the shortest clip."""
    c = audio_config(fmt)
    model = synthetic.make_model(c, fmt, seed=41, audio=True)
    mel = synthetic.make_log_mel(c, frames, seed=41)
    oa = oracle_audio(model)
    gm = _load(model)
    try:
        steps = c.packed_steps(frames)
        out = gm.audio_project(mel, c.audio_output_dim)
        assert out.shape == (steps, c.audio_output_dim)
        conv = gm.debug_audio(0, steps, c.audio_d_model)
        tower = gm.debug_audio(1, steps, c.audio_d_model)
        oa.encode_conv(mel)
        ref_conv = oa.encoded(c.audio_d_model)
        oa.encode_tower()
        ref_tower = oa.encoded(c.audio_d_model)
        ref_out = oa.project_steps(c.audio_output_dim)
        r = [rel(conv, ref_conv), rel(tower, ref_tower), rel(out, ref_out)]
        cs = [cosine(conv.ravel(), ref_conv.ravel()), cosine(out.ravel(), ref_out.ravel())]
        print(f"audio {fmt} {frames} frames, {steps} steps: rel conv/tower/out {r}, cosine {cs}")
        assert max(r) <= REL_SMALL, r
        assert min(cs) >= 0.9999999, cs
        # The same clip again: the result does not depend on earlier clips' scratch.
        again = gm.audio_project(mel, c.audio_output_dim)
        assert np.array_equal(again, out)
    finally:
        gm.close()
        oa.close()


def test_released_tower_geometry_matches_oracle(gpu, cuda_lib, oracle_lib):
    """configs' 0.6B tower (18 layers, width 896, 480 convolution channels,
    104-step windows) on a 3.3-second clip (4 chunks, the last partial)."""
    c = small_config(quant.Q4, layers=1, vocab=4096, max_positions=256)
    model = synthetic.make_model(c, quant.Q4, seed=43, audio=True)
    frames = 330
    mel = synthetic.make_log_mel(c, frames, seed=43)
    oa = oracle_audio(model)
    gm = _load(model)
    try:
        out = gm.audio_project(mel, c.audio_output_dim)
        ref = oa.project(mel, c.audio_output_dim)
        tower = gm.debug_audio(1, out.shape[0], c.audio_d_model)
        r = [rel(tower, oa.encoded(c.audio_d_model)), rel(out, ref)]
        print(f"released 0.6B tower, {frames} frames, {out.shape[0]} steps: rel tower/out {r}, "
              f"cosine {cosine(out.ravel(), ref.ravel()):.9f}")
        assert out.shape == ref.shape == (c.packed_steps(frames), c.text_hidden_size)
        assert max(r) <= REL_DEEP, r
    finally:
        gm.close()
        oa.close()


def _audio_prompt(c, steps, text_ids, seed):
    rng = np.random.default_rng([seed, 4])
    ids = rng.integers(0, c.vocab_size - 16, size=text_ids)
    return np.concatenate([[c.token_audio_start], np.full(steps, c.token_audio_pad), [c.token_audio_end],
                           ids]).astype(np.uint32)


@pytest.mark.parametrize("fmt", [quant.Q8, quant.Q4])
def test_decode_begin_features_matches_oracle(gpu, cuda_lib, oracle_lib, fmt):
    """qw_decode_begin's flow (model.zig:370-410): the tower's rows feed the
    prompt's audio placeholders. The oracle projects the same clip and
    prefills its decoder with those rows; the greedy chains are compared
    teacher-forced like the decoder parity tests (a mismatch must be a near
    tie: the oracle's margin within twice the logit error)."""
    c = audio_config(fmt)
    model = synthetic.make_model(c, fmt, seed=47, audio=True)
    frames = 420
    mel = synthetic.make_log_mel(c, frames, seed=47)
    steps = c.packed_steps(frames)
    prompt = _audio_prompt(c, steps, 6, 47)
    oa = oracle_audio(model)
    om = oracle_model(model)
    gm = _load(model)
    try:
        rows = oa.project(mel, c.audio_output_dim)
        nxt = om.prefill(prompt, rows, steps)
        gm.set_option(rt.OPTION_KEEP_LOGITS, 1)
        gm.set_option(rt.OPTION_IGNORE_EOS, 1)
        gm.set_option(rt.OPTION_STEP_CHUNK, 1)
        gm.decode_begin_features(prompt, mel, 12)
        ties = 0
        for _ in range(10):
            lo, lg = om.logits(c.vocab_size), gm.debug_logits()
            err = float(np.max(np.abs(lo - lg)))
            assert err <= 2e-2 and cosine(lo, lg) >= 0.9999
            held = gm.debug_hold()
            if held != nxt:
                assert lo[nxt] - lo[held] <= 2 * err
                ties += 1
                gm.debug_hold(force=nxt)
            assert gm.decode_step() == nxt
            nxt = om.step(nxt)
        assert ties <= 1
        gm.decode_end()
    finally:
        gm.close()
        om.close()
        oa.close()


def test_stream_begin_features_on_a_batched_handle(gpu, cuda_lib, oracle_lib):
    """Two slots of a multi-stream handle begin from two clips; each slot's
    first prediction and the projected rows match a single-stream handle's."""
    c = audio_config(quant.Q8)
    model = synthetic.make_model(c, quant.Q8, seed=53, audio=True)
    mels = [synthetic.make_log_mel(c, f, seed=53, stream=s) for s, f in enumerate((230, 410))]
    prompts = [_audio_prompt(c, c.packed_steps(m.shape[1]), 5, 53 + s) for s, m in enumerate(mels)]
    batched = _load(model, streams=2)
    single = _load(model)
    try:
        for s in range(2):
            batched.stream_begin_features(s, prompts[s], mels[s], 8)
        toks, res, n = batched.streams_step(2)
        assert n == 2 and np.all(res == 1)
        for s in range(2):
            single.decode_begin_features(prompts[s], mels[s], 8)
            assert single.decode_step() == int(toks[s])
            single.decode_end()
    finally:
        batched.close()
        single.close()


def test_audio_refusals(gpu, cuda_lib):
    c = audio_config(quant.Q8)
    model = synthetic.make_model(c, quant.Q8, seed=59, audio=True)
    gm = _load(model)
    code = rt.STATUS_CODE
    try:
        with pytest.raises(rt.QwcError) as e:  # beyond the mel capacity (mel.zig:55-58)
            gm.audio_project(np.zeros((128, 3001), np.float32), c.audio_output_dim)
        assert e.value.status == code["audio_too_long"]
        with pytest.raises(rt.QwcError) as e:  # output buffer too small (CapacityExceeded)
            gm.audio_project(np.zeros((128, 200), np.float32), c.audio_output_dim, capacity=10)
        assert e.value.status == code["limit_exceeded"]
        with pytest.raises(rt.QwcError) as e:  # features not a whole number of mel columns
            gm.decode_begin_features([c.token_audio_pad], np.zeros(127, np.float32), 4)
        assert e.value.status == code["shape_mismatch"]
        with pytest.raises(rt.QwcError) as e:  # one placeholder too few (PromptMismatch)
            steps = c.packed_steps(150)
            gm.decode_begin_features(np.full(steps - 1, c.token_audio_pad, np.uint32),
                                     np.zeros((128, 150), np.float32), 4)
        assert e.value.status == code["shape_mismatch"]
        # The longest clip runs (3000 frames, 390 steps).
        out = gm.audio_project(synthetic.make_log_mel(c, 3000, seed=59), c.audio_output_dim)
        assert out.shape == (390, c.audio_output_dim) and np.all(np.isfinite(out))
    finally:
        gm.close()
    # A tower with one tensor missing fails the load (MissingTensor -> not_found).
    gm = rt.CudaModel(0)
    try:
        gm.begin()
        for t in model.tensors:
            if (t.kind, t.layer) != (synthetic.A_FFN_OUT_B, synthetic.AUDIO_LAYER_BASE + 1):
                gm.add_tensor(t.kind, t.layer, t.fmt, t.rows, t.cols, t.payload)
        gm.set_cache_format(rt.CACHE_Q8)
        with pytest.raises(rt.QwcError) as e:
            gm.finish(c.pack())
        assert e.value.status == code["not_found"]
    finally:
        gm.close()

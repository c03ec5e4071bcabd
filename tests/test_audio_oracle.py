"""The audio-tower restatement composed end to end (oracle/qw_oracle_audio.cpp,
Model.projectAudio: src/core/qwen3_asr/model.zig:445-744) against an
independent float64 numpy restatement of the same model, and the tower's
refusals (missing tensor, wrong shape, clip too long; abi.zig:91-147).

The numpy version follows the reference's definitions, not its rounding:
chunks of 100 mel frames zero-padded, three 3x3 stride-2 convolutions with
GELU, (channel, frequency) flattened per time step through conv_out plus the
sinusoidal row of the step within its chunk, pre-norm blocks with windowed
bidirectional attention and a GELU feed-forward, a final LayerNorm, and the
two-layer projector. Agreement to float32 rounding pins the restatement's
composition; the kernel-level known answers are in test_oracle_audio_kat.py.
"""

import math

import numpy as np
import pytest

import oracle as O
from qwenscriber_b200 import quant, synthetic

from .parity import audio_config, oracle_audio

pytestmark = pytest.mark.usefixtures("oracle_lib")


def _gelu(x):
    return 0.5 * x * (1.0 + np.vectorize(math.erf)(x / math.sqrt(2.0)))


def _conv(x, w, b):
    """x [cin][h][w], w [cout][cin*9] (f16 bits): 3x3, stride 2, padding 1, then GELU."""
    cin, h, wd = x.shape
    wf = w.view(np.float16).astype(np.float64).reshape(w.shape[0], cin, 3, 3)
    xp = np.pad(x, ((0, 0), (1, 1), (1, 1)))
    oh, ow = (h - 1) // 2 + 1, (wd - 1) // 2 + 1
    out = np.zeros((w.shape[0], oh, ow))
    for ky in range(3):
        for kx in range(3):
            patch = xp[:, ky:ky + 2 * oh:2, kx:kx + 2 * ow:2]  # [cin][oh][ow]
            out += np.tensordot(wf[:, :, ky, kx], patch, axes=([1], [0]))
    return _gelu(out + b[:, None, None])


def _layer_norm(x, w, b, eps):
    mu = x.mean(axis=1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * w + b


def _numpy_tower(model, log_mel):
    c = model.config
    t = {(x.kind, x.layer): x for x in model.tensors}

    def mat(kind, layer):
        x = t[(kind, layer)]
        s, codes = quant.split_payload(x.fmt, x.rows, x.cols, x.payload)
        return quant.dequantize(x.fmt, s, codes, x.cols).astype(np.float64)

    def vec(kind, layer):
        return t[(kind, layer)].payload.astype(np.float64)

    cf, cs, d = c.audio_chunk_frames, c.audio_chunk_steps, c.audio_d_model
    frames = log_mel.shape[1]
    rows = []
    for chunk in range((frames + cf - 1) // cf):
        m = np.zeros((c.mel_bins, cf))
        valid = min(frames - chunk * cf, cf)
        m[:, :valid] = log_mel[:, chunk * cf:chunk * cf + valid]
        h = _conv(m[None], t[(synthetic.A_CONV1_W, 0)].payload, vec(synthetic.A_CONV1_B, 0))
        h = _conv(h, t[(synthetic.A_CONV2_W, 0)].payload, vec(synthetic.A_CONV2_B, 0))
        h = _conv(h, t[(synthetic.A_CONV3_W, 0)].payload, vec(synthetic.A_CONV3_B, 0))  # [C][bins][cs]
        w_out = mat(synthetic.A_CONV_OUT_W, 0)
        half = d // 2
        inc = math.log(10000.0) / (half - 1)
        for step in range(min(cs, c.conv_steps(valid))):
            flat = h[:, :, step].reshape(-1)
            ang = step * np.exp(-inc * np.arange(half))
            rows.append(w_out @ flat + np.concatenate([np.sin(ang), np.cos(ang)]))
    x = np.array(rows)
    steps = x.shape[0]
    window = (c.audio_n_window_infer // cf) * cs
    hd = c.audio_head_dim
    for i in range(c.audio_layers):
        L = synthetic.AUDIO_LAYER_BASE + i
        n = _layer_norm(x, vec(synthetic.A_ATTN_NORM_W, L), vec(synthetic.A_ATTN_NORM_B, L), c.audio_layer_norm_eps)
        q = n @ mat(synthetic.A_Q_W, L).T + vec(synthetic.A_Q_B, L)
        k = n @ mat(synthetic.A_K_W, L).T + vec(synthetic.A_K_B, L)
        v = n @ mat(synthetic.A_V_W, L).T + vec(synthetic.A_V_B, L)
        a = np.zeros_like(q)
        for w0 in range(0, steps, window):
            sl = slice(w0, min(w0 + window, steps))
            for h in range(c.audio_attention_heads):
                hs = slice(h * hd, (h + 1) * hd)
                s = q[sl, hs] @ k[sl, hs].T / math.sqrt(hd)
                p = np.exp(s - s.max(axis=1, keepdims=True))
                a[sl, hs] = (p / p.sum(axis=1, keepdims=True)) @ v[sl, hs]
        x = x + a @ mat(synthetic.A_OUT_W, L).T + vec(synthetic.A_OUT_B, L)
        n = _layer_norm(x, vec(synthetic.A_LAYER_NORM_W, L), vec(synthetic.A_LAYER_NORM_B, L), c.audio_layer_norm_eps)
        f = _gelu(n @ mat(synthetic.A_FFN_IN_W, L).T + vec(synthetic.A_FFN_IN_B, L))
        x = x + f @ mat(synthetic.A_FFN_OUT_W, L).T + vec(synthetic.A_FFN_OUT_B, L)
    x = _layer_norm(x, vec(synthetic.A_FINAL_NORM_W, 0), vec(synthetic.A_FINAL_NORM_B, 0), c.audio_layer_norm_eps)
    p = _gelu(x @ mat(synthetic.P_IN_W, 0).T + vec(synthetic.P_IN_B, 0))
    return x, p @ mat(synthetic.P_OUT_W, 0).T + vec(synthetic.P_OUT_B, 0)


@pytest.mark.parametrize("fmt,frames", [(quant.Q8, 350), (quant.Q4, 130), (quant.Q5, 260)])
def test_oracle_tower_matches_float64(fmt, frames):
    c = audio_config(fmt)
    model = synthetic.make_model(c, fmt, seed=31, audio=True)
    mel = synthetic.make_log_mel(c, frames, seed=31)
    oa = oracle_audio(model)
    try:
        assert oa.packed_steps(frames) == c.packed_steps(frames)
        out = oa.project(mel, c.audio_output_dim)
        tower = oa.encoded(c.audio_d_model)
        ref_tower, ref_out = _numpy_tower(model, mel)
        assert out.shape == ref_out.shape == (c.packed_steps(frames), c.text_hidden_size)
        np.testing.assert_allclose(tower, ref_tower, rtol=1e-4, atol=1e-4)
        np.testing.assert_allclose(out, ref_out, rtol=1e-4, atol=2e-4 * np.abs(ref_out).max())
        # Stage by stage (encodeConvStage, encodeTowerStage, projectSteps) equals the whole call.
        oa.encode_conv(mel)
        oa.encode_tower()
        assert np.array_equal(oa.project_steps(c.audio_output_dim), out)
    finally:
        oa.close()


def test_oracle_tower_refusals():
    c = audio_config(quant.Q8)
    model = synthetic.make_model(c, quant.Q8, seed=5, audio=True)
    audio = [t for t in model.tensors if t.kind < synthetic.EMBED]
    # One tensor missing: MissingTensor -> not_found.
    oa = O.OracleAudio(c.pack())
    for t in audio[1:]:
        assert oa.set_tensor(t.kind, t.layer, t.fmt, t.rows, t.cols, t.payload) == 0
    assert oa.finish() == -10
    oa.close()
    # A matrix of the wrong shape: UnexpectedShape -> shape_mismatch.
    oa = O.OracleAudio(c.pack())
    for t in audio:
        rows = t.rows // 2 if t.kind == synthetic.A_Q_W else t.rows
        assert oa.set_tensor(t.kind, t.layer, t.fmt, rows, t.cols, t.payload) == 0
    assert oa.finish() == -7
    oa.close()
    # A clip beyond the mel capacity (3000 frames): audio_too_long.
    oa = oracle_audio(model)
    with pytest.raises(RuntimeError, match="-14"):
        oa.encode_conv(np.zeros((c.mel_bins, 3001), np.float32))
    oa.close()

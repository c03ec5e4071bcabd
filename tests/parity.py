"""Shared helpers for the decoder parity tests: the same synthetic model and
prompt loaded into the CPU oracle and into the CUDA backend."""

from __future__ import annotations

import dataclasses
import os

import numpy as np

import oracle as O
from qwenscriber_b200 import config as cfgmod
from qwenscriber_b200 import quant, synthetic


def small_config(fmt: int, layers: int = 2, vocab: int = 8192, max_positions: int = 512, big: bool = False):
    """Released decoder geometry (0.6B, or 1.7B when `big`) with fewer layers and a smaller vocabulary;
    the special token ids move inside the vocabulary."""
    base = cfgmod.qwen3_asr_1p7b() if big else cfgmod.qwen3_asr_0p6b()
    specials = dict(token_audio_start=vocab - 8, token_audio_end=vocab - 7, token_audio_pad=vocab - 6,
                    token_im_start=vocab - 5, token_im_end=vocab - 4, token_endoftext=vocab - 3,
                    token_asr_text=vocab - 2, token_eos_primary=vocab - 3, token_eos_secondary=vocab - 4,
                    token_pad=vocab - 3)
    return dataclasses.replace(base, text_layers=layers, vocab_size=vocab, max_positions=max_positions,
                               max_decode_tokens=512, **specials)


def oracle_model(model: synthetic.Model, threads: int | None = None) -> O.OracleModel:
    om = O.OracleModel(model.config.pack(), cache_format=1, threads=threads or os.cpu_count() or 8)
    for t in model.tensors:
        if t.kind >= synthetic.EMBED:  # the decoder's tensors; the tower has its own oracle
            om.set_tensor(t.kind, t.layer, t.fmt, t.rows, t.cols, t.payload)
    om.finish()
    return om


def audio_config(fmt: int, layers: int = 2, d_model: int = 128, heads: int = 2, ffn: int = 256, channels: int = 32,
                 n_window_infer: int = 200, text_layers: int = 2):
    """A small tower (2 layers of width 128 by default, 32 convolution channels, attention windows
    of two chunks = 26 packed steps) in front of small_config's decoder."""
    base = small_config(fmt, layers=text_layers)
    return dataclasses.replace(base, audio_d_model=d_model, audio_layers=layers, audio_attention_heads=heads,
                               audio_ffn_dim=ffn, audio_downsample_hidden_size=channels,
                               audio_n_window_infer=n_window_infer)


def oracle_audio(model: synthetic.Model, threads: int | None = None) -> O.OracleAudio:
    oa = O.OracleAudio(model.config.pack(), threads=threads or os.cpu_count() or 8)
    for t in model.tensors:
        if t.kind < synthetic.EMBED:
            st = oa.set_tensor(t.kind, t.layer, t.fmt, t.rows, t.cols, t.payload)
            assert st == 0, (t.kind, t.layer, st)
    st = oa.finish()
    assert st == 0, st
    return oa


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64)
    b = b.astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def kv_compare(gpu_bytes: np.ndarray, oracle_bytes: np.ndarray, config, positions: int) -> dict:
    """Compares the used rows of two q8 caches in the reference layout: codes and f16 scales."""
    kvw = config.kv_width
    groups = kvw // 64
    mp = config.max_positions
    scales_bytes = mp * groups * 2
    stride = scales_bytes + mp * kvw
    codes_diff, scale_ulps = [], []
    for layer in range(config.text_layers):
        base = layer * stride
        gs = gpu_bytes[base:base + scales_bytes].view(np.uint16).reshape(mp, groups)[:positions]
        os_ = oracle_bytes[base:base + scales_bytes].view(np.uint16).reshape(mp, groups)[:positions]
        gc = gpu_bytes[base + scales_bytes:base + stride].reshape(mp, kvw)[:positions].astype(np.int32)
        oc = oracle_bytes[base + scales_bytes:base + stride].reshape(mp, kvw)[:positions].astype(np.int32)
        codes_diff.append(np.abs(gc - oc))
        scale_ulps.append(np.abs(gs.astype(np.int32) - os_.astype(np.int32)))
    cd = np.concatenate([c.ravel() for c in codes_diff])
    su = np.concatenate([s.ravel() for s in scale_ulps])
    return {"codes_exact": float(np.mean(cd == 0)), "codes_max": int(cd.max()), "scales_exact": float(np.mean(su == 0)),
            "scale_ulps_max": int(su.max())}

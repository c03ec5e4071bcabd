"""Writes the decoder golden fixtures in tests/golden/ (QWFIX001 containers).

    python tests/golden/make_golden.py

The fixtures come from the CPU oracle (oracle/, the restatement of the
reference's Zig decode path; the Zig reference itself cannot be built here)
on two small seeded decoders: the released 0.6B layer geometry with 2 layers
and a 2048-token vocabulary, one with q8 and one with q4 weights. Each gets a
prompt of 20 audio rows and 4 text ids and 5 greedy steps:

  decoder_<fmt>_tokens.qwfix   [6]            the greedy ids: after the prompt, then after each step
  decoder_<fmt>_logits.qwfix   [6, 2048]      the logits those ids were taken from
  decoder_<fmt>_kv_last.qwfix  [2, 2, 1040]   per layer, the key and value rows of the last position in
                                              the q8 cache: 1024 codes then 16 f16 scale bit patterns

tests/test_golden.py regenerates them with the oracle and requires the same
bits; tests/test_gpu_golden.py checks the CUDA decode path against them.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import qwfix  # noqa: E402
from qwenscriber_b200 import quant, synthetic  # noqa: E402
from tests.parity import oracle_model, small_config  # noqa: E402

FORMATS = {"q8": quant.Q8, "q4": quant.Q4}
SEED = 21
AUDIO_ROWS, TEXT_IDS, STEPS, VOCAB = 20, 4, 5, 2048


def case(fmt: int):
    """The seeded model and prompt of one fixture set."""
    c = small_config(fmt, layers=2, vocab=VOCAB, max_positions=64)
    return c, synthetic.make_model(c, fmt, SEED), synthetic.make_prompt(c, AUDIO_ROWS, TEXT_IDS, SEED)


def kv_last_rows(om, c) -> np.ndarray:
    """Key and value rows of the newest cached position, per layer, from the
    oracle's q8 cache in the reference layout (decoder.zig:45-65)."""
    kvw, groups, mp = c.kv_width, c.kv_width // 64, c.max_positions
    scales_bytes = mp * groups * 2
    stride = scales_bytes + mp * kvw
    p = om.position - 1
    out = np.zeros((c.text_layers, 2, kvw + groups), np.float32)
    for i, cache in enumerate(om.cache_q8()):
        for layer in range(c.text_layers):
            base = layer * stride
            sc = cache[base:base + scales_bytes].view(np.uint16).reshape(mp, groups)[p]
            codes = cache[base + scales_bytes:base + stride].reshape(mp, kvw)[p]
            out[layer, i, :kvw] = codes
            out[layer, i, kvw:] = sc
    return out


def generate(fmt: int) -> dict[str, np.ndarray]:
    """Runs the oracle: prompt, then STEPS greedy steps."""
    c, model, prompt = case(fmt)
    om = oracle_model(model)
    try:
        tokens, logits = [], []
        nxt = om.prefill(prompt.tokens, prompt.audio, prompt.audio.shape[0])
        for k in range(STEPS + 1):
            tokens.append(nxt)
            logits.append(om.logits(c.vocab_size).copy())
            if k < STEPS:
                nxt = om.step(nxt)
        return {"tokens": np.array(tokens, np.float32), "logits": np.stack(logits).astype(np.float32),
                "kv_last": kv_last_rows(om, c)}
    finally:
        om.close()


def path(name: str, what: str) -> str:
    return os.path.join(HERE, f"decoder_{name}_{what}.qwfix")


def main() -> None:
    for name, fmt in FORMATS.items():
        for what, arr in generate(fmt).items():
            qwfix.write(path(name, what), arr.shape, arr)
            print(f"wrote {path(name, what)} {arr.shape}")


if __name__ == "__main__":
    main()

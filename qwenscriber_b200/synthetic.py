"""Seeded synthetic decoders and prompts for the benchmark configurations.

No checkpoint or dataset is available, so every input is drawn with numpy's
PCG64 (`default_rng`), in the shapes and value distributions the benchmark
configurations state:

  * q8 (and q5) models: f32 weights N(0, 0.02), quantized with the
    reference's q8 (q5) blocks (quant.zig:197-288 via `quant.quantize`);
  * q4 "direct" models: int4 codes uniform in [-8, 7] (bytes uniform in
    [0, 255], i.e. two uniform nibbles) and f16 group scales |N(0, 0.003)|;
  * RMSNorm weights 1.0 f32; the lm_head tied to the embedding;
  * prompts: `audio_rows` N(0, 1) prefix embeddings, then `text_ids` token ids
    uniform in [0, vocab) (an id equal to Config.token_audio_pad is redrawn,
    since it would consume an audio row).

Tensors are generated in the reference's layout order (layout.zig: layer 0
tensors by kind, then decoder layers 1..L by kind) from one generator seeded
with `seed`; prompts come from `default_rng([seed, 1, stream])`.
"""

from __future__ import annotations

import dataclasses

import numpy as np

from . import quant
from .config import Config, qwen3_asr_0p6b, qwen3_asr_1p7b

# container.zig:333-376 (decoder kinds)
EMBED, FINAL_NORM, OUTPUT = 30, 31, 32
Q, K, V, O, Q_NORM, K_NORM, ATTN_NORM, FFN_NORM, GATE, UP, DOWN = range(33, 44)
# container.zig:334-362 (audio tower and projector kinds); audio layer i is 1024 + i
(A_CONV1_W, A_CONV1_B, A_CONV2_W, A_CONV2_B, A_CONV3_W, A_CONV3_B, A_CONV_OUT_W, A_FINAL_NORM_W, A_FINAL_NORM_B,
 A_Q_W, A_Q_B, A_K_W, A_K_B, A_V_W, A_V_B, A_OUT_W, A_OUT_B, A_ATTN_NORM_W, A_ATTN_NORM_B, A_FFN_IN_W, A_FFN_IN_B,
 A_FFN_OUT_W, A_FFN_OUT_B, A_LAYER_NORM_W, A_LAYER_NORM_B, P_IN_W, P_IN_B, P_OUT_W, P_OUT_B) = range(1, 30)
AUDIO_LAYER_BASE = 1024


@dataclasses.dataclass
class Tensor:
    kind: int
    layer: int
    fmt: int
    rows: int
    cols: int
    payload: np.ndarray


@dataclasses.dataclass
class Model:
    config: Config
    fmt: int
    tensors: list[Tensor]

    @property
    def weight_bytes(self) -> int:
        return sum(t.payload.nbytes for t in self.tensors if t.fmt != quant.F32)


def _matrix(rng: np.random.Generator, fmt: int, rows: int, cols: int, std: float, q4_scale_std: float) -> np.ndarray:
    if fmt in (quant.Q8, quant.Q5):
        w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(std)
        scales, codes = quant.quantize(fmt, w)
    else:
        codes = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
        s = np.abs(rng.standard_normal((rows, cols // quant.GROUP), dtype=np.float32) * np.float32(q4_scale_std))
        scales = s.astype(np.float16).view(np.uint16)
    return quant.payload(fmt, scales, codes)


def make_audio(config: Config, fmt: int, seed: int, std: float = 0.02, q4_scale_std: float = 0.003) -> list[Tensor]:
    """The audio tower and projector in the reference's layout (layout.zig:150-262), drawn from
    default_rng([seed, 2]): convolution weights f16 N(0, 1/fan_in), biases N(0, 0.02), LayerNorm
    weights 1 + N(0, 0.05) and biases N(0, 0.02), matrices like the decoder's (`_matrix`)."""
    rng = np.random.default_rng([seed, 2])
    c = config
    d, ch, ffn = c.audio_d_model, c.audio_downsample_hidden_size, c.audio_ffn_dim

    def vec(n, scale=0.02, base=0.0):
        return (base + rng.standard_normal(n, dtype=np.float32) * np.float32(scale)).astype(np.float32)

    def conv(cin):
        w = rng.standard_normal((ch, cin * 9), dtype=np.float32) / np.float32(np.sqrt(cin * 9))
        return w.astype(np.float16).view(np.uint16)

    def mat(rows, cols):
        return _matrix(rng, fmt, rows, cols, std, q4_scale_std)

    t = [Tensor(A_CONV1_W, 0, quant.F16, ch, 9, conv(1)), Tensor(A_CONV1_B, 0, quant.F32, 1, ch, vec(ch)),
         Tensor(A_CONV2_W, 0, quant.F16, ch, ch * 9, conv(ch)), Tensor(A_CONV2_B, 0, quant.F32, 1, ch, vec(ch)),
         Tensor(A_CONV3_W, 0, quant.F16, ch, ch * 9, conv(ch)), Tensor(A_CONV3_B, 0, quant.F32, 1, ch, vec(ch)),
         Tensor(A_CONV_OUT_W, 0, fmt, d, c.audio_conv_out_features, mat(d, c.audio_conv_out_features)),
         Tensor(A_FINAL_NORM_W, 0, quant.F32, 1, d, vec(d, 0.05, 1.0)),
         Tensor(A_FINAL_NORM_B, 0, quant.F32, 1, d, vec(d))]
    for i in range(c.audio_layers):
        L = AUDIO_LAYER_BASE + i
        for kind in (A_Q_W, A_K_W, A_V_W, A_OUT_W):
            t.append(Tensor(kind, L, fmt, d, d, mat(d, d)))
            t.append(Tensor(kind + 1, L, quant.F32, 1, d, vec(d)))
        t.append(Tensor(A_ATTN_NORM_W, L, quant.F32, 1, d, vec(d, 0.05, 1.0)))
        t.append(Tensor(A_ATTN_NORM_B, L, quant.F32, 1, d, vec(d)))
        t.append(Tensor(A_FFN_IN_W, L, fmt, ffn, d, mat(ffn, d)))
        t.append(Tensor(A_FFN_IN_B, L, quant.F32, 1, ffn, vec(ffn)))
        t.append(Tensor(A_FFN_OUT_W, L, fmt, d, ffn, mat(d, ffn)))
        t.append(Tensor(A_FFN_OUT_B, L, quant.F32, 1, d, vec(d)))
        t.append(Tensor(A_LAYER_NORM_W, L, quant.F32, 1, d, vec(d, 0.05, 1.0)))
        t.append(Tensor(A_LAYER_NORM_B, L, quant.F32, 1, d, vec(d)))
    t += [Tensor(P_IN_W, 0, fmt, d, d, mat(d, d)), Tensor(P_IN_B, 0, quant.F32, 1, d, vec(d)),
          Tensor(P_OUT_W, 0, fmt, c.audio_output_dim, d, mat(c.audio_output_dim, d)),
          Tensor(P_OUT_B, 0, quant.F32, 1, c.audio_output_dim, vec(c.audio_output_dim))]
    return t


def make_log_mel(config: Config, frames: int, seed: int, stream: int = 0) -> np.ndarray:
    """A clip's log-mel stand-in: [mel_bins][frames] f32, N(0, 0.5) (default_rng([seed, 3, stream]))."""
    rng = np.random.default_rng([seed, 3, stream])
    return (rng.standard_normal((config.mel_bins, frames), dtype=np.float32) * np.float32(0.5)).astype(np.float32)


def make_model(config: Config, fmt: int, seed: int, std: float = 0.02, q4_scale_std: float = 0.003,
               audio: bool = False) -> Model:
    rng = np.random.default_rng(seed)
    c = config
    h, qw, kvw, ffn = c.text_hidden_size, c.q_width, c.kv_width, c.text_ffn_dim
    ones = lambda n: np.ones(n, np.float32)  # noqa: E731
    tensors = [Tensor(EMBED, 0, fmt, c.vocab_size, h, _matrix(rng, fmt, c.vocab_size, h, std, q4_scale_std)),
               Tensor(FINAL_NORM, 0, quant.F32, 1, h, ones(h))]
    if not c.tied:
        tensors.append(Tensor(OUTPUT, 0, fmt, c.vocab_size, h, _matrix(rng, fmt, c.vocab_size, h, std, q4_scale_std)))
    for layer in range(1, c.text_layers + 1):
        for kind, rows, cols in ((Q, qw, h), (K, kvw, h), (V, kvw, h), (O, h, qw)):
            tensors.append(Tensor(kind, layer, fmt, rows, cols, _matrix(rng, fmt, rows, cols, std, q4_scale_std)))
        tensors.append(Tensor(Q_NORM, layer, quant.F32, 1, c.text_head_dim, ones(c.text_head_dim)))
        tensors.append(Tensor(K_NORM, layer, quant.F32, 1, c.text_head_dim, ones(c.text_head_dim)))
        tensors.append(Tensor(ATTN_NORM, layer, quant.F32, 1, h, ones(h)))
        tensors.append(Tensor(FFN_NORM, layer, quant.F32, 1, h, ones(h)))
        for kind, rows, cols in ((GATE, ffn, h), (UP, ffn, h), (DOWN, h, ffn)):
            tensors.append(Tensor(kind, layer, fmt, rows, cols, _matrix(rng, fmt, rows, cols, std, q4_scale_std)))
    if audio:
        tensors += make_audio(c, fmt, seed, std, q4_scale_std)
    return Model(c, fmt, tensors)


@dataclasses.dataclass
class Prompt:
    tokens: np.ndarray  # uint32 [n]
    audio: np.ndarray   # float32 [audio_steps, hidden]


def make_prompt(config: Config, audio_rows: int, text_ids: int, seed: int, stream: int = 0) -> Prompt:
    rng = np.random.default_rng([seed, 1, stream])
    audio = rng.standard_normal((audio_rows, config.text_hidden_size), dtype=np.float32)
    ids = rng.integers(0, config.vocab_size, size=text_ids, dtype=np.int64)
    while np.any(ids == config.token_audio_pad):
        bad = ids == config.token_audio_pad
        ids[bad] = rng.integers(0, config.vocab_size, size=int(bad.sum()))
    tokens = np.concatenate([np.full(audio_rows, config.token_audio_pad, np.int64), ids]).astype(np.uint32)
    return Prompt(tokens, audio)


# BASELINE.json configs[0..4]
@dataclasses.dataclass
class Workload:
    name: str
    config: Config
    fmt: int
    seed: int
    audio_rows: int | tuple[int, int]
    text_ids: int
    decode: int
    streams: int


def workloads() -> dict[str, Workload]:
    return {
        "cfg0_0p6b_q8_b1": Workload("cfg0_0p6b_q8_b1", qwen3_asr_0p6b(max_positions=512, max_decode_tokens=512),
                                    quant.Q8, 0, 188, 8, 64, 1),
        "cfg1_0p6b_q4_b1": Workload("cfg1_0p6b_q4_b1", qwen3_asr_0p6b(max_positions=1024, max_decode_tokens=1024),
                                    quant.Q4, 0, 500, 12, 256, 1),
        "cfg2_1p7b_q4_b1": Workload("cfg2_1p7b_q4_b1", qwen3_asr_1p7b(max_positions=1024, max_decode_tokens=1024),
                                    quant.Q4, 1, 375, 16, 448, 1),
        "cfg3_1p7b_q4_s64": Workload("cfg3_1p7b_q4_s64", qwen3_asr_1p7b(max_positions=2048, max_decode_tokens=1024),
                                     quant.Q4, 1, (100, 1500), 16, 256, 64),
        "cfg4_1p7b_q4_s64_long": Workload("cfg4_1p7b_q4_s64_long",
                                          qwen3_asr_1p7b(max_positions=4096, max_decode_tokens=1024),
                                          quant.Q4, 1, (2048, 3584), 16, 512, 64),
        # Not a benchmark configuration: configs[0]'s model and prompt with q5
        # weights (the format the reference ships to browsers), for the q5 path.
        "q5_0p6b_b1": Workload("q5_0p6b_b1", qwen3_asr_0p6b(max_positions=512, max_decode_tokens=512),
                               quant.Q5, 0, 188, 8, 64, 1),
    }


def prefix_lengths(w: Workload, world: int = 1, rank: int = 0) -> list[int]:
    """Audio-prefix rows of the streams one GPU decodes in a multi-stream
    workload (uniform in the stated range, per-workload seed): rank `rank` of
    `world` takes global streams [rank * streams, (rank + 1) * streams)."""
    from . import shards

    if isinstance(w.audio_rows, int):
        return [w.audio_rows] * w.streams
    lo, hi = w.audio_rows
    every = shards.prefix_lengths(lo, hi, w.seed, w.streams * world)
    return [every[g] for g in shards.shard(w.streams * world, world, rank)]


def load_into(model: Model, target, cache_format: int = 1, streams: int | None = None) -> None:
    """Loads a synthetic model through the reference-shaped model family of `target`
    (a `runtime.CudaModel`, or anything with the same methods)."""
    target.begin()
    for t in model.tensors:
        target.add_tensor(t.kind, t.layer, t.fmt, t.rows, t.cols, t.payload)
    target.set_cache_format(cache_format)
    if streams is not None:
        target.set_streams(streams)
    target.finish(model.config.pack())

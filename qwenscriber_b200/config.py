"""The 160-byte model configuration (src/core/model_config.zig:110-177).

`Config` packs to exactly the bytes the reference's converter writes to
`config.bin` and its runtime validates, so the same bytes drive the CUDA
backend (`qwc_model_finish`) and the CPU oracle.
"""

from __future__ import annotations

import dataclasses
import struct

MAGIC = b"QWCFG001"
FORMAT_VERSION = 1
ARCH_QWEN3_ASR = 1
SIZE = 160
FLAG_OUTPUT_PROJECTION_TIED = 1

# (name, struct code) in on-disk order, model_config.zig:110-173.
_FIELDS = [
    ("format_version", "I"), ("architecture", "I"),
    ("audio_d_model", "I"), ("audio_layers", "I"), ("audio_attention_heads", "I"), ("audio_ffn_dim", "I"),
    ("audio_downsample_hidden_size", "I"), ("audio_n_window", "I"), ("audio_n_window_infer", "I"),
    ("audio_max_position_steps", "I"), ("audio_output_dim", "I"), ("mel_bins", "I"), ("audio_layer_norm_eps", "f"),
    ("text_hidden_size", "I"), ("text_layers", "I"), ("text_attention_heads", "I"), ("text_key_value_heads", "I"),
    ("text_head_dim", "I"), ("text_ffn_dim", "I"), ("vocab_size", "I"), ("text_rms_norm_eps", "f"),
    ("rope_theta", "f"), ("max_positions", "I"), ("max_decode_tokens", "I"),
    ("token_audio_start", "I"), ("token_audio_end", "I"), ("token_audio_pad", "I"), ("token_im_start", "I"),
    ("token_im_end", "I"), ("token_endoftext", "I"), ("token_asr_text", "I"), ("token_eos_primary", "I"),
    ("token_eos_secondary", "I"), ("token_pad", "I"),
    ("flags", "I"), ("reserved1", "I"), ("reserved2", "I"), ("reserved3", "I"),
]
_FORMAT = "<8s" + "".join(code for _, code in _FIELDS)
assert struct.calcsize(_FORMAT) == SIZE


@dataclasses.dataclass
class Config:
    # Defaults: the released 0.6B checkpoint (model_config.zig:377-415), tied output projection.
    format_version: int = FORMAT_VERSION
    architecture: int = ARCH_QWEN3_ASR
    audio_d_model: int = 896
    audio_layers: int = 18
    audio_attention_heads: int = 14
    audio_ffn_dim: int = 3584
    audio_downsample_hidden_size: int = 480
    audio_n_window: int = 50
    audio_n_window_infer: int = 800
    audio_max_position_steps: int = 13
    audio_output_dim: int = 1024
    mel_bins: int = 128
    audio_layer_norm_eps: float = 1e-5
    text_hidden_size: int = 1024
    text_layers: int = 28
    text_attention_heads: int = 16
    text_key_value_heads: int = 8
    text_head_dim: int = 128
    text_ffn_dim: int = 3072
    vocab_size: int = 151936
    text_rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    max_positions: int = 4096
    max_decode_tokens: int = 1024
    token_audio_start: int = 151669
    token_audio_end: int = 151670
    token_audio_pad: int = 151676
    token_im_start: int = 151644
    token_im_end: int = 151645
    token_endoftext: int = 151643
    token_asr_text: int = 151704
    token_eos_primary: int = 151643
    token_eos_secondary: int = 151645
    token_pad: int = 151643
    flags: int = FLAG_OUTPUT_PROJECTION_TIED
    reserved1: int = 0
    reserved2: int = 0
    reserved3: int = 0
    magic: bytes = MAGIC

    def pack(self) -> bytes:
        values = [getattr(self, name) for name, _ in _FIELDS]
        return struct.pack(_FORMAT, self.magic, *values)

    @classmethod
    def unpack(cls, data: bytes) -> "Config":
        if len(data) != SIZE:
            raise ValueError("a configuration is exactly 160 bytes")
        parts = struct.unpack(_FORMAT, data)
        kwargs = {name: parts[i + 1] for i, (name, _) in enumerate(_FIELDS)}
        return cls(magic=parts[0], **kwargs)

    @property
    def q_width(self) -> int:
        return self.text_attention_heads * self.text_head_dim

    @property
    def kv_width(self) -> int:
        return self.text_key_value_heads * self.text_head_dim

    @property
    def tied(self) -> bool:
        return bool(self.flags & FLAG_OUTPUT_PROJECTION_TIED)

    # The audio tower's derived geometry (model_config.zig:190-240).
    @staticmethod
    def conv_steps(n: int) -> int:
        """postConvolutionSteps: three kernel-3, stride-2, padding-1 halvings (0 stays 0)."""
        if n == 0:
            return 0
        for _ in range(3):
            n = (n - 1) // 2 + 1
        return n

    @property
    def audio_head_dim(self) -> int:
        return self.audio_d_model // self.audio_attention_heads

    @property
    def audio_chunk_frames(self) -> int:
        return self.audio_n_window * 2

    @property
    def audio_chunk_steps(self) -> int:
        return self.conv_steps(self.audio_chunk_frames)

    @property
    def audio_frequency_bins(self) -> int:
        return self.conv_steps(self.mel_bins)

    @property
    def audio_conv_out_features(self) -> int:
        return self.audio_downsample_hidden_size * self.audio_frequency_bins

    def packed_steps(self, frames: int) -> int:
        """packedStepCount: whole chunks convolved separately, then the partial one."""
        chunk = self.audio_chunk_frames
        return (frames // chunk) * self.conv_steps(chunk) + self.conv_steps(frames % chunk)


def qwen3_asr_0p6b(**overrides) -> Config:
    """Decoder geometry of the released 0.6B checkpoint (model_config.zig:377-415)."""
    return dataclasses.replace(Config(), **overrides)


def qwen3_asr_1p7b(**overrides) -> Config:
    """Decoder geometry of the released 1.7B checkpoint (model_config.zig:441-480)."""
    base = Config(
        audio_d_model=1024, audio_layers=24, audio_attention_heads=16, audio_ffn_dim=4096, audio_output_dim=2048,
        text_hidden_size=2048, text_ffn_dim=6144,
    )
    return dataclasses.replace(base, **overrides)

/*
 * qwenscriber_cuda.h -- C ABI of libqwenscriber_cuda, the sm_100a (B200)
 * backend for Qwenscriber's decoder token loop.
 *
 * The library is a drop-in `cuda` backend beside the reference's `wasm` and
 * `webgpu` backends. Its model and decode families mirror the reference's
 * `qw_model_*` / `qw_decode_*` exports (src/wasm/exports.zig) and their state
 * machine (src/wasm/model.zig:9-26): idle -> ready -> loaded -> decoding.
 * Status codes are the reference's own numbers (src/wasm/abi.zig:50-84).
 *
 * Conventions (src/wasm/abi.zig:1-17, docs/src/reference/c-abi.md):
 *   - fixed-width integers, pointer plus explicit length, no library types;
 *   - every call returns a status (0 ok, negative failure) unless noted;
 *   - caller-owned buffers; the library never frees caller memory;
 *   - a handle is bound to one CUDA device and is not thread-safe; use one
 *     handle per GPU, each driven by its own host thread or process.
 *
 * Unlike the WASM build, which borrows the caller's shard bytes for the life
 * of the model (src/wasm/model.zig:28-42), this library copies each tensor
 * payload into device memory (HBM) when it is added, after which the caller
 * may release its buffer.
 */
#ifndef QWENSCRIBER_CUDA_H
#define QWENSCRIBER_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ABI version: major << 16 | minor (src/wasm/abi.zig:15-28). */
#define QWC_ABI_MAJOR 1u
#define QWC_ABI_MINOR 0u

/* Status codes: identical numbers to src/wasm/abi.zig:50-84. */
enum {
  QWC_OK = 0,
  QWC_INVALID_ARGUMENT = -1,
  QWC_OUT_OF_MEMORY = -2,
  QWC_UNSUPPORTED = -3,
  QWC_BAD_MAGIC = -4,
  QWC_BAD_VERSION = -5,
  QWC_CHECKSUM_MISMATCH = -6,
  QWC_SHAPE_MISMATCH = -7,
  QWC_INVALID_STATE = -8,
  QWC_LIMIT_EXCEEDED = -9,
  QWC_NOT_FOUND = -10,
  QWC_TRUNCATED = -11,
  QWC_INVALID_ENCODING = -12,
  QWC_UNSUPPORTED_MODEL = -13,
  QWC_AUDIO_TOO_LONG = -14
};

/* Tensor formats: src/core/dtype.zig:17-24. */
enum { QWC_FORMAT_F32 = 0, QWC_FORMAT_F16 = 1, QWC_FORMAT_BF16 = 2, QWC_FORMAT_Q4 = 16, QWC_FORMAT_Q5 = 17, QWC_FORMAT_Q8 = 18 };

/* Key/value cache formats: src/wasm/abi.zig:36-46. */
enum { QWC_CACHE_F32 = 0, QWC_CACHE_Q8 = 1 };

/* Decoder tensor kinds: the reference's container.TensorKind values
 * (src/core/container.zig:333-376). Decoder layers are numbered 1..=layers
 * and tensors outside a layer use layer 0 (src/core/qwen3_asr/layout.zig:14-28). */
enum {
  QWC_KIND_DECODER_EMBED_TOKENS = 30,
  QWC_KIND_DECODER_FINAL_NORM = 31,
  QWC_KIND_DECODER_OUTPUT = 32,
  QWC_KIND_DECODER_Q = 33,
  QWC_KIND_DECODER_K = 34,
  QWC_KIND_DECODER_V = 35,
  QWC_KIND_DECODER_O = 36,
  QWC_KIND_DECODER_Q_NORM = 37,
  QWC_KIND_DECODER_K_NORM = 38,
  QWC_KIND_DECODER_ATTENTION_NORM = 39,
  QWC_KIND_DECODER_FFN_NORM = 40,
  QWC_KIND_DECODER_GATE = 41,
  QWC_KIND_DECODER_UP = 42,
  QWC_KIND_DECODER_DOWN = 43
};

/* Audio tower and projector kinds (container.zig:334-362). Audio layer i is
 * numbered 1024 + i (container.zig:307); the convolutions, conv_out, the
 * final norm and the projector use layer 0. The three convolution weights are
 * f16 [out][in][3][3] (layout.zig:150-175; through qwc_model_add_tensor as
 * `out` rows of in * 9 values); biases and norm vectors f32; the matrices
 * q4/q5/q8 like the decoder's. */
enum {
  QWC_KIND_AUDIO_CONV1_WEIGHT = 1,
  QWC_KIND_AUDIO_CONV1_BIAS = 2,
  QWC_KIND_AUDIO_CONV2_WEIGHT = 3,
  QWC_KIND_AUDIO_CONV2_BIAS = 4,
  QWC_KIND_AUDIO_CONV3_WEIGHT = 5,
  QWC_KIND_AUDIO_CONV3_BIAS = 6,
  QWC_KIND_AUDIO_CONV_OUT_WEIGHT = 7,
  QWC_KIND_AUDIO_FINAL_NORM_WEIGHT = 8,
  QWC_KIND_AUDIO_FINAL_NORM_BIAS = 9,
  QWC_KIND_AUDIO_Q_WEIGHT = 10,
  QWC_KIND_AUDIO_Q_BIAS = 11,
  QWC_KIND_AUDIO_K_WEIGHT = 12,
  QWC_KIND_AUDIO_K_BIAS = 13,
  QWC_KIND_AUDIO_V_WEIGHT = 14,
  QWC_KIND_AUDIO_V_BIAS = 15,
  QWC_KIND_AUDIO_OUT_WEIGHT = 16,
  QWC_KIND_AUDIO_OUT_BIAS = 17,
  QWC_KIND_AUDIO_ATTENTION_NORM_WEIGHT = 18,
  QWC_KIND_AUDIO_ATTENTION_NORM_BIAS = 19,
  QWC_KIND_AUDIO_FFN_IN_WEIGHT = 20,
  QWC_KIND_AUDIO_FFN_IN_BIAS = 21,
  QWC_KIND_AUDIO_FFN_OUT_WEIGHT = 22,
  QWC_KIND_AUDIO_FFN_OUT_BIAS = 23,
  QWC_KIND_AUDIO_FINAL_LAYER_NORM_WEIGHT = 24,
  QWC_KIND_AUDIO_FINAL_LAYER_NORM_BIAS = 25,
  QWC_KIND_PROJECTOR_IN_WEIGHT = 26,
  QWC_KIND_PROJECTOR_IN_BIAS = 27,
  QWC_KIND_PROJECTOR_OUT_WEIGHT = 28,
  QWC_KIND_PROJECTOR_OUT_BIAS = 29
};
#define QWC_AUDIO_LAYER_BASE 1024u

/* Feature bits (src/wasm/abi.zig:179-207): model and decode families, plus
 * the batched multi-stream family this backend adds. */
#define QWC_FEATURE_MODEL (1u << 3)
#define QWC_FEATURE_DECODE (1u << 4)
#define QWC_FEATURE_STREAMS (1u << 8)

/* qw_model_requirements layout, 48 bytes (src/wasm/abi.zig:281-290). */
typedef struct qwc_requirements {
  uint64_t weight_bytes;  /* device bytes holding the weight payloads */
  uint64_t cache_bytes;   /* key/value cache, all layers, all stream slots */
  uint64_t scratch_bytes; /* activations, rope tables, logits, partials */
  uint64_t total_bytes;   /* weight_bytes + cache_bytes + scratch_bytes */
  uint32_t max_positions;
  uint32_t max_audio_frames;
  uint32_t max_decode_tokens;
  uint32_t reserved;
} qwc_requirements;

/* qw_model_tensor_descriptor layout, 64 bytes (src/wasm/abi.zig:370-382). */
typedef struct qwc_tensor_descriptor {
  uint64_t offset_bytes; /* from the start of its shard's bytes; 0 for a tensor added alone */
  uint64_t len_bytes;    /* its payload bytes */
  uint32_t kind;
  uint32_t layer;
  uint32_t format;
  uint32_t rank;
  uint32_t dims[4];      /* unused dimensions are 1, as the container writes them */
  uint32_t shard_index;  /* its shard, in the order shards were added; 0xFFFFFFFF if added alone */
  uint32_t reserved[3];
} qwc_tensor_descriptor;

/* qw_model_audio_config layout, 72 bytes (src/wasm/abi.zig:292-340): the
 * audio tower's geometry, every derived value resolved by the configuration
 * helpers the forward pass uses. */
typedef struct qwc_audio_config {
  uint32_t d_model;                 /* tower width, in and out of every block */
  uint32_t layers;                  /* encoder blocks */
  uint32_t attention_heads;
  uint32_t head_dim;                /* d_model / attention_heads */
  uint32_t ffn_dim;
  uint32_t downsample_hidden_size;  /* the convolution stack's output channels */
  uint32_t n_window;                /* mel frames per half-chunk */
  uint32_t n_window_infer;          /* mel frames one attention window spans */
  uint32_t chunk_frames;            /* mel frames one convolution chunk consumes */
  uint32_t frequency_bins;          /* mel bins left after the convolution stack */
  uint32_t conv_out_input_features; /* downsample_hidden_size * frequency_bins */
  uint32_t chunk_steps;             /* time steps the stack emits per chunk */
  uint32_t max_position_steps;
  uint32_t output_dim;              /* projector output width, the decoder's hidden size */
  uint32_t mel_bins;
  float layer_norm_eps;
  uint32_t reserved_0;
  uint32_t reserved_1;
} qwc_audio_config;

/* Handle options (qwc_set_option). */
enum {
  /* Nonzero: decode does not stop at end-of-sequence tokens (fixed-length
   * benchmarking, as src/cli/transcribe.zig:200-208 runs Decoder.step). */
  QWC_OPTION_IGNORE_EOS = 1,
  /* Nonzero: keep the last computed logits of each stream on the device so
   * qwc_debug_logits can return them (parity testing). */
  QWC_OPTION_KEEP_LOGITS = 2,
  /* Decode steps computed ahead per device launch (1..256, default 16). */
  QWC_OPTION_STEP_CHUNK = 3,
  /* Nonzero: every launch records a phase timeline of its first step
   * (%globaltimer per CTA at each phase boundary); see qwc_debug_trace. */
  QWC_OPTION_TRACE = 4,
  /* Prompt prefill of single-stream handles: 0 (default) batched on the
   * tensor cores, 64 positions per step; 1 token by token through the
   * persistent decode kernel. */
  QWC_OPTION_PREFILL_SERIAL = 5,
  /* Single-stream handles. Nonzero: every f32 operation of the decode runs
   * in the order the reference's CPU path writes it (Decoder.forwardToken,
   * decoder.zig:133-287): each dot product's four lanes summed in index
   * order, sums of squares and softmax sums in order, attention over the
   * whole history per kv head, no contracted multiply-adds, and exp computed
   * as the host C library's expf. Logits, cache rows and greedy tokens then
   * equal the CPU oracle's bit for bit. The prompt is prefilled token by
   * token through the same kernel. Slower than the default. */
  QWC_OPTION_EXACT = 6,
  /* Bound on every device-side wait of the decode kernels (mbarrier phases,
   * grid barriers, split-K counters), in microseconds; 0 restores the default
   * (4 s single-stream, 2 s batched). A wait that runs out makes the call
   * return QWC_INVALID_STATE instead of hanging; the handle stays usable. */
  QWC_OPTION_WAIT_LIMIT_US = 7,
  /* Failure-path testing, single-stream handles. Nonzero: the next launch of
   * the decode kernel (only that one) makes its grid barriers wait for one
   * more CTA than the launch has, so they can only end when their bound
   * (QWC_OPTION_WAIT_LIMIT_US) runs out, and the call returns
   * QWC_INVALID_STATE. No device fault is involved. */
  QWC_OPTION_TEST_STALL = 8
};

/* ---- version and lifecycle (src/wasm/exports.zig:49-120) ---- */

/* qw_abi_version (exports.zig:49). */
uint32_t qwc_abi_version(void);
/* qw_features (exports.zig:300-309; abi.zig:202-207). */
uint32_t qwc_features(void);
/* qw_create: returns a nonzero handle bound to CUDA device `device`, or 0. */
uint32_t qwc_create(int32_t device);
/* qw_destroy: releases every device allocation of the handle. */
int32_t qwc_destroy(uint32_t handle);
/* Text of a status code (abi.zig:153-171); never NULL. */
const char* qwc_status_message(int32_t status);
int32_t qwc_set_option(uint32_t handle, uint32_t option, uint32_t value);

/* ---- model family (src/wasm/exports.zig:320-425; src/wasm/model.zig:136-263) ---- */

/* qw_model_begin: starts a model attempt; legal in every state and also the unload path. */
int32_t qwc_model_begin(uint32_t handle);
/* One tensor without a container (the per-tensor form of qwc_model_add_shard): `payload` holds that tensor's
 * container payload -- for q4/q5/q8 the f16 scale plane, padding to 16 bytes,
 * then the code plane (src/core/quant.zig:144-176); for f32 vectors the
 * values. Copied to device memory before returning. */
int32_t qwc_model_add_tensor(uint32_t handle, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows,
                             uint32_t cols, const void* payload, uint64_t len);
/* qw_model_add_shard (src/wasm/exports.zig:333-340; src/wasm/model.zig:156-178):
 * validates one `.qw` shard in place -- magic, version, index order and
 * ranges, every tensor's shape and byte length, and the payload checksum
 * (src/core/container.zig:98-291) -- and copies its decoder tensors to device
 * memory, as qwc_model_add_tensor does. `bytes` must be 16-byte aligned and
 * may be freed after the call. Tensors of other kinds (audio tower,
 * projector) are validated and not kept. A shard whose payload checksum
 * matches one already added, or a tensor already added, is invalid_argument; a decoder tensor in a
 * format the kernels do not run (f16, bf16) is unsupported_model; more
 * than 64 shards is limit_exceeded. A shard refused by any of these checks, or whose copy to
 * the device fails part way (out_of_memory), leaves the handle unchanged. */
int32_t qwc_model_add_shard(uint32_t handle, const void* bytes, uint64_t len);
/* container.File.parse followed by verifyChecksum on its own: no handle and
 * no device. Returns QWC_OK (and the tensor count) or the status the shard
 * would be refused with. */
int32_t qwc_shard_validate(const void* bytes, uint64_t len, uint32_t* tensor_count);
/* The payload checksum a shard header stores: the low 32 bits of FNV-1a 64
 * over `len` bytes (container.zig:283-286); for shard writers. */
uint32_t qwc_shard_checksum(const void* bytes, uint64_t len);
/* qw_model_set_cache_format (exports.zig:352-363): ready state only. */
int32_t qwc_model_set_cache_format(uint32_t handle, uint32_t format);
/* Number of independent decode streams the next finish allocates (default 1), 1..64. */
int32_t qwc_model_set_streams(uint32_t handle, uint32_t streams);
/* qw_model_finish: validates the 160-byte Config (src/core/model_config.zig:110-177,
 * 260-328), resolves every tensor, allocates caches and scratch. */
int32_t qwc_model_finish(uint32_t handle, const void* config, uint32_t config_len);
/* qw_model_requirements (exports.zig:371-378). */
int32_t qwc_model_requirements(uint32_t handle, qwc_requirements* out);
/* qw_model_tensor_count (exports.zig:384-389, model.zig:265-279): every entry of every shard
 * added, audio-tower and projector tensors included, plus each tensor added alone. */
int32_t qwc_model_tensor_count(uint32_t handle, uint32_t* out);
/* qw_model_tensor_descriptor (exports.zig:402-412, model.zig:281-319): entry `index` of that
 * enumeration -- shards in the order they were added, each shard's entries in its index order,
 * then tensors added alone in call order -- with its offset within its shard's bytes, length,
 * shape and shard. Entries the decoder does not use are described though not kept on the device.
 * QWC_NOT_FOUND past the last entry, QWC_INVALID_STATE before qwc_model_finish. */
int32_t qwc_model_tensor_descriptor(uint32_t handle, uint32_t index, qwc_tensor_descriptor* out);

/* qw_model_audio_config (exports.zig:415-426, model.zig:327-360): in the loaded and decoding
 * states, QWC_INVALID_STATE otherwise. */
int32_t qwc_model_audio_config(uint32_t handle, qwc_audio_config* out);

/* ---- audio family: the tower and projector (src/core/qwen3_asr/model.zig:445-744) ----
 * A model that carries the audio-tower and projector tensors (all of them:
 * qwc_model_finish returns QWC_NOT_FOUND when some are missing) runs them on
 * the device. `log_mel` / `features` is the log-mel spectrogram of one clip,
 * mel_bins x frames f32 row major (what qw_mel_compute writes), at most 3000
 * frames (QWC_AUDIO_TOO_LONG beyond). A handle without a tower returns
 * QWC_NOT_FOUND. */

/* Model.projectAudio (model.zig:451-460): the convolution stack, the tower and
 * the projector over one clip; writes steps x output_dim f32 rows to `out`
 * (host memory, capacity in floats; QWC_LIMIT_EXCEEDED when too small) and
 * the step count (Config.packedStepCount of the frames) to *steps_out. */
int32_t qwc_audio_project(uint32_t handle, const float* log_mel, uint32_t frames, float* out,
                          uint64_t out_capacity_floats, uint32_t* steps_out);

/* ---- decode family, stream slot 0 (src/wasm/exports.zig:440-497; model.zig:370-474) ---- */

/* qw_decode_begin after the audio tower: resets stream 0's cache, prefills
 * `prompt` (token == Config.token_audio_pad consumes the next of `audio_steps`
 * rows of `audio`, text_hidden_size f32 each; decoder.zig:308-333) and holds
 * the first predicted token. */
int32_t qwc_decode_begin(uint32_t handle, const uint32_t* prompt, uint32_t prompt_len, const float* audio,
                         uint32_t audio_steps, uint32_t max_tokens);
/* qw_decode_begin from the clip's log-mel features (exports.zig:440-458,
 * model.zig:370-410): runs the tower and projector on the device, then
 * prefills `prompt` with the projected rows, which stay on the device. The
 * prompt's token ids come from the caller (the reference builds them from its
 * vocabulary, prompt.zig): it must hold one Config.token_audio_pad per packed
 * step (QWC_SHAPE_MISMATCH otherwise). features_len is in bytes, a whole
 * number of mel_bins f32 columns. */
int32_t qwc_decode_begin_features(uint32_t handle, const uint32_t* prompt, uint32_t prompt_len, const float* features,
                                  uint64_t features_len, uint32_t max_tokens);
/* qw_decode_step: 1 and *token_out written, 0 when finished, <0 status. */
int32_t qwc_decode_step(uint32_t handle, uint32_t* token_out);
/* qw_decode_tokens: copies the ids produced so far, returns their count. */
int32_t qwc_decode_tokens(uint32_t handle, uint32_t* out, uint32_t capacity);
/* qw_decode_end: back to loaded; the cache is cleared. */
int32_t qwc_decode_end(uint32_t handle);

/* ---- multi-stream family: independent streams batched per device step ----
 * With qwc_model_set_streams(n), 2 <= n <= 64, every step runs all slots
 * together (projections on the tensor cores with the slots as GEMM columns,
 * as in qwc_op_gemm_streams). qwc_stream_begin prefills the slot's prompt
 * (64 positions per tensor-core step) and holds its first prediction, as
 * qw_decode_begin does; each qwc_streams_step then emits every decoding
 * slot's held token and computes the next (decodeStep, model.zig:423-451).
 * The qwc_decode_* family is for single-stream handles, whose prompts are
 * prefilled the same way. */

int32_t qwc_stream_begin(uint32_t handle, uint32_t slot, const uint32_t* prompt, uint32_t prompt_len,
                         const float* audio, uint32_t audio_steps, uint32_t max_tokens);
/* qwc_decode_begin_features for stream slot `slot`. */
int32_t qwc_stream_begin_features(uint32_t handle, uint32_t slot, const uint32_t* prompt, uint32_t prompt_len,
                                  const float* features, uint64_t features_len, uint32_t max_tokens);
/* Advances every decoding slot by one token. results[slot]: 1 token written
 * to tokens_out[slot], 0 finished or idle, <0 status of that slot
 * (QWC_LIMIT_EXCEEDED at max_positions). Returns the number of tokens
 * produced, or <0 status. Both arrays hold `streams` entries. */
int32_t qwc_streams_step(uint32_t handle, uint32_t* tokens_out, int32_t* results);
int32_t qwc_stream_tokens(uint32_t handle, uint32_t slot, uint32_t* out, uint32_t capacity);
int32_t qwc_stream_end(uint32_t handle, uint32_t slot);
/* Measurement: `steps` greedy steps of every decoding slot of a batched
 * handle (all past their prompts), chained on the device without host
 * round trips or end-of-sequence handling; device time in milliseconds. */
int32_t qwc_streams_run_timed(uint32_t handle, uint32_t steps, float* device_ms);

/* ---- measurement and parity (not part of the reference ABI) ---- */

/* Runs `steps` greedy decode steps of stream 0 on the device (held token
 * first), without end-of-sequence handling, and reports their device time in
 * milliseconds measured with CUDA events on the handle's stream. */
int32_t qwc_decode_run_timed(uint32_t handle, uint32_t steps, float* device_ms);
/* Last logits computed for `slot` (QWC_OPTION_KEEP_LOGITS must be set). */
int32_t qwc_debug_logits(uint32_t handle, uint32_t slot, float* out, uint32_t count);
/* Reads the token `slot` holds for its next qwc_decode_step into *held_out;
 * when `force` >= 0, replaces it with `force` first (teacher forcing for
 * parity runs). Requires one decode step per launch (QWC_OPTION_STEP_CHUNK 1)
 * or no steps computed ahead. */
int32_t qwc_debug_hold(uint32_t handle, uint32_t slot, int64_t force, uint32_t* held_out);
/* Device scratch of the last launch's last forward pass, last layer:
 * which 0 = hidden (after the final residual add), 1 = q|k|v projections
 * (before QK-norm and RoPE), 2 = attention output, 3 = silu(gate) * up.
 * which 4 (handles with the batched engine): the batched step's q|k|v
 * projections of the last layer before QK-norm and RoPE, 64 rows (one per
 * GEMM column) of q width + 2 kv width floats. */
int32_t qwc_debug_scratch(uint32_t handle, uint32_t which, float* out, uint32_t count);
/* Phase timeline of the last launch (QWC_OPTION_TRACE): grid x 512 nanosecond
 * stamps. A token walks six stages per layer (QKV, attention, O, gate, up,
 * down) and then the lm_head stage; each stage records three stamps (input
 * ready, output done, grid barrier passed; gate has no barrier of its own).
 * The last three words of a CTA's row are its thread 0's time with streamed
 * tiles in hand, waiting for tiles, and waiting at grid barriers. Returns
 * the count. */
int32_t qwc_debug_trace(uint32_t handle, uint64_t* out, uint32_t count);
/* Raw key (which = 0) or value (which = 1) cache bytes of `slot`, in the
 * reference's layer-major two-plane layout (src/core/qwen3_asr/decoder.zig:45-65). */
int32_t qwc_debug_cache(uint32_t handle, uint32_t slot, uint32_t which, void* out, uint64_t len);
/* The audio tower's packed sequence of the last clip, steps x d_model f32:
 * which 0 = after the convolution stack, conv_out and the position rows
 * (Model.encodeConvStage, model.zig:476-485); which 1 = after the tower's
 * blocks and its final LayerNorm (encodeTowerStage + encodedSteps,
 * model.zig:491-499). `count` floats at most; returns the count written. */
int32_t qwc_debug_audio(uint32_t handle, uint32_t which, float* out, uint64_t count);
/* Measurement: uploads `log_mel` once, then runs the tower and projector
 * `reps` times on the device (inputs resident, outputs left on the device),
 * reporting the device time of all reps in milliseconds (CUDA events on the
 * handle's stream) and the kernels one clip launches in *launches_out. */
int32_t qwc_audio_run_timed(uint32_t handle, const float* log_mel, uint32_t frames, uint32_t reps, float* device_ms,
                            uint32_t* launches_out);
/* Device kernels launched by this handle since creation. */
uint64_t qwc_kernel_launches(uint32_t handle);
/* Rotary tables as the model builds them (src/core/qwen3_asr/kernels.zig:534-564):
 * max_positions rows of head_dim / 2 values each. Host-only. */
int32_t qwc_rope_tables(float theta, uint32_t head_dim, uint32_t max_positions, float* cos_out, float* sin_out);

/* ---- device-pointer operators (caller's CUDA stream; NULL = default stream) ----
 * The per-token kernels' building blocks, exposed so a host can run one step
 * of the token loop on its own buffers and so parity tests can check each
 * against the reference arithmetic. All pointers are device pointers. */

/* quant.dequantizeRow (src/core/quant.zig:348-364) over `rows` rows: bit exact.
 * Formats q4, q5, q8; `scales` 2-byte aligned (else QWC_INVALID_ARGUMENT). */
int32_t qwc_op_dequantize(uint32_t format, const void* scales, const void* codes, uint32_t rows, uint32_t cols,
                          float* out, void* stream);
/* quant.quantizeRow(.q8) (src/core/quant.zig:197-288) over `rows` rows: bit exact. */
int32_t qwc_op_quantize_q8(const float* values, uint32_t rows, uint32_t cols, void* scales, void* codes,
                           void* stream);
/* kernels.linearQuantized with one token (src/core/qwen3_asr/kernels.zig:118-158): out[rows].
 * Formats q4, q5, q8. Alignment (else QWC_INVALID_ARGUMENT, before any launch): `codes` and `x`
 * 16-byte aligned for q4/q8, `codes` 8-byte and `x` 4-byte aligned for q5, `scales` 2-byte. */
int32_t qwc_op_gemv(uint32_t format, const void* scales, const void* codes, uint32_t rows, uint32_t cols,
                    const float* x, float* out, void* stream);
/* kernels.decodeAttentionStepQ8 (src/core/qwen3_asr/kernels.zig:697-767) over
 * `cached` rows of a cache laid out as planes of `max_positions` rows. */
int32_t qwc_op_attention_q8(const float* query, const void* keys_scales, const void* keys_codes,
                            const void* values_scales, const void* values_codes, uint32_t cached, uint32_t heads,
                            uint32_t kv_heads, uint32_t head_dim, float* out, void* stream);
/* Decoder.argmaxLogits (src/core/qwen3_asr/decoder.zig:290-301): first index
 * of the maximum. Uses a device workspace the library allocates per call. */
int32_t qwc_op_argmax(const float* values, uint32_t count, uint32_t* out_index, void* stream);
/* The same argmax with no device allocation: its scratch is a fixed 4 KiB
 * array compiled into the library. No counterpart in the reference; for
 * callers that must not enter the CUDA allocator while decoding, such as a
 * serving process that has handed all free HBM to its weight and KV-cache
 * pools, where an allocation can fail or wait on other work. At most
 * QWC_ARGMAX_NOALLOC_MAX_COUNT values (else QWC_LIMIT_EXCEEDED). The first
 * call on each device looks up the scratch address (cudaGetSymbolAddress),
 * so make it before any stream capture. One scratch per device: calls that
 * overlap on a device (other streams or host threads) race; calls on one
 * stream are ordered. */
#define QWC_ARGMAX_NOALLOC_MAX_COUNT 4194304u
int32_t qwc_op_argmax_noalloc(const float* values, uint32_t count, uint32_t* out_index, void* stream);
/* kernels.linearQuantized (src/core/qwen3_asr/kernels.zig:118-158) for up to
 * 64 independent streams at once on the tensor cores: out[s][r] = sum_k
 * W[r][k] * x[s][k], x as [streams][cols] f32, out as [streams][rows] f32.
 * Each dequantized weight enters as an exact pair of f16 values (hi + lo)
 * and each activation as f16 hi + lo (22 significant bits); products
 * accumulate in f32. Formats q4, q5 and q8; cols must be a multiple of 512;
 * `scales` and `codes` 16-byte aligned. Uses a device workspace the library
 * allocates per call. */
int32_t qwc_op_gemm_streams(uint32_t format, const void* scales, const void* codes, uint32_t rows, uint32_t cols,
                            const float* x, uint32_t streams, float* out, void* stream);
/* math.rmsNormInPlace per row (src/core/math.zig:120-130), out of place. */
int32_t qwc_op_rmsnorm(const float* x, const float* weight, uint32_t width, uint32_t rows, float eps, float* out,
                       void* stream);
/* kernels.ropeInPlace at one position (src/core/qwen3_asr/kernels.zig:495-527). */
int32_t qwc_op_rope(float* x, uint32_t heads, uint32_t head_dim, const float* cos_table, const float* sin_table,
                    uint32_t position, void* stream);
/* kernels.siluMul (src/core/qwen3_asr/kernels.zig:233-239). */
int32_t qwc_op_silu_mul(const float* gate, const float* up, uint32_t n, float* out, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* QWENSCRIBER_CUDA_H */

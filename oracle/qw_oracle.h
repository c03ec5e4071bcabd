/*
 * qw_oracle.h -- CPU restatement of the Qwenscriber decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend in qwenscriber_b200/. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it. The product
 * library never links or calls it.
 *
 * It restates, operation for operation, the reference's Zig CPU path
 * (mattneel/qwenscriber, Zig 0.17-dev, which cannot be built in this
 * environment):
 *   src/core/half_float.zig:14-23        f16 <-> f32 (round to nearest even)
 *   src/core/quant.zig:47-391            q4/q5/q8 group layout, quantizeRow, dequantize, dotRow
 *   src/core/math.zig:27-130             rsqrt, silu, softmax, rmsNormInPlace
 *   src/core/qwen3_asr/kernels.zig       dotF32, linearQuantized, rope, decode attention (f32, q8)
 *   src/core/qwen3_asr/decoder.zig       forwardToken, argmaxLogits, prefill, step, KV layout
 *   src/core/qwen3_asr/model.zig         tied lm_head, scratch, cacheBytes, rope tables
 *   src/core/selftest.zig:73-126         quant_hash known-answer pattern
 *
 * Every function is plain C ABI so tests can bind it with ctypes.
 */
#ifndef QW_ORACLE_H
#define QW_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype.zig:17-24 */
enum { ORC_F32 = 0, ORC_F16 = 1, ORC_BF16 = 2, ORC_Q4 = 16, ORC_Q5 = 17, ORC_Q8 = 18 };

uint16_t orc_to_f16(float value);
float orc_from_f16(uint16_t bits);

uint32_t orc_data_bytes_per_group(int format);
int32_t orc_bias(int format);

void orc_quantize_row(int format, const float* values, size_t cols, uint8_t* scales_out, uint8_t* data_out);
void orc_quantize_rows(int format, const float* values, size_t rows, size_t cols, uint8_t* scales_out,
                       uint8_t* data_out, int threads);
void orc_dequantize_row(int format, const uint8_t* scales, const uint8_t* data, size_t cols, float* out);
float orc_dot_row(int format, const uint8_t* scales, const uint8_t* data, const float* x, size_t cols);
float orc_dot_f32(const float* a, const float* b, size_t n);

/* kernels.zig:118-158; rows processed in parallel (threads <= 1: serial). */
int32_t orc_linear_quantized(float* out, const float* x, int format, const uint8_t* scales, const uint8_t* data,
                             uint32_t rows, uint32_t cols, uint32_t tokens, int threads);

void orc_rmsnorm(float* x, const float* weight, uint32_t width, uint32_t tokens, float eps);
void orc_silu_mul(float* out, const float* gate, const float* up, size_t n);
float orc_silu(float x);
void orc_softmax(float* row, size_t n);
float orc_inverse_frequency(uint32_t index, uint32_t head_dim, float theta);
float orc_pow_f32(float x, float y);
void orc_build_rope_tables(float* cos_table, float* sin_table, uint32_t half, float theta, uint32_t max_positions,
                           uint32_t stride);
void orc_rope(float* rotated, const uint32_t* positions, uint32_t n_positions, uint32_t heads, uint32_t head_dim,
              const float* cos_table, const float* sin_table, uint32_t table_stride);
int32_t orc_decode_attention_f32(float* out, const float* query, const float* keys, const float* values,
                                 uint32_t cached, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, float* scores);
int32_t orc_decode_attention_q8(float* out, const float* query, const uint8_t* keys_scales, const uint8_t* keys_codes,
                                const uint8_t* values_scales, const uint8_t* values_codes, uint32_t cached,
                                uint32_t heads, uint32_t kv_heads, uint32_t head_dim, float* scores);
uint32_t orc_argmax(const float* values, size_t n);
uint64_t orc_quant_hash(void);

/* ---- the decoder (decoder.zig) over borrowed weight payloads ---- */
typedef struct OrcModel OrcModel;

/* config: the 160-byte Config of model_config.zig:110-177. cache_format: 0 = f32, 1 = q8. */
OrcModel* orc_model_new(const void* config, uint32_t config_len, uint32_t cache_format);
void orc_model_free(OrcModel* model);
void orc_model_set_threads(OrcModel* model, int threads);
/* Borrows payload (scales plane, 16-byte padding, codes plane) until orc_model_free. */
int32_t orc_model_set_tensor(OrcModel* model, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows,
                             uint32_t cols, const void* payload, size_t len);
int32_t orc_model_finish(OrcModel* model);
void orc_decoder_reset(OrcModel* model);
uint32_t orc_decoder_position(const OrcModel* model);
/* Test and timing support (no reference counterpart): replaces the q8 cache
 * contents (keys, values: the whole cache, len bytes each) and moves the
 * decoder to `position`, as if that many positions had been prefilled. */
int32_t orc_decoder_set_state(OrcModel* model, const uint8_t* keys, const uint8_t* values, uint64_t len,
                              uint32_t position);
int32_t orc_forward_token(OrcModel* model, uint32_t token, const float* audio_row, int want_logits);
uint32_t orc_argmax_logits(const OrcModel* model);
int32_t orc_prefill(OrcModel* model, const uint32_t* tokens, uint32_t n_tokens, const float* audio, uint32_t audio_steps,
                    uint32_t* next_out);
int32_t orc_step(OrcModel* model, uint32_t token, uint32_t* next_out);
const float* orc_logits(const OrcModel* model);
const float* orc_hidden(const OrcModel* model);
/* Scratch of the last forward pass's last layer: 0 hidden, 1 query (normed,
 * rotated), 2 key (normed, rotated), 3 value, 4 attention_out, 5 silu(gate)*up. */
const float* orc_scratch(const OrcModel* model, int which, uint32_t* count_out);
const uint8_t* orc_cache_keys_q8(const OrcModel* model, uint64_t* len_out);
const uint8_t* orc_cache_values_q8(const OrcModel* model, uint64_t* len_out);
const float* orc_rope_cos(const OrcModel* model);
const float* orc_rope_sin(const OrcModel* model);

/* ---- the audio tower and projector (qw_oracle_audio.cpp; model.zig:445-870,
 * kernels.zig:210-487, math.zig:46-116) ---- */
float orc_erf(float x);
float orc_gelu(float x);
void orc_layer_norm(float* x, const float* weight, const float* bias, uint32_t width, uint32_t tokens, float eps);
/* out [out_ch][h'][w'], input [in_ch][in_h][in_w], weights [out_ch][in_ch][3][3] (f16 bits). */
int32_t orc_conv3x3_stride2_gelu(float* out, const float* input, const uint16_t* weights, const float* bias,
                                 uint32_t out_ch, uint32_t in_ch, uint32_t in_h, uint32_t in_w, int threads);
int32_t orc_audio_attention_window(float* out, uint32_t out_stride, const float* q, uint32_t q_stride, const float* k,
                                   uint32_t k_stride, const float* v, uint32_t v_stride, uint32_t window_start,
                                   uint32_t window_length, uint32_t heads, uint32_t head_dim);
void orc_add_sinusoidal_position(float* row, uint32_t step, uint32_t channels);

typedef struct OrcAudio OrcAudio;
OrcAudio* orc_audio_new(const void* config, uint32_t config_len);
void orc_audio_free(OrcAudio* audio);
void orc_audio_set_threads(OrcAudio* audio, int threads);
/* Borrows payload until orc_audio_free: f32 vectors (rows 1), f16 convolution
 * weights [out][in * 9], q4/q5/q8 matrix container payloads. */
int32_t orc_audio_set_tensor(OrcAudio* audio, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows,
                             uint32_t cols, const void* payload, size_t len);
int32_t orc_audio_finish(OrcAudio* audio);
uint32_t orc_audio_packed_steps(const OrcAudio* audio, uint32_t frames);
/* log_mel: [mel_bins][frames] row major. */
int32_t orc_audio_encode_conv(OrcAudio* audio, const float* log_mel, uint32_t frames, uint32_t* steps_out);
int32_t orc_audio_encode_tower(OrcAudio* audio, uint32_t steps);
int32_t orc_audio_project_steps(OrcAudio* audio, uint32_t steps, float* out);
int32_t orc_audio_project(OrcAudio* audio, const float* log_mel, uint32_t frames, float* out, uint64_t capacity_floats,
                          uint32_t* steps_out);
const float* orc_audio_encoded(const OrcAudio* audio, uint32_t* count_out);

#ifdef __cplusplus
}
#endif
#endif

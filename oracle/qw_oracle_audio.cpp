// qw_oracle_audio.cpp -- CPU restatement of the Qwen3-ASR audio tower and
// projector (TEST INFRASTRUCTURE ONLY: the parity checker of the CUDA audio
// path; the product library never links it).
//
// Restated operation for operation, in the reference's order, from
//   src/core/qwen3_asr/model.zig:445-744   projectAudio, encodeConvStage, convolveAndPack,
//                                          projectConvStep, runAudioTower, runProjector,
//                                          addSinusoidalPosition, projectQkv,
//                                          runWindowedAttention, projectAttentionOutput, activateFfn
//   src/core/qwen3_asr/kernels.zig:210-487 addBias, addInPlace, layerNorm(Into),
//                                          conv3x3Stride2Gelu, convolveChannel, convolvePlane,
//                                          audioAttentionWindow
//   src/core/math.zig:46-116               erf, gelu, softmaxInPlace, layerNormInPlace
//   src/core/model_config.zig:84-240       postConvolutionSteps, audioChunkFrames/Steps,
//                                          audioFrequencyBinsAfterConvolutions, packedStepCount
//   src/core/qwen3_asr/layout.zig:150-262  the tower's tensor inventory and shapes
// Built with -ffp-contract=off like the decoder restatement: every product
// and sum is rounded where the reference rounds it.

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <map>
#include <thread>
#include <vector>

#include "qw_oracle.h"

#define QW_ORACLE_TRY(expr)        \
  do {                             \
    const int32_t _s = (expr);     \
    if (_s != kOk) return _s;      \
  } while (0)

namespace {

constexpr int32_t kOk = 0;
constexpr int32_t kInvalidArgument = -1;
constexpr int32_t kShapeMismatch = -7;
constexpr int32_t kLimitExceeded = -9;
constexpr int32_t kNotFound = -10;
constexpr int32_t kUnsupportedModel = -13;
constexpr int32_t kAudioTooLong = -14;
constexpr uint32_t kGroup = 64;
constexpr uint32_t kCapacityFrames = 3000;  // mel.zig:55-58
constexpr uint32_t kAudioLayerBase = 1024;  // container.zig:307

// model_config.zig:110-177, byte for byte (the audio fields are read here).
struct Config {
  uint8_t magic[8];
  uint32_t format_version, architecture;
  uint32_t audio_d_model, audio_layers, audio_attention_heads, audio_ffn_dim, audio_downsample_hidden_size,
      audio_n_window, audio_n_window_infer, audio_max_position_steps, audio_output_dim, mel_bins;
  float audio_layer_norm_eps;
  uint32_t rest[25];
};
static_assert(sizeof(Config) == 160, "model_config.zig:364");

// container.zig:334-362
enum Kind : uint32_t {
  kConv1W = 1, kConv1B, kConv2W, kConv2B, kConv3W, kConv3B, kConvOutW, kFinalNormW, kFinalNormB,
  kQW, kQB, kKW, kKB, kVW, kVB, kOutW, kOutB, kAttnNormW, kAttnNormB, kFfnInW, kFfnInB, kFfnOutW, kFfnOutB,
  kLayerNormW, kLayerNormB, kProjInW, kProjInB, kProjOutW, kProjOutB,
};

// model_config.zig:84-90
uint32_t post_conv_steps(uint32_t frames) {
  if (frames == 0) return 0;
  uint32_t s = frames;
  for (int i = 0; i < 3; ++i) s = (s - 1) / 2 + 1;
  return s;
}

template <typename Fn>
void parallel_for(size_t n, int threads, Fn fn) {
  if (threads <= 1 || n < 2) {
    fn(size_t(0), n);
    return;
  }
  const size_t count = std::min<size_t>(static_cast<size_t>(threads), n);
  std::vector<std::thread> pool;
  for (size_t t = 0; t < count; ++t) {
    const size_t begin = n * t / count, end = n * (t + 1) / count;
    pool.emplace_back([=] { fn(begin, end); });
  }
  for (auto& th : pool) th.join();
}

struct Tensor {
  uint32_t format = 0, rows = 0, cols = 0;
  const uint8_t* payload = nullptr;
  size_t len = 0;
  const uint8_t* scales = nullptr;  // quantized: scale plane
  const uint8_t* data = nullptr;    // quantized: code plane
};

struct AudioLayer {
  const Tensor *q, *k, *v, *out, *ffn_in, *ffn_out;
  const float *q_b, *k_b, *v_b, *out_b, *attn_norm_w, *attn_norm_b, *ffn_in_b, *ffn_out_b, *norm_w, *norm_b;
};

}  // namespace

struct OrcAudio {
  Config c{};
  int threads = 1;
  bool finished = false;
  std::map<std::pair<uint32_t, uint32_t>, Tensor> tensors;
  const uint16_t *conv_w[3] = {nullptr, nullptr, nullptr};
  const float *conv_b[3] = {nullptr, nullptr, nullptr};
  const Tensor* conv_out = nullptr;
  const float *final_w = nullptr, *final_b = nullptr;
  const Tensor *proj_in = nullptr, *proj_out = nullptr;
  const float *proj_in_b = nullptr, *proj_out_b = nullptr;
  std::vector<AudioLayer> layers;
  // model.zig scratch: encoder (steps x d_model), the per-chunk planes.
  std::vector<float> encoder, normed, block, qkv, ffn, mel_chunk, conv1, conv2, conv3, flat, scores;
  uint32_t steps = 0;

  uint32_t chunk_frames() const { return c.audio_n_window * 2; }                 // model_config.zig:196-198
  uint32_t chunk_steps() const { return post_conv_steps(chunk_frames()); }      // :219-224
  uint32_t freq_bins() const {                                                   // :206-211
    uint32_t b = c.mel_bins;
    for (int i = 0; i < 3; ++i) b = (b - 1) / 2 + 1;
    return b;
  }
  uint32_t conv_out_features() const { return c.audio_downsample_hidden_size * freq_bins(); }  // :214-216
  uint32_t packed_steps(uint32_t frames) const {                                 // :235-239
    const uint32_t chunk = chunk_frames();
    return (frames / chunk) * post_conv_steps(chunk) + post_conv_steps(frames % chunk);
  }
  uint32_t max_window() const { return (c.audio_n_window_infer / chunk_frames()) * chunk_steps(); }  // model.zig:243-246
  uint32_t head_dim() const { return c.audio_d_model / c.audio_attention_heads; }
};

namespace {

const float* f32_of(const Tensor* t) { return reinterpret_cast<const float*>(t->payload); }

// kernels.zig:182-206 (the quantized arm): out[tokens][rows] = W x.
int32_t apply(const OrcAudio* a, const Tensor* w, float* out, const float* x, uint32_t tokens) {
  return orc_linear_quantized(out, x, static_cast<int>(w->format), w->scales, w->data, w->rows, w->cols, tokens,
                              a->threads);
}

// kernels.zig:210-218
void add_bias(float* x, const float* bias, uint32_t rows, uint32_t tokens) {
  for (uint32_t t = 0; t < tokens; ++t) {
    float* row = x + size_t(t) * rows;
    for (uint32_t i = 0; i < rows; ++i) row[i] = row[i] + bias[i];
  }
}

// kernels.zig:221-230 (the 4-lane vector add is element-wise).
void add_in_place(float* x, const float* y, size_t n) {
  for (size_t i = 0; i < n; ++i) x[i] = x[i] + y[i];
}

// math.zig:99-116
void layer_norm_row(float* row, const float* weight, const float* bias, uint32_t n, float eps) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < n; ++i) sum = sum + row[i];
  const float mean = sum / static_cast<float>(n);
  float sum_squares = 0.0f;
  for (uint32_t i = 0; i < n; ++i) {
    const float centered = row[i] - mean;
    sum_squares = sum_squares + centered * centered;
  }
  const float variance = sum_squares / static_cast<float>(n);
  const float inverse_std = 1.0f / std::sqrt(variance + eps);
  for (uint32_t i = 0; i < n; ++i) row[i] = (row[i] - mean) * inverse_std * weight[i] + bias[i];
}

// kernels.zig:259-272
void layer_norm_into(float* target, const float* source, const float* w, const float* b, uint32_t width,
                     uint32_t tokens, float eps) {
  std::memcpy(target, source, size_t(width) * tokens * 4);
  for (uint32_t t = 0; t < tokens; ++t) layer_norm_row(target + size_t(t) * width, w, b, width, eps);
}

// kernels.zig:388-432: one input channel's taps added into an output plane.
void convolve_plane(float* out, const float* input, const uint16_t* weights, uint32_t in_h, uint32_t in_w) {
  const uint32_t out_h = (in_h - 1) / 2 + 1, out_w = (in_w - 1) / 2 + 1;
  float kw[9];
  for (int i = 0; i < 9; ++i) kw[i] = orc_from_f16(weights[i]);
  for (uint32_t r = 0; r < out_h; ++r) {
    for (uint32_t col = 0; col < out_w; ++col) {
      float acc = 0.0f;
      for (int kr = 0; kr < 3; ++kr) {
        const int64_t ir = int64_t(r) * 2 + kr - 1;
        if (ir < 0 || ir >= int64_t(in_h)) continue;
        for (int kc = 0; kc < 3; ++kc) {
          const int64_t ic = int64_t(col) * 2 + kc - 1;
          if (ic < 0 || ic >= int64_t(in_w)) continue;
          acc = acc + kw[kr * 3 + kc] * input[size_t(ir) * in_w + size_t(ic)];
        }
      }
      out[size_t(r) * out_w + col] = out[size_t(r) * out_w + col] + acc;
    }
  }
}

}  // namespace

extern "C" {

// math.zig:46-60
float orc_erf(float x) {
  const float sign = x < 0.0f ? -1.0f : 1.0f;
  const float m = std::fabs(x);
  const float t = 1.0f / (1.0f + 0.5f * m);
  const float poly =
      1.00002368f +
      t * (0.37409196f +
           t * (0.09678418f +
                t * (-0.18628806f + t * (0.27886807f + t * (-1.13520398f + t * (1.48851587f +
                                                                                 t * (-0.82215223f + t * 0.17087277f)))))));
  const float tau = t * std::exp(-m * m - 1.26551223f + t * poly);
  return sign * (1.0f - tau);
}

// math.zig:63-66
float orc_gelu(float x) {
  const float inverse_sqrt_two = 0.70710678f;
  return 0.5f * x * (1.0f + orc_erf(x * inverse_sqrt_two));
}

// math.zig:99-116 over `tokens` rows, in place (kernels.zig:242-256).
void orc_layer_norm(float* x, const float* weight, const float* bias, uint32_t width, uint32_t tokens, float eps) {
  for (uint32_t t = 0; t < tokens; ++t) layer_norm_row(x + size_t(t) * width, weight, bias, width, eps);
}

// kernels.zig:332-362: out [out_ch][out_h][out_w], input [in_ch][in_h][in_w],
// weights [out_ch][in_ch][3][3] f16 bits.
int32_t orc_conv3x3_stride2_gelu(float* out, const float* input, const uint16_t* weights, const float* bias,
                                 uint32_t out_ch, uint32_t in_ch, uint32_t in_h, uint32_t in_w, int threads) {
  if (!out || !input || !weights || !bias || in_h == 0 || in_w == 0) return kShapeMismatch;
  const uint32_t out_h = (in_h - 1) / 2 + 1, out_w = (in_w - 1) / 2 + 1;
  const size_t in_plane = size_t(in_h) * in_w, out_plane = size_t(out_h) * out_w;
  parallel_for(out_ch, threads, [&](size_t begin, size_t end) {
    for (size_t oc = begin; oc < end; ++oc) {
      float* plane = out + oc * out_plane;
      for (size_t i = 0; i < out_plane; ++i) plane[i] = bias[oc];  // convolveChannel's @memset
      for (uint32_t ic = 0; ic < in_ch; ++ic) {
        convolve_plane(plane, input + ic * in_plane, weights + (oc * in_ch + ic) * 9, in_h, in_w);
      }
      for (size_t i = 0; i < out_plane; ++i) plane[i] = orc_gelu(plane[i]);
    }
  });
  return kOk;
}

// kernels.zig:435-487
int32_t orc_audio_attention_window(float* out, uint32_t out_stride, const float* q, uint32_t q_stride, const float* k,
                                   uint32_t k_stride, const float* v, uint32_t v_stride, uint32_t window_start,
                                   uint32_t window_length, uint32_t heads, uint32_t head_dim) {
  std::vector<float> scores(window_length);
  const float scaling = 1.0f / std::sqrt(static_cast<float>(head_dim));
  for (uint32_t h = 0; h < heads; ++h) {
    for (uint32_t qi = 0; qi < window_length; ++qi) {
      const float* qr = q + size_t(window_start + qi) * q_stride + size_t(h) * head_dim;
      for (uint32_t key = 0; key < window_length; ++key) {
        const float* kr = k + size_t(window_start + key) * k_stride + size_t(h) * head_dim;
        scores[key] = orc_dot_f32(qr, kr, head_dim) * scaling;
      }
      orc_softmax(scores.data(), window_length);
      float* orow = out + size_t(window_start + qi) * out_stride + size_t(h) * head_dim;
      for (uint32_t i = 0; i < head_dim; ++i) orow[i] = 0.0f;
      for (uint32_t key = 0; key < window_length; ++key) {
        const float* vr = v + size_t(window_start + key) * v_stride + size_t(h) * head_dim;
        const float w = scores[key];
        for (uint32_t i = 0; i < head_dim; ++i) orow[i] = orow[i] + vr[i] * w;
      }
    }
  }
  return kOk;
}

// model.zig:750-762: concat(sin, cos) of step * exp(-ln(10000)/(half-1) * i),
// computed in f64 and added to the row in f32.
void orc_add_sinusoidal_position(float* row, uint32_t step, uint32_t channels) {
  const uint32_t half = channels / 2;
  const double increment = std::log(10000.0) / (static_cast<double>(half) - 1.0);
  const double position = static_cast<double>(step);
  for (uint32_t i = 0; i < half; ++i) {
    const double inverse_timescale = std::exp(-increment * static_cast<double>(i));
    const double angle = position * inverse_timescale;
    row[i] = row[i] + static_cast<float>(std::sin(angle));
    row[half + i] = row[half + i] + static_cast<float>(std::cos(angle));
  }
}

OrcAudio* orc_audio_new(const void* config, uint32_t config_len) {
  if (!config || config_len != sizeof(Config)) return nullptr;
  OrcAudio* a = new OrcAudio();
  std::memcpy(&a->c, config, sizeof(Config));
  return a;
}

void orc_audio_free(OrcAudio* a) { delete a; }

void orc_audio_set_threads(OrcAudio* a, int threads) { a->threads = threads < 1 ? 1 : threads; }

// Borrows payload until orc_audio_free. Vectors are f32 (rows = 1), the
// convolution weights f16 [out][in * 9], matrices q4/q5/q8 container
// payloads (scale plane, 16-byte pad, code plane; quant.zig:144-176).
int32_t orc_audio_set_tensor(OrcAudio* a, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows,
                             uint32_t cols, const void* payload, size_t len) {
  if (a->finished || !payload || kind < kConv1W || kind > kProjOutB) return kInvalidArgument;
  if (a->tensors.count({kind, layer})) return kInvalidArgument;
  Tensor t;
  t.format = format;
  t.rows = rows;
  t.cols = cols;
  t.payload = static_cast<const uint8_t*>(payload);
  t.len = len;
  if (format == ORC_Q4 || format == ORC_Q5 || format == ORC_Q8) {
    if (cols % kGroup != 0) return kShapeMismatch;
    const size_t groups = size_t(rows) * (cols / kGroup);
    const size_t codes_off = (groups * 2 + 15) / 16 * 16;
    if (len < codes_off + groups * orc_data_bytes_per_group(static_cast<int>(format))) return kShapeMismatch;
    t.scales = t.payload;
    t.data = t.payload + codes_off;
  } else if (format == ORC_F16) {
    if (len < size_t(rows) * cols * 2) return kShapeMismatch;
  } else if (format == ORC_F32) {
    if (len < size_t(rows) * cols * 4) return kShapeMismatch;
  } else {
    return kUnsupportedModel;
  }
  a->tensors.emplace(std::make_pair(kind, layer), t);
  return kOk;
}

// model.zig:965-990 (loadAudioLayers) with layout.zig:150-262's shapes.
int32_t orc_audio_finish(OrcAudio* a) {
  const Config& c = a->c;
  const uint32_t d = c.audio_d_model, ch = c.audio_downsample_hidden_size, ffn = c.audio_ffn_dim;
  if (d == 0 || c.audio_attention_heads == 0 || d % c.audio_attention_heads != 0 || c.audio_n_window == 0) {
    return kShapeMismatch;
  }
  int32_t st = kOk;
  auto find = [&](uint32_t kind, uint32_t layer) -> const Tensor* {
    auto it = a->tensors.find({kind, layer});
    if (it == a->tensors.end()) {
      if (st == kOk) st = kNotFound;  // MissingTensor
      return nullptr;
    }
    return &it->second;
  };
  auto vec = [&](uint32_t kind, uint32_t layer, uint32_t width) -> const float* {
    const Tensor* t = find(kind, layer);
    if (!t) return nullptr;
    if (t->format != ORC_F32 || size_t(t->rows) * t->cols != width) {
      if (st == kOk) st = kShapeMismatch;
      return nullptr;
    }
    return f32_of(t);
  };
  auto mat = [&](uint32_t kind, uint32_t layer, uint32_t rows, uint32_t cols) -> const Tensor* {
    const Tensor* t = find(kind, layer);
    if (!t) return nullptr;
    if (!(t->format == ORC_Q4 || t->format == ORC_Q5 || t->format == ORC_Q8) || t->rows != rows || t->cols != cols) {
      if (st == kOk) st = kShapeMismatch;
      return nullptr;
    }
    return t;
  };
  const uint32_t conv_kinds[3] = {kConv1W, kConv2W, kConv3W};
  for (int i = 0; i < 3; ++i) {
    const Tensor* t = find(conv_kinds[i], 0);
    const uint32_t in = i == 0 ? 1u : ch;
    if (t && (t->format != ORC_F16 || t->rows != ch || t->cols != in * 9)) st = st == kOk ? kShapeMismatch : st;
    if (t) a->conv_w[i] = reinterpret_cast<const uint16_t*>(t->payload);
    a->conv_b[i] = vec(conv_kinds[i] + 1, 0, ch);
  }
  a->conv_out = mat(kConvOutW, 0, d, a->conv_out_features());
  a->final_w = vec(kFinalNormW, 0, d);
  a->final_b = vec(kFinalNormB, 0, d);
  a->proj_in = mat(kProjInW, 0, d, d);
  a->proj_in_b = vec(kProjInB, 0, d);
  a->proj_out = mat(kProjOutW, 0, c.audio_output_dim, d);
  a->proj_out_b = vec(kProjOutB, 0, c.audio_output_dim);
  a->layers.resize(c.audio_layers);
  for (uint32_t i = 0; i < c.audio_layers; ++i) {
    const uint32_t L = kAudioLayerBase + i;
    AudioLayer& l = a->layers[i];
    l.q = mat(kQW, L, d, d);
    l.q_b = vec(kQB, L, d);
    l.k = mat(kKW, L, d, d);
    l.k_b = vec(kKB, L, d);
    l.v = mat(kVW, L, d, d);
    l.v_b = vec(kVB, L, d);
    l.out = mat(kOutW, L, d, d);
    l.out_b = vec(kOutB, L, d);
    l.attn_norm_w = vec(kAttnNormW, L, d);
    l.attn_norm_b = vec(kAttnNormB, L, d);
    l.ffn_in = mat(kFfnInW, L, ffn, d);
    l.ffn_in_b = vec(kFfnInB, L, ffn);
    l.ffn_out = mat(kFfnOutW, L, d, ffn);
    l.ffn_out_b = vec(kFfnOutB, L, d);
    l.norm_w = vec(kLayerNormW, L, d);
    l.norm_b = vec(kLayerNormB, L, d);
  }
  if (st != kOk) return st;
  const uint32_t max_steps = a->packed_steps(kCapacityFrames);
  a->encoder.assign(size_t(max_steps) * d, 0.0f);
  a->normed.assign(size_t(max_steps) * d, 0.0f);
  a->block.assign(size_t(max_steps) * d, 0.0f);
  a->qkv.assign(size_t(max_steps) * 3 * d, 0.0f);
  a->ffn.assign(size_t(max_steps) * std::max(ffn, d), 0.0f);
  a->finished = true;
  return kOk;
}

uint32_t orc_audio_packed_steps(const OrcAudio* a, uint32_t frames) { return a->packed_steps(frames); }

// model.zig:476-485 + 506-612: per chunk, the convolution stack, then every
// valid time step through conv_out and the sinusoidal position.
int32_t orc_audio_encode_conv(OrcAudio* a, const float* log_mel, uint32_t frames, uint32_t* steps_out) {
  if (!a->finished) return kInvalidArgument;
  const Config& c = a->c;
  const uint32_t steps = a->packed_steps(frames);
  if (steps > a->packed_steps(kCapacityFrames) || frames > kCapacityFrames) return kAudioTooLong;
  if (frames == 0) return kShapeMismatch;
  const uint32_t cf = a->chunk_frames(), cs = a->chunk_steps(), bins = a->freq_bins();
  const uint32_t ch = c.audio_downsample_hidden_size, d = c.audio_d_model, feats = a->conv_out_features();
  const uint32_t h1 = (c.mel_bins - 1) / 2 + 1, w1 = (cf - 1) / 2 + 1;
  const uint32_t h2 = (h1 - 1) / 2 + 1, w2 = (w1 - 1) / 2 + 1;
  a->mel_chunk.assign(size_t(c.mel_bins) * cf, 0.0f);
  a->conv1.assign(size_t(ch) * h1 * w1, 0.0f);
  a->conv2.assign(size_t(ch) * h2 * w2, 0.0f);
  a->conv3.assign(size_t(ch) * bins * cs, 0.0f);
  a->flat.assign(feats, 0.0f);
  const uint32_t chunk_count = (frames + cf - 1) / cf;
  uint32_t packed = 0;
  for (uint32_t chunk = 0; chunk < chunk_count; ++chunk) {
    const uint32_t start = chunk * cf;
    const uint32_t valid = std::min(frames > start ? frames - start : 0u, cf);
    std::fill(a->mel_chunk.begin(), a->mel_chunk.end(), 0.0f);
    for (uint32_t b = 0; b < c.mel_bins; ++b) {
      std::memcpy(&a->mel_chunk[size_t(b) * cf], log_mel + size_t(b) * frames + start, size_t(valid) * 4);
    }
    orc_conv3x3_stride2_gelu(a->conv1.data(), a->mel_chunk.data(), a->conv_w[0], a->conv_b[0], ch, 1, c.mel_bins, cf,
                             a->threads);
    orc_conv3x3_stride2_gelu(a->conv2.data(), a->conv1.data(), a->conv_w[1], a->conv_b[1], ch, ch, h1, w1, a->threads);
    orc_conv3x3_stride2_gelu(a->conv3.data(), a->conv2.data(), a->conv_w[2], a->conv_b[2], ch, ch, h2, w2, a->threads);
    const uint32_t valid_steps = post_conv_steps(valid);
    for (uint32_t step = 0; step < cs && step < valid_steps; ++step) {
      float* row = &a->encoder[size_t(packed) * d];
      // model.zig:580-597: flat[c * bins + f] = conv3[c][f][step].
      for (uint32_t cc = 0; cc < ch; ++cc) {
        for (uint32_t f = 0; f < bins; ++f) a->flat[size_t(cc) * bins + f] = a->conv3[(size_t(cc) * bins + f) * cs + step];
      }
      const int32_t st = apply(a, a->conv_out, row, a->flat.data(), 1);
      if (st != kOk) return st;
      orc_add_sinusoidal_position(row, step, d);
      ++packed;
    }
  }
  if (packed != steps) return kShapeMismatch;
  a->steps = steps;
  if (steps_out) *steps_out = steps;
  return kOk;
}

// model.zig:622-704 (runAudioTower) with projectQkv :764-782,
// runWindowedAttention :788-817, projectAttentionOutput :820-845 and
// activateFfn :849-870; then the final LayerNorm.
int32_t orc_audio_encode_tower(OrcAudio* a, uint32_t steps) {
  if (!a->finished || steps == 0 || steps > a->steps) return kInvalidArgument;
  const Config& c = a->c;
  const uint32_t d = c.audio_d_model, ffn = c.audio_ffn_dim, window = a->max_window();
  const float eps = c.audio_layer_norm_eps;
  float* enc = a->encoder.data();
  float* normed = a->normed.data();
  float* block = a->block.data();
  float* qkv = a->qkv.data();
  const size_t total = size_t(steps) * d;
  std::vector<float> proj(total);
  for (const AudioLayer& l : a->layers) {
    layer_norm_into(normed, enc, l.attn_norm_w, l.attn_norm_b, d, steps, eps);
    // projectQkv: one row per step, [q | k | v] with stride 3d. Each output
    // is dotF32(dequantized row, input row) whatever the token count.
    const Tensor* w3[3] = {l.q, l.k, l.v};
    const float* b3[3] = {l.q_b, l.k_b, l.v_b};
    for (int j = 0; j < 3; ++j) {
      QW_ORACLE_TRY(apply(a, w3[j], proj.data(), normed, steps));
      add_bias(proj.data(), b3[j], d, steps);
      for (uint32_t s = 0; s < steps; ++s) {
        std::memcpy(qkv + size_t(s) * 3 * d + size_t(j) * d, proj.data() + size_t(s) * d, size_t(d) * 4);
      }
    }
    for (uint32_t w0 = 0; w0 < steps;) {
      const uint32_t len = std::min(window, steps - w0);
      orc_audio_attention_window(block, d, qkv, 3 * d, qkv + d, 3 * d, qkv + 2 * d, 3 * d, w0, len,
                                 c.audio_attention_heads, a->head_dim());
      w0 += len;
    }
    QW_ORACLE_TRY(apply(a, l.out, normed, block, steps));
    add_bias(normed, l.out_b, d, steps);
    std::memcpy(block, normed, total * 4);
    add_in_place(enc, block, total);

    layer_norm_into(normed, enc, l.norm_w, l.norm_b, d, steps, eps);
    float* wide = a->ffn.data();
    QW_ORACLE_TRY(apply(a, l.ffn_in, wide, normed, steps));
    add_bias(wide, l.ffn_in_b, ffn, steps);
    for (size_t i = 0; i < size_t(steps) * ffn; ++i) wide[i] = orc_gelu(wide[i]);
    QW_ORACLE_TRY(apply(a, l.ffn_out, block, wide, steps));
    add_bias(block, l.ffn_out_b, d, steps);
    add_in_place(enc, block, total);
  }
  orc_layer_norm(enc, a->final_w, a->final_b, d, steps, eps);
  return kOk;
}

// model.zig:707-733: linear, GELU, linear.
int32_t orc_audio_project_steps(OrcAudio* a, uint32_t steps, float* out) {
  if (!a->finished || steps == 0 || steps > a->steps || !out) return kInvalidArgument;
  const uint32_t d = a->c.audio_d_model, hidden = a->c.audio_output_dim;
  float* mid = a->ffn.data();
  QW_ORACLE_TRY(apply(a, a->proj_in, mid, a->encoder.data(), steps));
  add_bias(mid, a->proj_in_b, d, steps);
  for (size_t i = 0; i < size_t(steps) * d; ++i) mid[i] = orc_gelu(mid[i]);
  QW_ORACLE_TRY(apply(a, a->proj_out, out, mid, steps));
  add_bias(out, a->proj_out_b, hidden, steps);
  return kOk;
}

// model.zig:451-460
int32_t orc_audio_project(OrcAudio* a, const float* log_mel, uint32_t frames, float* out, uint64_t capacity_floats,
                          uint32_t* steps_out) {
  uint32_t steps = 0;
  QW_ORACLE_TRY(orc_audio_encode_conv(a, log_mel, frames, &steps));
  QW_ORACLE_TRY(orc_audio_encode_tower(a, steps));
  if (capacity_floats < uint64_t(steps) * a->c.audio_output_dim) return kLimitExceeded;
  QW_ORACLE_TRY(orc_audio_project_steps(a, steps, out));
  if (steps_out) *steps_out = steps;
  return kOk;
}

// model.zig:496-499 (encodedSteps): the packed sequence after the last
// stage that ran (the conv stage, or the tower with its final norm).
const float* orc_audio_encoded(const OrcAudio* a, uint32_t* count_out) {
  if (count_out) *count_out = a->steps * a->c.audio_d_model;
  return a->encoder.data();
}

}  // extern "C"

// qwc_audio_model.h -- the audio tower and projector of one model handle:
// device weights, their TMA descriptors, scratch sized for the longest clip,
// and the launch sequence of Model.projectAudio (src/core/qwen3_asr/model.zig:445-744).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <functional>
#include <vector>

namespace qwc {

// A tensor's device payload as the handle holds it (the container payload:
// f32 values, f16 values, or a quantized scale plane and code plane).
struct AudioTensorView {
  uint32_t format = 0, rows = 0, cols = 0;
  const uint8_t* dev = nullptr;
  uint64_t scales_offset = 0, codes_offset = 0;
};

// The tower's geometry (abi.zig:296-340's AudioConfig plus the scratch bounds).
struct AudioGeometry {
  uint32_t d_model, layers, heads, head_dim, ffn, channels, n_window, n_window_infer, chunk_frames, bins,
      conv_features, chunk_steps, max_position_steps, output_dim, mel_bins;
  float eps;
  uint32_t window;      // packed steps per attention window (model.zig:243-246)
  uint32_t max_frames;  // mel frames one clip may hold (mel.zig:55-58)
  uint32_t max_chunks, max_steps;
};

// packedStepCount (model_config.zig:235-239) and its per-chunk part (:84-90).
uint32_t audio_post_conv_steps(uint32_t frames);
uint32_t audio_packed_steps(const AudioGeometry& g, uint32_t frames);

class AudioModel {
 public:
  using Find = std::function<bool(uint32_t kind, uint32_t layer, AudioTensorView* out)>;

  AudioModel() = default;
  AudioModel(const AudioModel&) = delete;
  AudioModel& operator=(const AudioModel&) = delete;
  ~AudioModel();

  // Resolves every tower tensor (layout.zig:150-262 shapes), repacks the
  // convolution weights, builds the TMA descriptors and allocates scratch.
  // Returns a QWC_* status: NOT_FOUND for a missing tensor, SHAPE_MISMATCH for
  // a wrong shape or storage, UNSUPPORTED_MODEL for geometry these kernels do
  // not take.
  int32_t build(const AudioGeometry& geometry, const Find& find, int sms);

  // One clip: mel [mel_bins][frames] on the device -> out [steps][output_dim]
  // on the device, every launch on `stream`. Returns a QWC_* status after the
  // stream has drained (the GEMMs' bounded waits report through an error word).
  int32_t run(const float* mel_dev, uint32_t frames, float* out_dev, cudaStream_t stream, uint64_t timeout_ns,
              uint32_t* steps_out, bool sync = true);
  // Kernel launches of the last run.
  uint64_t launches() const { return launches_; }
  int32_t check_error(cudaStream_t stream);

  // [steps][d_model] on the device: the conv stage's packed sequence
  // (encodeConvStage) and the tower's output after its final LayerNorm.
  const float* conv_stage() const { return static_cast<const float*>(conv_stage_); }
  const float* tower() const { return static_cast<const float*>(x_); }
  // Device bytes of the tower's scratch, and of its weight copies made here.
  uint64_t scratch_bytes() const { return scratch_bytes_; }
  float* mel_buffer() const { return static_cast<float*>(mel_); }

  AudioGeometry g{};

 private:
  struct Mat {
    alignas(64) uint8_t codes[128];
    alignas(64) uint8_t scales[128];
    uint32_t rows = 0, cols = 0, format = 0;
  };
  struct Layer {
    Mat q, k, v, o, ffn_in, ffn_out;
    const float *attn_norm_w, *attn_norm_b, *o_b, *ffn_in_b, *ffn_out_b, *norm_w, *norm_b;
  };
  void* alloc(size_t bytes);
  // Enqueues one clip's launches on `stream` (the body of run(), captured
  // into a graph there).
  int32_t enqueue(const float* mel_dev, uint32_t frames, float* out_dev, cudaStream_t stream, uint64_t timeout_ns);

  struct Graph {
    uint32_t frames;
    const float* mel;
    float* out;
    uint64_t timeout_ns;
    cudaGraphExec_t exec;
    uint64_t launches;
  };
  static constexpr size_t kMaxGraphs = 8;
  std::vector<Graph> graphs_;

  std::vector<void*> owned_;
  uint64_t scratch_bytes_ = 0;
  uint64_t launches_ = 0;
  int sms_ = 148;
  uint32_t kpad_ = 0;
  const void* conv1_w_ = nullptr;
  void* conv_w_[2] = {nullptr, nullptr};  // convolutions 2 and 3, [channels][kpad] f16, K = (tap, input channel)
  alignas(64) uint8_t conv_map_[2][128];
  const float* conv_b_[3] = {nullptr, nullptr, nullptr};
  Mat conv_out_, proj_in_, proj_out_;
  const float *final_w_ = nullptr, *final_b_ = nullptr, *proj_in_b_ = nullptr, *proj_out_b_ = nullptr;
  std::vector<Layer> layers_;
  float* qkv_bias_ = nullptr;  // [layer][3 d_model]
  float* position_ = nullptr;  // [chunk_steps][d_model]
  void *mel_ = nullptr, *conv1_ = nullptr, *im2col_ = nullptr, *conv2_ = nullptr, *conv3_ = nullptr, *parts_ = nullptr,
       *xb_ = nullptr, *x_ = nullptr, *conv_stage_ = nullptr;
  int32_t* err_ = nullptr;
  size_t parts_floats_ = 0;
};

}  // namespace qwc

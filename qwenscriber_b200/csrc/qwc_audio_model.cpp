// qwc_audio_model.cpp -- host side of the audio tower (Model.projectAudio,
// src/core/qwen3_asr/model.zig:445-744): tensor resolution with the
// reference's shapes (layout.zig:150-262), weight repacking, TMA descriptors,
// scratch, and the launch sequence of one clip.
//
// Per clip (chunks of chunk_frames mel frames, `steps` packed encoder steps):
//   conv1 (direct, CUDA cores; one input channel)
//   conv2, conv3: im2col -> dense f16 tcgen05 GEMM -> bias + GELU
//   flatten (channel, frequency) per step -> conv_out GEMM -> + position row
//   per layer: LayerNorm -> Q|K|V GEMM (+ bias) -> windowed attention ->
//              O GEMM (+ bias, + residual) -> LayerNorm -> FFN-in GEMM
//              (+ bias, GELU) -> FFN-out GEMM (+ bias, + residual)
//   final LayerNorm -> projector-in GEMM (+ bias, GELU) -> projector-out GEMM (+ bias)

#include "qwc_audio_model.h"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "../../include/qwenscriber_cuda.h"
#include "qwc_internal.h"

namespace qwc {

namespace {

constexpr uint32_t kAudioLayerBase = 1024;  // container.zig:307
constexpr uint32_t kColsPerBlock = 64;      // GEMM columns per column block
constexpr uint32_t kKBlock = 64;

// container.zig:334-362
enum AudioKind : uint32_t {
  kConv1W = 1, kConv1B, kConv2W, kConv2B, kConv3W, kConv3B, kConvOutW, kFinalNormW, kFinalNormB,
  kQW, kQB, kKW, kKB, kVW, kVB, kOutW, kOutB, kAttnNormW, kAttnNormB, kFfnInW, kFfnInB, kFfnOutW, kFfnOutB,
  kLayerNormW, kLayerNormB, kProjInW, kProjInB, kProjOutW, kProjOutB,
};

int32_t cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return QWC_OK;
  cudaGetLastError();
  return e == cudaErrorMemoryAllocation ? QWC_OUT_OF_MEMORY : QWC_INVALID_STATE;
}

#define AUDIO_TRY(expr)              \
  do {                               \
    const int32_t _st = (expr);      \
    if (_st != QWC_OK) return _st;   \
  } while (0)
#define AUDIO_CUDA(expr) AUDIO_TRY(cuda_status(expr))
#define AUDIO_LAUNCH(expr)                                              \
  do {                                                                  \
    AUDIO_TRY(cuda_status(static_cast<cudaError_t>(expr)));             \
    ++launches_;                                                        \
  } while (0)

uint32_t ceil_div(uint32_t a, uint32_t b) { return (a + b - 1) / b; }

}  // namespace

uint32_t audio_post_conv_steps(uint32_t frames) {
  if (frames == 0) return 0;
  uint32_t s = frames;
  for (int i = 0; i < 3; ++i) s = (s - 1) / 2 + 1;
  return s;
}

uint32_t audio_packed_steps(const AudioGeometry& g, uint32_t frames) {
  return (frames / g.chunk_frames) * audio_post_conv_steps(g.chunk_frames) +
         audio_post_conv_steps(frames % g.chunk_frames);
}

AudioModel::~AudioModel() {
  for (Graph& gr : graphs_) cudaGraphExecDestroy(gr.exec);
  for (void* p : owned_) cudaFree(p);
}

void* AudioModel::alloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  owned_.push_back(p);
  scratch_bytes_ += bytes;
  return p;
}

int32_t AudioModel::build(const AudioGeometry& geometry, const Find& find, int sms) {
  g = geometry;
  sms_ = sms;
  const uint32_t d = g.d_model, C = g.channels;
  // What these kernels take: 8-channel taps for the im2col loads, 8-value
  // chunks of every row, LayerNorm rows of at most 4096, head_dim <= 128, and
  // an attention window whose keys and values fit in shared memory.
  if (C % 8 != 0 || C > 1024 || d % 8 != 0 || g.ffn % 8 != 0 || g.output_dim % 8 != 0 || d > 4096 || g.head_dim > 128 ||
      g.window == 0 || audio_attention_smem(g.window, g.head_dim) > 200 * 1024) {
    return QWC_UNSUPPORTED_MODEL;
  }
  int32_t st = QWC_OK;
  auto fail = [&](int32_t s) {
    if (st == QWC_OK) st = s;
  };
  auto get = [&](uint32_t kind, uint32_t layer, AudioTensorView* v) {
    if (!find(kind, layer, v)) {
      fail(QWC_NOT_FOUND);  // MissingTensor (abi.zig:130-132)
      return false;
    }
    return true;
  };
  auto vec = [&](uint32_t kind, uint32_t layer, uint32_t width) -> const float* {
    AudioTensorView v;
    if (!get(kind, layer, &v)) return nullptr;
    if (v.format != QWC_FORMAT_F32 || uint64_t(v.rows) * v.cols != width) {
      fail(QWC_SHAPE_MISMATCH);
      return nullptr;
    }
    return reinterpret_cast<const float*>(v.dev);
  };
  auto mat = [&](uint32_t kind, uint32_t layer, uint32_t rows, uint32_t cols, Mat* m) {
    AudioTensorView v;
    if (!get(kind, layer, &v)) return;
    if (v.rows != rows || v.cols != cols) return fail(QWC_SHAPE_MISMATCH);
    if (v.format != QWC_FORMAT_Q4 && v.format != QWC_FORMAT_Q5 && v.format != QWC_FORMAT_Q8) {
      return fail(QWC_UNSUPPORTED_MODEL);
    }
    m->rows = rows;
    m->cols = cols;
    m->format = v.format;
    // TMA strides are multiples of 16 bytes: a scale plane whose rows are not
    // (widths that are not a multiple of 512, e.g. the 0.6B tower's 896) is
    // copied into rows padded to the next multiple of 16 bytes.
    const uint32_t scale_row = cols / 64 * 2;
    const uint8_t* scales = v.dev + v.scales_offset;
    uint32_t stride = 0;
    if (scale_row % 16 != 0) {
      stride = (scale_row + 15) / 16 * 16;
      void* padded = alloc(size_t(rows) * stride);
      if (!padded) return fail(QWC_OUT_OF_MEMORY);
      if (cudaMemset(padded, 0, size_t(rows) * stride) != cudaSuccess ||
          cudaMemcpy2D(padded, stride, scales, scale_row, scale_row, rows, cudaMemcpyDeviceToDevice) != cudaSuccess) {
        cudaGetLastError();
        return fail(QWC_INVALID_STATE);
      }
      scales = static_cast<const uint8_t*>(padded);
    }
    fail(gemm_weight_maps(v.format, v.dev + v.codes_offset, scales, rows, cols, m->codes, m->scales, stride));
  };
  auto conv = [&](uint32_t kind, uint32_t in_channels) -> const uint8_t* {
    AudioTensorView v;
    if (!get(kind, 0, &v)) return nullptr;
    if (v.format != QWC_FORMAT_F16 || v.rows != C || v.cols != in_channels * 9) {
      fail(QWC_SHAPE_MISMATCH);
      return nullptr;
    }
    return v.dev;
  };

  conv1_w_ = conv(kConv1W, 1);
  const uint8_t* w2 = conv(kConv2W, C);
  const uint8_t* w3 = conv(kConv3W, C);
  conv_b_[0] = vec(kConv1B, 0, C);
  conv_b_[1] = vec(kConv2B, 0, C);
  conv_b_[2] = vec(kConv3B, 0, C);
  mat(kConvOutW, 0, d, g.conv_features, &conv_out_);
  final_w_ = vec(kFinalNormW, 0, d);
  final_b_ = vec(kFinalNormB, 0, d);
  mat(kProjInW, 0, d, d, &proj_in_);
  proj_in_b_ = vec(kProjInB, 0, d);
  mat(kProjOutW, 0, g.output_dim, d, &proj_out_);
  proj_out_b_ = vec(kProjOutB, 0, g.output_dim);
  layers_.assign(g.layers, Layer{});
  std::vector<const float*> qkv_b(3 * size_t(g.layers), nullptr);
  for (uint32_t i = 0; i < g.layers; ++i) {
    const uint32_t L = kAudioLayerBase + i;
    Layer& l = layers_[i];
    mat(kQW, L, d, d, &l.q);
    mat(kKW, L, d, d, &l.k);
    mat(kVW, L, d, d, &l.v);
    mat(kOutW, L, d, d, &l.o);
    mat(kFfnInW, L, g.ffn, d, &l.ffn_in);
    mat(kFfnOutW, L, d, g.ffn, &l.ffn_out);
    qkv_b[3 * i] = vec(kQB, L, d);
    qkv_b[3 * i + 1] = vec(kKB, L, d);
    qkv_b[3 * i + 2] = vec(kVB, L, d);
    l.o_b = vec(kOutB, L, d);
    l.attn_norm_w = vec(kAttnNormW, L, d);
    l.attn_norm_b = vec(kAttnNormB, L, d);
    l.ffn_in_b = vec(kFfnInB, L, g.ffn);
    l.ffn_out_b = vec(kFfnOutB, L, d);
    l.norm_w = vec(kLayerNormW, L, d);
    l.norm_b = vec(kLayerNormB, L, d);
  }
  if (st != QWC_OK) return st;

  // Convolutions 2 and 3 as [channels][kpad] f16, K = (ky * 3 + kx) * C + ic:
  // the 8 consecutive K of one GEMM chunk are 8 input channels of one tap,
  // contiguous in the channel-last planes.
  kpad_ = ceil_div(9 * C, kKBlock) * kKBlock;
  std::vector<uint16_t> src(size_t(C) * C * 9), dst(size_t(C) * kpad_, 0);
  const uint8_t* conv_src[2] = {w2, w3};
  for (int j = 0; j < 2; ++j) {
    AUDIO_CUDA(cudaMemcpy(src.data(), conv_src[j], src.size() * 2, cudaMemcpyDeviceToHost));
    for (uint32_t oc = 0; oc < C; ++oc) {
      for (uint32_t ic = 0; ic < C; ++ic) {
        for (uint32_t tap = 0; tap < 9; ++tap) {
          dst[size_t(oc) * kpad_ + tap * C + ic] = src[(size_t(oc) * C + ic) * 9 + tap];
        }
      }
    }
    conv_w_[j] = alloc(dst.size() * 2);
    if (!conv_w_[j]) return QWC_OUT_OF_MEMORY;
    AUDIO_CUDA(cudaMemcpy(conv_w_[j], dst.data(), dst.size() * 2, cudaMemcpyHostToDevice));
    AUDIO_TRY(gemm_dense_weight_map(conv_w_[j], C, kpad_, conv_map_[j]));
  }

  // The q|k|v biases of each layer side by side, for one epilogue.
  qkv_bias_ = static_cast<float*>(alloc(size_t(g.layers) * 3 * d * 4));
  if (!qkv_bias_) return QWC_OUT_OF_MEMORY;
  for (size_t i = 0; i < qkv_b.size(); ++i) {
    AUDIO_CUDA(cudaMemcpy(qkv_bias_ + i * d, qkv_b[i], size_t(d) * 4, cudaMemcpyDeviceToDevice));
  }

  // model.zig:750-762: the sinusoidal rows of the chunk's time steps,
  // computed in double and rounded to f32 once, as the reference adds them.
  std::vector<float> pos(size_t(g.chunk_steps) * d);
  const uint32_t half = d / 2;
  const double increment = std::log(10000.0) / (static_cast<double>(half) - 1.0);
  for (uint32_t s = 0; s < g.chunk_steps; ++s) {
    for (uint32_t i = 0; i < half; ++i) {
      const double angle = static_cast<double>(s) * std::exp(-increment * static_cast<double>(i));
      pos[size_t(s) * d + i] = static_cast<float>(std::sin(angle));
      pos[size_t(s) * d + half + i] = static_cast<float>(std::cos(angle));
    }
  }
  position_ = static_cast<float*>(alloc(pos.size() * 4));
  if (!position_) return QWC_OUT_OF_MEMORY;
  AUDIO_CUDA(cudaMemcpy(position_, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice));

  // Scratch for the longest clip.
  const uint32_t h1 = (g.mel_bins - 1) / 2 + 1, w1 = (g.chunk_frames - 1) / 2 + 1;
  const uint32_t h2 = (h1 - 1) / 2 + 1, w2n = (w1 - 1) / 2 + 1;
  const uint32_t cols2 = g.max_chunks * h2 * w2n, cols3 = g.max_chunks * g.bins * g.chunk_steps;
  const uint32_t maxk = std::max({g.conv_features, d, g.ffn});
  const size_t steps_blocks = ceil_div(g.max_steps, kColsPerBlock);
  // Split partials: the largest GEMM output (columns x rows) times the
  // largest split count a launch is allowed (run() clamps to this).
  const size_t out_max = std::max({size_t(cols2) * C, size_t(g.max_steps) * 3 * d, size_t(g.max_steps) * g.ffn,
                                   size_t(g.max_steps) * g.output_dim});
  parts_floats_ = out_max * 4;
  mel_ = alloc(size_t(g.mel_bins) * g.max_frames * 4);
  conv1_ = alloc(size_t(g.max_chunks) * h1 * w1 * C * 4);
  im2col_ = alloc(size_t(ceil_div(cols2, kColsPerBlock)) * 2 * kColsPerBlock * kpad_ * 2);
  conv2_ = alloc(size_t(cols2) * C * 4);
  conv3_ = alloc(size_t(cols3) * C * 4);
  parts_ = alloc(parts_floats_ * 4);
  xb_ = alloc(steps_blocks * 2 * kColsPerBlock * maxk * 2);
  x_ = alloc(size_t(g.max_steps) * d * 4);
  conv_stage_ = alloc(size_t(g.max_steps) * d * 4);
  err_ = static_cast<int32_t*>(alloc(256));
  for (void* p : {mel_, conv1_, im2col_, conv2_, conv3_, parts_, xb_, x_, conv_stage_, static_cast<void*>(err_)}) {
    if (!p) return QWC_OUT_OF_MEMORY;
  }
  AUDIO_CUDA(cudaMemset(im2col_, 0, size_t(ceil_div(cols2, kColsPerBlock)) * 2 * kColsPerBlock * kpad_ * 2));
  AUDIO_CUDA(cudaMemset(xb_, 0, steps_blocks * 2 * kColsPerBlock * maxk * 2));
  AUDIO_CUDA(cudaMemset(err_, 0, 256));
  AUDIO_CUDA(static_cast<cudaError_t>(prepare_gemm_kernel()));
  AUDIO_CUDA(static_cast<cudaError_t>(prepare_gemm_dense_kernel()));
  AUDIO_CUDA(static_cast<cudaError_t>(prepare_audio_kernels(g.window, g.head_dim)));
  return QWC_OK;
}

int32_t AudioModel::check_error(cudaStream_t stream) {
  int32_t herr = 0;
  AUDIO_CUDA(cudaMemcpyAsync(&herr, err_, 4, cudaMemcpyDeviceToHost, stream));
  AUDIO_CUDA(cudaStreamSynchronize(stream));
  if (herr != 0) {
    cudaMemsetAsync(err_, 0, 256, stream);
    cudaStreamSynchronize(stream);
    return QWC_INVALID_STATE;
  }
  return QWC_OK;
}

int32_t AudioModel::run(const float* mel_dev, uint32_t frames, float* out_dev, cudaStream_t stream,
                        uint64_t timeout_ns, uint32_t* steps_out, bool sync) {
  if (frames == 0) return QWC_SHAPE_MISMATCH;         // UnexpectedShape (model.zig:383)
  if (frames > g.max_frames) return QWC_AUDIO_TOO_LONG;  // model.zig:386
  // One CUDA graph per clip length (and buffers and wait bound): about 300
  // launches replayed with one call. Kept for the last kMaxGraphs lengths.
  Graph* hit = nullptr;
  for (Graph& gr : graphs_) {
    if (gr.frames == frames && gr.mel == mel_dev && gr.out == out_dev && gr.timeout_ns == timeout_ns) hit = &gr;
  }
  if (!hit) {
    if (graphs_.size() >= kMaxGraphs) {
      cudaGraphExecDestroy(graphs_.front().exec);
      graphs_.erase(graphs_.begin());
    }
    cudaGraph_t graph = nullptr;
    AUDIO_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    const int32_t st = enqueue(mel_dev, frames, out_dev, stream, timeout_ns);
    const cudaError_t end = cudaStreamEndCapture(stream, &graph);
    if (st != QWC_OK || end != cudaSuccess) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();
      return st != QWC_OK ? st : cuda_status(end);
    }
    Graph gr{frames, mel_dev, out_dev, timeout_ns, nullptr, launches_};
    const cudaError_t inst = cudaGraphInstantiate(&gr.exec, graph, 0);
    cudaGraphDestroy(graph);
    AUDIO_CUDA(inst);
    graphs_.push_back(gr);
    hit = &graphs_.back();
  }
  AUDIO_CUDA(cudaGraphLaunch(hit->exec, stream));
  launches_ = hit->launches;
  if (steps_out) *steps_out = audio_packed_steps(g, frames);
  if (!sync) return QWC_OK;
  return check_error(stream);
}

int32_t AudioModel::enqueue(const float* mel_dev, uint32_t frames, float* out_dev, cudaStream_t stream,
                            uint64_t timeout_ns) {
  launches_ = 0;
  const uint32_t d = g.d_model, C = g.channels, cf = g.chunk_frames;
  const uint32_t chunks = ceil_div(frames, cf), steps = audio_packed_steps(g, frames);
  const uint32_t h1 = (g.mel_bins - 1) / 2 + 1, w1 = (cf - 1) / 2 + 1;
  const uint32_t h2 = (h1 - 1) / 2 + 1, w2 = (w1 - 1) / 2 + 1;
  const uint32_t blocks = ceil_div(steps, kColsPerBlock);
  float* parts = static_cast<float*>(parts_);
  float* x = static_cast<float*>(x_);
  void* st = stream;

  // Split count for a GEMM of `rows` x `k` over `columns`, within the
  // partials buffer.
  auto splits_for = [&](uint32_t rows, uint32_t k, uint32_t columns) {
    uint32_t s = gemm_splits(rows, k, sms_, ceil_div(columns, kColsPerBlock));
    while (s > 1 && size_t(s) * columns * rows > parts_floats_) --s;
    const uint32_t kb = k / kKBlock, kps = ceil_div(kb, s);
    return ceil_div(kb, kps);  // the launch's real split count
  };
  // A quantized GEMM of up to three matrices over the packed activations xb
  // (K = k), `columns` columns, into parts[split][columns][ld].
  auto gemm = [&](const Mat* const* mats, uint32_t n, uint32_t k, uint32_t columns, uint32_t ld) -> int32_t {
    alignas(64) uint8_t cm[3][128], sm[3][128], bm[128];
    uint32_t rows[3], fmts[3], offs[3], total = 0;
    for (uint32_t j = 0; j < n; ++j) {
      std::memcpy(cm[j], mats[j]->codes, 128);
      std::memcpy(sm[j], mats[j]->scales, 128);
      rows[j] = mats[j]->rows;
      fmts[j] = mats[j]->format;
      offs[j] = total;
      total += rows[j];
    }
    const uint32_t cb = ceil_div(columns, kColsPerBlock);
    AUDIO_TRY(gemm_act_map(xb_, k, bm, cb));
    const uint32_t s = splits_for(total, k, columns);
    AUDIO_LAUNCH(launch_gemm_jobs(cm, sm, rows, fmts, offs, n, bm, k, columns, s, parts, ld, err_, st, cb, timeout_ns));
    return static_cast<int32_t>(s);
  };
  auto conv_gemm = [&](int j, const float* in, uint32_t ih, uint32_t iw, float* out) -> int32_t {
    const uint32_t oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1, columns = chunks * oh * ow;
    AUDIO_LAUNCH(launch_audio_im2col(in, chunks, ih, iw, C, kpad_, im2col_, st));
    alignas(64) uint8_t bm[128];
    AUDIO_TRY(gemm_act_map(im2col_, kpad_, bm, ceil_div(columns, kColsPerBlock)));
    const uint32_t s = splits_for(C, kpad_, columns);
    AUDIO_LAUNCH(launch_gemm_dense(conv_map_[j], bm, C, kpad_, columns, s, parts, err_, timeout_ns, st));
    AUDIO_LAUNCH(launch_audio_conv_epilogue(parts, s, columns, C, conv_b_[j + 1], out, st));
    return QWC_OK;
  };

  // Convolution stack (model.zig:506-577).
  AUDIO_LAUNCH(launch_audio_conv1(mel_dev, frames, g.mel_bins, cf, chunks, conv1_w_, conv_b_[0], C,
                                  static_cast<float*>(conv1_), st));
  AUDIO_TRY(conv_gemm(0, static_cast<float*>(conv1_), h1, w1, static_cast<float*>(conv2_)));
  AUDIO_TRY(conv_gemm(1, static_cast<float*>(conv2_), h2, w2, static_cast<float*>(conv3_)));
  // conv_out and the position rows (model.zig:580-601).
  AUDIO_LAUNCH(launch_audio_flatten(static_cast<float*>(conv3_), steps, g.chunk_steps, g.bins, C, xb_, st));
  {
    const Mat* m[1] = {&conv_out_};
    const int32_t s = gemm(m, 1, g.conv_features, steps, d);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_epilogue(0, parts, s, steps, d, d, position_, g.chunk_steps, x, d, nullptr, st));
  }
  AUDIO_CUDA(cudaMemcpyAsync(conv_stage_, x, size_t(steps) * d * 4, cudaMemcpyDeviceToDevice, stream));

  // The tower's blocks (model.zig:622-704). Each block's residual add of
  // O (and of the feed-forward) runs in the LayerNorm kernel that follows it:
  // the block's ffn norm, the next block's attention norm, or the final norm
  // (in place, as the reference's last layerNorm).
  if (!layers_.empty()) {
    AUDIO_LAUNCH(launch_audio_layernorm(x, nullptr, 0, nullptr, layers_[0].attn_norm_w, layers_[0].attn_norm_b, d,
                                        g.eps, steps, nullptr, xb_, st));
  } else {
    AUDIO_LAUNCH(launch_audio_layernorm(x, nullptr, 0, nullptr, final_w_, final_b_, d, g.eps, steps, x, xb_, st));
  }
  for (uint32_t li = 0; li < g.layers; ++li) {
    const Layer& l = layers_[li];
    const Mat* m3[3] = {&l.q, &l.k, &l.v};
    int32_t s = gemm(m3, 3, d, steps, 3 * d);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_attention(parts, s, qkv_bias_ + size_t(li) * 3 * d, steps, d, g.heads, g.head_dim,
                                        g.window, xb_, st));
    const Mat* mo[1] = {&l.o};
    s = gemm(mo, 1, d, steps, d);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_layernorm(x, parts, s, l.o_b, l.norm_w, l.norm_b, d, g.eps, steps, nullptr, xb_, st));
    const Mat* mi[1] = {&l.ffn_in};
    s = gemm(mi, 1, d, steps, g.ffn);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_epilogue(3, parts, s, steps, g.ffn, g.ffn, l.ffn_in_b, 0, nullptr, 0, xb_, st));
    const Mat* mf[1] = {&l.ffn_out};
    s = gemm(mf, 1, g.ffn, steps, d);
    if (s < 0) return s;
    if (li + 1 < g.layers) {
      const Layer& next = layers_[li + 1];
      AUDIO_LAUNCH(launch_audio_layernorm(x, parts, s, l.ffn_out_b, next.attn_norm_w, next.attn_norm_b, d, g.eps,
                                          steps, nullptr, xb_, st));
    } else {
      AUDIO_LAUNCH(launch_audio_layernorm(x, parts, s, l.ffn_out_b, final_w_, final_b_, d, g.eps, steps, x, xb_,
                                          st));
    }
  }

  // Projector (model.zig:707-733).
  {
    const Mat* mi[1] = {&proj_in_};
    int32_t s = gemm(mi, 1, d, steps, d);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_epilogue(3, parts, s, steps, d, d, proj_in_b_, 0, nullptr, 0, xb_, st));
    const Mat* mo[1] = {&proj_out_};
    s = gemm(mo, 1, d, steps, g.output_dim);
    if (s < 0) return s;
    AUDIO_LAUNCH(launch_audio_epilogue(1, parts, s, steps, g.output_dim, g.output_dim, proj_out_b_, 0, out_dev,
                                       g.output_dim, nullptr, st));
  }
  (void)blocks;
  return QWC_OK;
}

}  // namespace qwc

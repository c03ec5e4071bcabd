// qwc_api.cpp -- host runtime of libqwenscriber_cuda: the C ABI declared in
// include/qwenscriber_cuda.h.
//
// Mirrors the reference's model/decode state machine (src/wasm/model.zig),
// argument validation and status mapping (src/wasm/exports.zig,
// src/wasm/abi.zig), Config validation (src/core/model_config.zig:260-328) and
// the decoder's capacity rules (src/core/qwen3_asr/model.zig:62, decoder.zig:142).
// Device work is launched on one CUDA stream per handle.

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/qwenscriber_cuda.h"
#include "qwc_audio_model.h"
#include "qwc_internal.h"
#include "qwc_shard.h"

namespace qwc {
namespace {

// ---- Config (src/core/model_config.zig:110-177), byte for byte ----
struct Config {
  uint8_t magic[8];
  uint32_t format_version, architecture;
  uint32_t audio_d_model, audio_layers, audio_attention_heads, audio_ffn_dim, audio_downsample_hidden_size,
      audio_n_window, audio_n_window_infer, audio_max_position_steps, audio_output_dim, mel_bins;
  float audio_layer_norm_eps;
  uint32_t text_hidden_size, text_layers, text_attention_heads, text_key_value_heads, text_head_dim, text_ffn_dim,
      vocab_size;
  float text_rms_norm_eps, rope_theta;
  uint32_t max_positions, max_decode_tokens;
  uint32_t token_audio_start, token_audio_end, token_audio_pad, token_im_start, token_im_end, token_endoftext,
      token_asr_text, token_eos_primary, token_eos_secondary, token_pad;
  uint32_t flags, reserved1, reserved2, reserved3;
};
static_assert(sizeof(Config) == 160, "model_config.zig:364");
static_assert(offsetof(Config, audio_d_model) == 16, "model_config.zig:371");
static_assert(offsetof(Config, text_hidden_size) == 60, "model_config.zig:372");
static_assert(offsetof(Config, token_audio_start) == 104, "model_config.zig:373");
static_assert(offsetof(Config, flags) == 144, "model_config.zig:374");
static_assert(sizeof(qwc_requirements) == 48, "abi.zig:389");

constexpr uint32_t kMelBins = 128;          // src/core/mel.zig:50
constexpr uint32_t kCapacityFrames = 3000;  // src/core/mel.zig:55-58
constexpr uint32_t kFieldMax = 1u << 24;    // model_config.zig:26
constexpr uint32_t kLayerMax = 512;
constexpr uint32_t kVocabMax = 1u << 21;
constexpr uint32_t kDecodeTokensMax = 8192;

uint32_t conv_steps(uint32_t n) {
  for (int i = 0; i < 3; ++i) n = (n - 1) / 2 + 1;
  return n;
}

// model_config.zig:260-328. Every failure other than magic, version and
// capacity maps to invalid_argument, as abi.zig:91-147 reports them.
int32_t validate_config(const Config& c) {
  if (std::memcmp(c.magic, "QWCFG001", 8) != 0) return QWC_BAD_MAGIC;
  if (c.format_version != 1) return QWC_BAD_VERSION;
  if ((c.flags & ~1u) != 0 || c.reserved1 || c.reserved2 || c.reserved3) return QWC_INVALID_ARGUMENT;
  if (c.architecture != 1) return QWC_INVALID_ARGUMENT;
  auto range = [](uint32_t v) { return v != 0 && v <= kFieldMax; };
  auto layers = [](uint32_t v) { return v != 0 && v <= kLayerMax; };
  if (!range(c.audio_d_model) || !range(c.audio_ffn_dim) || !range(c.audio_downsample_hidden_size) ||
      !range(c.audio_output_dim) || !range(c.text_hidden_size) || !range(c.text_ffn_dim) || !range(c.text_head_dim) ||
      !layers(c.audio_layers) || !layers(c.text_layers)) {
    return QWC_INVALID_ARGUMENT;
  }
  if (c.mel_bins != kMelBins) return QWC_INVALID_ARGUMENT;
  if (c.audio_attention_heads == 0 || c.audio_d_model % c.audio_attention_heads != 0) return QWC_INVALID_ARGUMENT;
  const uint32_t audio_head = c.audio_d_model / c.audio_attention_heads;
  if (audio_head < 2 || audio_head % 2 != 0) return QWC_INVALID_ARGUMENT;
  if (c.text_attention_heads == 0 || c.text_key_value_heads == 0) return QWC_INVALID_ARGUMENT;
  if (c.text_attention_heads % c.text_key_value_heads != 0) return QWC_INVALID_ARGUMENT;
  if (c.text_head_dim < 2 || c.text_head_dim % 2 != 0) return QWC_INVALID_ARGUMENT;
  if (c.text_hidden_size != c.audio_output_dim) return QWC_INVALID_ARGUMENT;
  if (c.audio_n_window == 0) return QWC_INVALID_ARGUMENT;
  const uint32_t chunk = c.audio_n_window * 2;
  if (chunk > kCapacityFrames || c.audio_n_window_infer % chunk != 0) return QWC_INVALID_ARGUMENT;
  if (c.audio_max_position_steps < conv_steps(chunk)) return QWC_INVALID_ARGUMENT;
  if (c.vocab_size == 0 || c.vocab_size > kVocabMax) return QWC_INVALID_ARGUMENT;
  if (!range(c.max_positions)) return QWC_INVALID_ARGUMENT;
  if (c.max_decode_tokens == 0 || c.max_decode_tokens > kDecodeTokensMax) return QWC_INVALID_ARGUMENT;
  if (!std::isfinite(c.audio_layer_norm_eps) || !(c.audio_layer_norm_eps > 0.0f)) return QWC_INVALID_ARGUMENT;
  if (!std::isfinite(c.text_rms_norm_eps) || !(c.text_rms_norm_eps > 0.0f)) return QWC_INVALID_ARGUMENT;
  if (!std::isfinite(c.rope_theta) || !(c.rope_theta > 1.0f)) return QWC_INVALID_ARGUMENT;
  const uint32_t tokens[] = {c.token_audio_start, c.token_audio_end, c.token_audio_pad, c.token_im_start,
                             c.token_im_end, c.token_endoftext, c.token_asr_text, c.token_eos_primary,
                             c.token_eos_secondary, c.token_pad};
  for (uint32_t t : tokens) {
    if (t >= c.vocab_size) return QWC_INVALID_ARGUMENT;
  }
  // model.zig:1006-1009 (validateCapacity): CapacityExceeded -> limit_exceeded.
  if (c.max_positions == 0 || c.max_positions > kPositionLimit) return QWC_LIMIT_EXCEEDED;
  return QWC_OK;
}

// ---- rotary tables: kernels.zig:534-564 with Zig's std.math.pow(f32) ----
// (the published Go math.Pow algorithm: exp(yf * log x) times x^yi by
// repeated squaring, in f32), restricted to x > 0 finite.
float pow_f32(float x, float y) {
  if (y == 0.0f || x == 1.0f) return 1.0f;
  if (std::isnan(x) || std::isnan(y)) return std::nanf("");
  if (y == 1.0f) return x;
  if (y == 0.5f) return std::sqrt(x);
  if (y == -0.5f) return 1.0f / std::sqrt(x);
  float yi;
  float yf = std::modf(std::fabs(y), &yi);
  float a1 = 1.0f;
  int32_t ae = 0;
  if (yf != 0.0f) {
    if (yf > 0.5f) {
      yf -= 1.0f;
      yi += 1.0f;
    }
    a1 = std::exp(yf * std::log(x));
  }
  int xe = 0;
  float x1 = std::frexp(x, &xe);
  for (int32_t i = static_cast<int32_t>(yi); i != 0; i >>= 1) {
    if (xe < -(1 << 9) || (1 << 9) < xe) {
      ae += xe;
      break;
    }
    if (i & 1) {
      a1 *= x1;
      ae += xe;
    }
    x1 *= x1;
    xe <<= 1;
    if (x1 < 0.5f) {
      x1 += x1;
      xe -= 1;
    }
  }
  if (y < 0.0f) {
    a1 = 1.0f / a1;
    ae = -ae;
  }
  return std::ldexp(a1, ae);
}

void build_rope(float theta, uint32_t head_dim, uint32_t max_positions, float* cos_out, float* sin_out) {
  const uint32_t half = head_dim / 2;
  std::vector<float> inv(half);
  for (uint32_t i = 0; i < half; ++i) {
    const float exponent = -2.0f * static_cast<float>(i) / static_cast<float>(head_dim);
    inv[i] = pow_f32(theta, exponent);
  }
  for (uint32_t p = 0; p < max_positions; ++p) {
    for (uint32_t i = 0; i < half; ++i) {
      const float angle = static_cast<float>(p) * inv[i];
      cos_out[size_t(p) * half + i] = std::cos(angle);
      sin_out[size_t(p) * half + i] = std::sin(angle);
    }
  }
}

// ---- handles ----

enum class State { kIdle, kReady, kLoaded };

struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() {
    if (ptr) cudaFree(ptr);
  }
  int32_t alloc(size_t n) {
    if (ptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    if (n == 0) return QWC_OK;
    if (cudaMalloc(&ptr, n) != cudaSuccess) {
      cudaGetLastError();
      ptr = nullptr;
      return QWC_OUT_OF_MEMORY;
    }
    bytes = n;
    return QWC_OK;
  }
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

struct Tensor {
  uint32_t kind, layer, format, rows, cols;
  std::unique_ptr<DevBuf> buf;
  uint64_t scales_offset = 0, codes_offset = 0;
  // Its payload length and shape as the caller described them.
  uint64_t src_len = 0;
  uint32_t rank = 2, dims[4] = {1, 1, 1, 1};
};

struct StreamSlot {
  bool decoding = false;
  bool finished = false;
  uint32_t position = 0;         // positions the device has filled
  uint32_t next_token = 0;       // predicted, not yet produced
  uint32_t max_tokens = 0;
  std::vector<uint32_t> generated;
  std::deque<uint32_t> ahead;    // predictions computed beyond next_token
  std::unique_ptr<DevBuf> audio;  // the prompt's audio rows (device)
  bool logits_batched = false;     // the last logits of this slot come from the batched step
  uint32_t logits_col = 0;         // ... in this column of its logits buffer
};

// TMA descriptors of one weight matrix for the stream GEMM.
struct MatMaps {
  alignas(64) uint8_t codes[128];
  alignas(64) uint8_t scales[128];
};

// Device state of the batched multi-stream step (streams > 1).
struct Batched {
  DevBuf hidden, xb_h, xb_q, xb_f, part0, qrot, attn_part, attn_count, logits, tokens, desc, audio_ptrs, err;
  DevBuf qkv_rows;  // the last layer's pre-norm q/k/v rows of the last step (qwc_debug_scratch 4)
  DevBuf history, counter;
  std::vector<MatMaps> mq, mk, mv, mo, mg, mu, md;
  MatMaps mlm;
  alignas(64) uint8_t b_h[128];
  alignas(64) uint8_t b_q[128];
  alignas(64) uint8_t b_f[128];
  KvMaps4 kv;
  uint32_t splits_qkv = 1, splits_o = 1, splits_gu = 1, splits_down = 1;
  uint32_t kernels_per_step = 0, kernels_per_step_nologits = 0;
  uint32_t history_rows = 0;
  int attn_grid = 0;
  StreamsStep P{};
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  // The step without the final norm, lm_head and argmax: prompt-prefill
  // steps whose logits nothing reads (every one but a prompt's last).
  cudaGraph_t graph_nologits = nullptr;
  cudaGraphExec_t exec_nologits = nullptr;
  SlotStep* host_desc = nullptr;    // pinned
  uint32_t* host_tokens = nullptr;  // pinned
  int32_t* host_err = nullptr;      // pinned
  ~Batched() {
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (exec_nologits) cudaGraphExecDestroy(exec_nologits);
    if (graph_nologits) cudaGraphDestroy(graph_nologits);
    if (host_desc) cudaFreeHost(host_desc);
    if (host_tokens) cudaFreeHost(host_tokens);
    if (host_err) cudaFreeHost(host_err);
  }
};

struct Handle {
  int device = 0;
  cudaStream_t stream = nullptr;
  State state = State::kIdle;
  uint32_t cache_format = QWC_CACHE_F32;  // the reference's default (model.zig:119)
  uint32_t streams = 1;
  bool ignore_eos = false;
  bool keep_logits = false;
  bool trace = false;
  bool prefill_serial = false;  // QWC_OPTION_PREFILL_SERIAL
  bool exact = false;           // QWC_OPTION_EXACT
  uint64_t wait_limit_ns = 0;   // QWC_OPTION_WAIT_LIMIT_US (0: the defaults)
  bool test_stall = false;      // QWC_OPTION_TEST_STALL (applies to the next launch only)
  uint32_t step_chunk = 16;
  uint64_t launches = 0;
  std::map<std::pair<uint32_t, uint32_t>, Tensor> tensors;
  // qwc_model_tensor_descriptor's enumeration (src/wasm/model.zig:265-319):
  // every entry of every shard, shards in the order they were added and each
  // shard's entries in index order, audio-tower and projector tensors
  // included; a tensor added alone follows in call order.
  std::vector<qwc_tensor_descriptor> descriptors;
  Config config{};
  int grid = 0;
  DevModel host_model{};
  DevBuf model_buf, rope_cos, rope_sin, k_cache, v_cache;
  DevBuf qkv, attn_out, hidden_g, act, attn_part, attn_count, amax_val, amax_idx, barrier, error, tokens_out, logits;
  DevBuf prompt_ids, prompt_rows, audio_rows, trace_buf, exact_scratch;
  uint32_t max_chunks = 0;
  bool wide_slots = false;  // decode with the three-slot kernel (launch_decode_wide)
  uint64_t weight_bytes = 0;
  KvMaps kv_maps{};
  std::unique_ptr<Batched> batched;  // streams > 1
  std::unique_ptr<AudioModel> audio;  // the audio tower and projector, when the model carries them
  DevBuf audio_out;                   // projected rows of the last clip [steps][text_hidden_size]
  std::vector<StreamSlot> slots;
  // Payload checksums of the shards added since qwc_model_begin, for the
  // reference's duplicate-shard check (src/wasm/model.zig:162-175).
  std::vector<uint32_t> shards;

  ~Handle() {
    if (stream) cudaStreamDestroy(stream);
  }
};

constexpr size_t kShardCountMax = 64;  // src/wasm/model.zig:81
// Default bounds on the device-side waits (QWC_OPTION_WAIT_LIMIT_US overrides).
constexpr uint64_t kDecodeWaitNs = 4000000000ull;
constexpr uint64_t kBatchedWaitNs = 2000000000ull;

std::mutex g_mutex;
std::map<uint32_t, std::unique_ptr<Handle>> g_handles;
uint32_t g_next_handle = 1;

Handle* lookup(uint32_t h) {
  std::lock_guard<std::mutex> lock(g_mutex);
  auto it = g_handles.find(h);
  return it == g_handles.end() ? nullptr : it->second.get();
}

int32_t status_of(cudaError_t e) {
  if (e == cudaSuccess) return QWC_OK;
  if (std::getenv("QWC_VERBOSE")) std::fprintf(stderr, "qwc: CUDA error: %s\n", cudaGetErrorString(e));
  cudaGetLastError();
  if (e == cudaErrorMemoryAllocation) return QWC_OUT_OF_MEMORY;
  return QWC_INVALID_STATE;
}

#define QWC_TRY(expr)                        \
  do {                                       \
    const int32_t _st = (expr);              \
    if (_st != QWC_OK) return _st;           \
  } while (0)

#define QWC_CUDA(expr) QWC_TRY(status_of(expr))

void release_model(Handle* h) {
  h->tensors.clear();
  h->descriptors.clear();
  h->shards.clear();
  for (DevBuf* b : {&h->model_buf, &h->rope_cos, &h->rope_sin, &h->k_cache, &h->v_cache, &h->qkv, &h->attn_out,
                    &h->hidden_g, &h->act, &h->attn_part, &h->attn_count, &h->amax_val, &h->amax_idx, &h->barrier,
                    &h->error, &h->tokens_out, &h->logits, &h->prompt_ids, &h->prompt_rows, &h->audio_rows, &h->trace_buf,
                    &h->exact_scratch}) {
    b->alloc(0);
  }
  h->slots.clear();
  h->batched.reset();
  h->audio.reset();
  h->audio_out.alloc(0);
  h->weight_bytes = 0;
}

bool is_vector_kind(uint32_t kind) {
  return kind == QWC_KIND_DECODER_FINAL_NORM || kind == QWC_KIND_DECODER_Q_NORM || kind == QWC_KIND_DECODER_K_NORM ||
         kind == QWC_KIND_DECODER_ATTENTION_NORM || kind == QWC_KIND_DECODER_FFN_NORM;
}

// container.zig:334-362: the audio tower and projector kinds (1-29); their
// biases and norm vectors; the f16 convolution weights.
bool is_audio_kind(uint32_t kind) { return kind >= QWC_KIND_AUDIO_CONV1_WEIGHT && kind <= QWC_KIND_PROJECTOR_OUT_BIAS; }
bool is_audio_vector_kind(uint32_t kind) {
  switch (kind) {
    case QWC_KIND_AUDIO_CONV1_BIAS: case QWC_KIND_AUDIO_CONV2_BIAS: case QWC_KIND_AUDIO_CONV3_BIAS:
    case QWC_KIND_AUDIO_FINAL_NORM_WEIGHT: case QWC_KIND_AUDIO_FINAL_NORM_BIAS: case QWC_KIND_AUDIO_Q_BIAS:
    case QWC_KIND_AUDIO_K_BIAS: case QWC_KIND_AUDIO_V_BIAS: case QWC_KIND_AUDIO_OUT_BIAS:
    case QWC_KIND_AUDIO_ATTENTION_NORM_WEIGHT: case QWC_KIND_AUDIO_ATTENTION_NORM_BIAS:
    case QWC_KIND_AUDIO_FFN_IN_BIAS: case QWC_KIND_AUDIO_FFN_OUT_BIAS: case QWC_KIND_AUDIO_FINAL_LAYER_NORM_WEIGHT:
    case QWC_KIND_AUDIO_FINAL_LAYER_NORM_BIAS: case QWC_KIND_PROJECTOR_IN_BIAS: case QWC_KIND_PROJECTOR_OUT_BIAS:
      return true;
    default:
      return false;
  }
}
bool is_conv_kind(uint32_t kind) {
  return kind == QWC_KIND_AUDIO_CONV1_WEIGHT || kind == QWC_KIND_AUDIO_CONV2_WEIGHT ||
         kind == QWC_KIND_AUDIO_CONV3_WEIGHT;
}

// The tower's geometry from the configuration (model_config.zig:190-240).
AudioGeometry audio_geometry(const Config& c) {
  AudioGeometry g{};
  g.d_model = c.audio_d_model;
  g.layers = c.audio_layers;
  g.heads = c.audio_attention_heads;
  g.head_dim = c.audio_d_model / c.audio_attention_heads;
  g.ffn = c.audio_ffn_dim;
  g.channels = c.audio_downsample_hidden_size;
  g.n_window = c.audio_n_window;
  g.n_window_infer = c.audio_n_window_infer;
  g.chunk_frames = c.audio_n_window * 2;
  g.bins = conv_steps(c.mel_bins);
  g.conv_features = g.channels * g.bins;
  g.chunk_steps = conv_steps(g.chunk_frames);
  g.max_position_steps = c.audio_max_position_steps;
  g.output_dim = c.audio_output_dim;
  g.mel_bins = c.mel_bins;
  g.eps = c.audio_layer_norm_eps;
  g.window = (c.audio_n_window_infer / g.chunk_frames) * g.chunk_steps;  // model.zig:243-246
  g.max_frames = kCapacityFrames;
  g.max_chunks = (kCapacityFrames + g.chunk_frames - 1) / g.chunk_frames;
  g.max_steps = audio_packed_steps(g, kCapacityFrames);
  return g;
}

DevMat make_mat(const Tensor& t) {
  DevMat m{};
  m.scales = static_cast<const uint8_t*>(t.buf->ptr) + t.scales_offset;
  m.codes = static_cast<const uint8_t*>(t.buf->ptr) + t.codes_offset;
  m.rows = t.rows;
  m.cols = t.cols;
  m.format = t.format;
  m.groups = t.cols / kGroup;
  m.scale_row = m.groups * 2;
  m.code_row = m.groups * data_bytes_per_group(t.format);
  return m;
}

// The decode kernel's layout rules for one matrix: q4/q5/q8, whole code spans
// per row (a warp reads 32 x 16 bytes per step, or 16 q5 groups = 640 bytes),
// K within the activation buffer, and one row per ring slot at least.
int32_t kernel_fits(const DevMat& m) {
  if (m.format != kFormatQ4 && m.format != kFormatQ5 && m.format != kFormatQ8) return QWC_UNSUPPORTED_MODEL;
  if (m.code_row % (m.format == kFormatQ5 ? 640u : 512u) != 0 || m.scale_row % 16 != 0) return QWC_UNSUPPORTED_MODEL;
  if (m.cols > 8192) return QWC_UNSUPPORTED_MODEL;
  if (m.scale_row + m.code_row > 28 * 1024) return QWC_UNSUPPORTED_MODEL;
  return QWC_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against libcuda).
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = []() -> EncodeTiledFn {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

}  // namespace

int32_t encode_tensor_map(uint8_t* out128, int type, uint32_t rank, void* base, const uint64_t* dims,
                               const uint64_t* strides, const uint32_t* box, bool swizzle128) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn || rank < 1 || rank > 5) return QWC_INVALID_STATE;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], el[5];
  for (uint32_t i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    el[i] = 1;
    if (i + 1 < rank) st[i] = strides[i];
  }
  const CUresult r =
      fn(reinterpret_cast<CUtensorMap*>(out128), type == kMapF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
         rank, base, d, st, b, el, CU_TENSOR_MAP_INTERLEAVE_NONE,
         swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? QWC_OK : QWC_INVALID_STATE;
}

namespace {

// One q8 cache plane of stream 0 as a 3-D u8 tensor [layer][position][row
// bytes], boxes of `box_x` bytes x kAttnChunk positions x 1 layer.
int32_t encode_plane(uint8_t* out, uint8_t* base, uint64_t row_bytes, uint64_t positions, uint64_t layers,
                     uint64_t layer_stride, uint32_t box_x) {
  const uint64_t dims[3] = {row_bytes, positions, layers};
  const uint64_t strides[2] = {row_bytes, layer_stride};
  const uint32_t box[3] = {box_x, kAttnChunk, 1};
  return encode_tensor_map(out, kMapU8, 3, base, dims, strides, box, false);
}

int32_t build_batched(Handle* h);

int32_t finish_model(Handle* h, const Config& c) {
  QWC_TRY(validate_config(c));
  const uint32_t hidden = c.text_hidden_size, qw = c.text_attention_heads * c.text_head_dim,
                 kvw = c.text_key_value_heads * c.text_head_dim, ffn = c.text_ffn_dim, L = c.text_layers;
  if (h->cache_format != QWC_CACHE_Q8) return QWC_UNSUPPORTED;  // this backend keeps the q8 cache
  if (L > kMaxLayers || c.text_head_dim != kHeadDim || c.text_attention_heads != 2 * c.text_key_value_heads) {
    return QWC_UNSUPPORTED_MODEL;
  }
  // A norm weight vector travels as one ring slot; the cache's TMA boxes need
  // 16-byte rows of scales (four kv heads).
  if (hidden % 4 != 0 || hidden > kHiddenMax || qw > 8192 || ffn > 8192) return QWC_UNSUPPORTED_MODEL;
  if (c.text_key_value_heads % 4 != 0) return QWC_UNSUPPORTED_MODEL;
  const bool tied = (c.flags & 1u) != 0;

  auto find = [&](uint32_t kind, uint32_t layer) -> const Tensor* {
    auto it = h->tensors.find({kind, layer});
    return it == h->tensors.end() ? nullptr : &it->second;
  };
  // Shapes of src/core/qwen3_asr/layout.zig:264-320 (decoder layers) and the fixed tensors.
  auto need_mat = [&](uint32_t kind, uint32_t layer, uint32_t rows, uint32_t cols, DevMat* out) -> int32_t {
    const Tensor* t = find(kind, layer);
    if (!t) return QWC_NOT_FOUND;
    if (is_vector_kind(kind) || t->rows != rows || t->cols != cols) return QWC_SHAPE_MISMATCH;
    *out = make_mat(*t);
    return kernel_fits(*out);
  };
  auto need_vec = [&](uint32_t kind, uint32_t layer, uint32_t width, const float** out) -> int32_t {
    const Tensor* t = find(kind, layer);
    if (!t) return QWC_NOT_FOUND;
    if (t->format != QWC_FORMAT_F32 || uint64_t(t->rows) * t->cols != width) return QWC_SHAPE_MISMATCH;
    *out = static_cast<const float*>(t->buf->ptr);
    return QWC_OK;
  };

  DevModel& m = h->host_model;
  m = DevModel{};
  QWC_TRY(need_mat(QWC_KIND_DECODER_EMBED_TOKENS, 0, c.vocab_size, hidden, &m.embed));
  QWC_TRY(need_vec(QWC_KIND_DECODER_FINAL_NORM, 0, hidden, &m.final_norm));
  if (tied) {
    m.lm_head = m.embed;  // model.zig:391-394
  } else {
    QWC_TRY(need_mat(QWC_KIND_DECODER_OUTPUT, 0, c.vocab_size, hidden, &m.lm_head));
  }
  for (uint32_t l = 0; l < L; ++l) {
    DevLayer& D = m.layers[l];
    const uint32_t layer = l + 1;  // decoder_layer_base (layout.zig:26)
    QWC_TRY(need_mat(QWC_KIND_DECODER_Q, layer, qw, hidden, &D.q));
    QWC_TRY(need_mat(QWC_KIND_DECODER_K, layer, kvw, hidden, &D.k));
    QWC_TRY(need_mat(QWC_KIND_DECODER_V, layer, kvw, hidden, &D.v));
    QWC_TRY(need_mat(QWC_KIND_DECODER_O, layer, hidden, qw, &D.o));
    QWC_TRY(need_vec(QWC_KIND_DECODER_Q_NORM, layer, c.text_head_dim, &D.q_norm));
    QWC_TRY(need_vec(QWC_KIND_DECODER_K_NORM, layer, c.text_head_dim, &D.k_norm));
    QWC_TRY(need_vec(QWC_KIND_DECODER_ATTENTION_NORM, layer, hidden, &D.attn_norm));
    QWC_TRY(need_vec(QWC_KIND_DECODER_FFN_NORM, layer, hidden, &D.ffn_norm));
    QWC_TRY(need_mat(QWC_KIND_DECODER_GATE, layer, ffn, hidden, &D.gate));
    QWC_TRY(need_mat(QWC_KIND_DECODER_UP, layer, ffn, hidden, &D.up));
    QWC_TRY(need_mat(QWC_KIND_DECODER_DOWN, layer, hidden, ffn, &D.down));
    if (D.q.format != D.k.format || D.q.format != D.v.format || D.gate.format != D.up.format) {
      return QWC_UNSUPPORTED_MODEL;
    }
  }

  cudaSetDevice(h->device);
  h->grid = decode_grid_size(h->device);
  if (h->grid <= 0) return QWC_INVALID_STATE;
  // Rows of a non-LM stage held by one CTA must fit the kernel's row buffers
  // (the gate-and-up stage holds a CTA's gate rows and as many up rows).
  if ((qw + 2 * kvw + h->grid - 1) / h->grid > 256 || 2 * ((ffn + h->grid - 1) / h->grid) > 256 ||
      (hidden + h->grid - 1) / h->grid > 256) {
    return QWC_UNSUPPORTED_MODEL;
  }
  // Every CTA streams at least one tile of each stage, which keeps a layer's
  // attention tiles (TMA reads of cache rows earlier tokens wrote) more than
  // a ring's depth of tiles behind those writes.
  if (std::min(hidden, ffn) < static_cast<uint32_t>(h->grid)) return QWC_UNSUPPORTED_MODEL;
  // The decode kernel's wide-slot copy pays off when a CTA's down-projection
  // rows fit one wide slot but not one narrow one (two tiles become one);
  // otherwise the five narrow slots keep the deeper prefetch.
  {
    const uint64_t down_bytes = uint64_t((hidden + h->grid - 1) / h->grid) *
                                (m.layers[0].down.scale_row + m.layers[0].down.code_row);
    h->wide_slots = down_bytes > kDecodeSlotBytes && down_bytes <= kDecodeWideSlotBytes;
  }

  m.n_layers = L;
  m.hidden = hidden;
  m.q_heads = c.text_attention_heads;
  m.kv_heads = c.text_key_value_heads;
  m.head_dim = c.text_head_dim;
  m.ffn = ffn;
  m.vocab = c.vocab_size;
  m.max_positions = c.max_positions;
  m.eps = c.text_rms_norm_eps;
  m.attn_scaling = 1.0f / std::sqrt(static_cast<float>(c.text_head_dim));
  const uint64_t kv_groups = kvw / kGroup;
  m.cache_scales_bytes = uint64_t(c.max_positions) * kv_groups * 2;
  m.cache_layer_stride = m.cache_scales_bytes + uint64_t(c.max_positions) * kvw;
  m.cache_stream_stride = m.cache_layer_stride * L;

  // Rotary tables, built on the host (kernels.zig:534-558) and uploaded.
  const size_t half = c.text_head_dim / 2;
  std::vector<float> cos_t(size_t(c.max_positions) * half), sin_t(cos_t.size());
  build_rope(c.rope_theta, c.text_head_dim, c.max_positions, cos_t.data(), sin_t.data());
  QWC_TRY(h->rope_cos.alloc(cos_t.size() * 4));
  QWC_TRY(h->rope_sin.alloc(sin_t.size() * 4));
  QWC_CUDA(cudaMemcpy(h->rope_cos.ptr, cos_t.data(), cos_t.size() * 4, cudaMemcpyHostToDevice));
  QWC_CUDA(cudaMemcpy(h->rope_sin.ptr, sin_t.data(), sin_t.size() * 4, cudaMemcpyHostToDevice));
  m.rope_cos = h->rope_cos.as<float>();
  m.rope_sin = h->rope_sin.as<float>();

  // q8 key/value cache per stream (decoder.zig:58-65, model.zig:253-260).
  QWC_TRY(h->k_cache.alloc(m.cache_stream_stride * h->streams));
  QWC_TRY(h->v_cache.alloc(m.cache_stream_stride * h->streams));
  QWC_CUDA(cudaMemset(h->k_cache.ptr, 0, h->k_cache.bytes));
  QWC_CUDA(cudaMemset(h->v_cache.ptr, 0, h->v_cache.bytes));
  {
    static_assert(sizeof(CUtensorMap) == 128, "KvMaps holds 128-byte tensor maps");
    const uint64_t kv_row = kvw, scale_row = uint64_t(kvw / kGroup) * 2;
    uint8_t* kc = h->k_cache.as<uint8_t>();
    uint8_t* vc = h->v_cache.as<uint8_t>();
    KvMaps& km = h->kv_maps;
    QWC_TRY(encode_plane(km.k_codes, kc + m.cache_scales_bytes, kv_row, c.max_positions, L, m.cache_layer_stride,
                         kHeadDim));
    QWC_TRY(encode_plane(km.v_codes, vc + m.cache_scales_bytes, kv_row, c.max_positions, L, m.cache_layer_stride,
                         kHeadDim));
    QWC_TRY(encode_plane(km.k_scales, kc, scale_row, c.max_positions, L, m.cache_layer_stride, 16));
    QWC_TRY(encode_plane(km.v_scales, vc, scale_row, c.max_positions, L, m.cache_layer_stride, 16));
  }

  h->max_chunks = (c.max_positions + kAttnChunk - 1) / kAttnChunk;
  QWC_TRY(h->qkv.alloc(size_t(qw + 2 * kvw) * 4));
  QWC_TRY(h->attn_out.alloc(size_t(qw) * 4));
  QWC_TRY(h->hidden_g.alloc(size_t(hidden) * 4));
  QWC_TRY(h->act.alloc(size_t(ffn) * 4));
  // The decode kernel's attention partials: one per chunk of cached positions
  // and one for the new row (max_chunks + 1 per query head).
  QWC_TRY(h->attn_part.alloc(size_t(c.text_attention_heads) * (h->max_chunks + 1) * kAttnPartStride * 4));
  QWC_TRY(h->attn_count.alloc(size_t(c.text_key_value_heads) * 4));
  QWC_CUDA(cudaMemset(h->attn_count.ptr, 0, h->attn_count.bytes));
  QWC_TRY(h->amax_val.alloc(size_t(h->grid) * 4));
  QWC_TRY(h->amax_idx.alloc(size_t(h->grid) * 4));
  QWC_TRY(h->barrier.alloc(kBarrierBytes));
  QWC_TRY(h->error.alloc(256));
  QWC_CUDA(cudaMemset(h->error.ptr, 0, h->error.bytes));
  QWC_TRY(h->tokens_out.alloc(size_t(std::max<uint32_t>(c.max_positions, 256)) * 4));
  QWC_TRY(h->logits.alloc(size_t(c.vocab_size) * 4));
  QWC_TRY(h->prompt_ids.alloc(size_t(c.max_positions) * 4));
  QWC_TRY(h->prompt_rows.alloc(size_t(c.max_positions) * 4));
  QWC_TRY(h->audio_rows.alloc(size_t(c.max_positions) * hidden * 4));
  // Exact mode's attention scores and value weights: [q_heads][3][max_positions].
  QWC_TRY(h->exact_scratch.alloc(size_t(c.text_attention_heads) * 3 * c.max_positions * 4));

  QWC_TRY(h->model_buf.alloc(sizeof(DevModel)));
  QWC_CUDA(cudaMemcpy(h->model_buf.ptr, &m, sizeof(DevModel), cudaMemcpyHostToDevice));
  h->slots.clear();
  h->slots.resize(h->streams);
  h->config = c;
  // Every handle gets the batched engine: it runs the prompt prefills (64
  // positions per step) and, with streams > 1, the batched decode steps.
  QWC_TRY(build_batched(h));
  // The audio tower and projector, when the model carries any of their
  // tensors (then all of them, as model.zig:965-990 requires).
  bool any_audio = false;
  for (const auto& kv : h->tensors) any_audio = any_audio || is_audio_kind(kv.first.first);
  if (any_audio) {
    auto audio = std::make_unique<AudioModel>();
    auto find_audio = [h](uint32_t kind, uint32_t layer, AudioTensorView* out) {
      auto it = h->tensors.find({kind, layer});
      if (it == h->tensors.end()) return false;
      const Tensor& t = it->second;
      out->format = t.format;
      out->rows = t.rows;
      out->cols = t.cols;
      out->dev = static_cast<const uint8_t*>(t.buf->ptr);
      out->scales_offset = t.scales_offset;
      out->codes_offset = t.codes_offset;
      return true;
    };
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device);
    QWC_TRY(audio->build(audio_geometry(c), find_audio, sms));
    QWC_TRY(h->audio_out.alloc(size_t(audio->g.max_steps) * c.audio_output_dim * 4));
    h->audio = std::move(audio);
  }
  return QWC_OK;
}

// One launch of the persistent decode kernel for stream 0; waits for it and
// reads back the produced tokens.
int32_t run_decode(Handle* h, uint32_t n_tokens, uint32_t first_position, uint32_t n_forced, uint32_t first_input,
                   uint32_t logits_from, std::vector<uint32_t>* tokens) {
  const DevModel& m = h->host_model;
  DecodeLaunch L{};
  L.model = h->model_buf.as<DevModel>();
  L.k_cache = h->k_cache.as<uint8_t>();
  L.v_cache = h->v_cache.as<uint8_t>();
  L.n_tokens = n_tokens;
  L.first_position = first_position;
  L.n_forced = n_forced;
  L.forced_token = h->prompt_ids.as<uint32_t>();
  L.forced_row = h->prompt_rows.as<int32_t>();
  L.audio = h->audio_rows.as<float>();
  L.first_input = first_input;
  L.logits_from = logits_from;
  L.tokens_out = h->tokens_out.as<uint32_t>();
  L.logits_out = h->keep_logits ? h->logits.as<float>() : nullptr;
  L.qkv = h->qkv.as<float>();
  L.attn_out = h->attn_out.as<float>();
  L.hidden_g = h->hidden_g.as<float>();
  L.act = h->act.as<float>();
  L.attn_part = h->attn_part.as<float>();
  L.attn_count = h->attn_count.as<uint32_t>();
  L.amax_val = h->amax_val.as<float>();
  L.amax_idx = h->amax_idx.as<uint32_t>();
  L.barrier = h->barrier.as<uint32_t>();
  L.error = h->error.as<int32_t>();
  L.timeout_ns = h->wait_limit_ns ? h->wait_limit_ns : kDecodeWaitNs;
  L.exact = h->exact ? 1u : 0u;
  L.stall = h->test_stall ? 1u : 0u;
  h->test_stall = false;
  L.exact_scratch = h->exact_scratch.as<float>();
  if (h->trace) {
    if (h->trace_buf.bytes == 0) QWC_TRY(h->trace_buf.alloc(size_t(h->grid) * kTraceEvents * 8));
    QWC_CUDA(cudaMemsetAsync(h->trace_buf.ptr, 0, h->trace_buf.bytes, h->stream));
    L.trace = h->trace_buf.as<uint64_t>();
    L.trace_token = 0;
  }
  L.max_chunks = h->max_chunks + 1;  // partial slots per query head (attn_part)
  (void)m;
  QWC_CUDA(cudaMemsetAsync(h->barrier.ptr, 0, kBarrierBytes, h->stream));
  const int e = h->wide_slots ? launch_decode_wide(L, h->kv_maps, h->grid, h->stream)
                              : launch_decode(L, h->kv_maps, h->grid, h->stream);
  if (e != 0) {
    if (std::getenv("QWC_VERBOSE")) std::fprintf(stderr, "qwc: decode launch failed: %s\n", cudaGetErrorString(static_cast<cudaError_t>(e)));
    return status_of(static_cast<cudaError_t>(e));
  }
  h->launches += 1;
  int32_t device_error = 0;
  QWC_CUDA(cudaMemcpyAsync(&device_error, h->error.ptr, 4, cudaMemcpyDeviceToHost, h->stream));
  if (tokens && n_tokens > logits_from) {
    tokens->resize(n_tokens);
    QWC_CUDA(cudaMemcpyAsync(tokens->data(), h->tokens_out.ptr, size_t(n_tokens) * 4, cudaMemcpyDeviceToHost,
                             h->stream));
  }
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  if (device_error != 0) {
    if (std::getenv("QWC_VERBOSE")) std::fprintf(stderr, "qwc: decode kernel gave up waiting (code %d)\n", device_error);
    cudaMemsetAsync(h->error.ptr, 0, 4, h->stream);
    cudaStreamSynchronize(h->stream);
    return QWC_INVALID_STATE;
  }
  return QWC_OK;
}

// src/wasm/model.zig:495-499
bool ends_sequence(const Config& c, uint32_t token) {
  return token == c.token_eos_primary || token == c.token_eos_secondary || token == c.token_endoftext;
}

// ---- batched multi-stream step ----

int32_t mat_maps(const DevMat& m, MatMaps* out) {
  return gemm_weight_maps(m.format, m.codes, m.scales, m.rows, m.cols, out->codes, out->scales);
}

int32_t act_map(uint8_t* out, void* base, uint32_t cols) { return gemm_act_map(base, cols, out); }

// `swizzle`: 128-byte rows land with the 128-byte swizzle (16-byte chunk c of
// row r at chunk c ^ (r % 8)), so tensor-core fragment loads of a tile are
// free of bank conflicts.
int32_t kv_map4(uint8_t* out, uint8_t* base, uint64_t row, const DevModel& m, uint32_t streams, uint32_t box_x,
                bool swizzle) {
  const uint64_t dims[4] = {row, m.max_positions, m.n_layers, streams};
  const uint64_t str[3] = {row, m.cache_layer_stride, m.cache_stream_stride};
  const uint32_t box[4] = {box_x, kAttnChunk, 1, 1};
  return encode_tensor_map(out, kMapU8, 4, base, dims, str, box, swizzle);
}

// Enqueues one whole step on the handle's stream (recorded into the graph);
// without `logits` it ends after the last layer's down projection.
int32_t record_step(Handle* h, bool logits) {
  Batched& b = *h->batched;
  const DevModel& m = h->host_model;
  const StreamsStep& P = b.P;
  void* st = h->stream;
  const uint32_t qw = m.q_heads * kHeadDim, kvw = m.kv_heads * kHeadDim;
  uint32_t kernels = 0;
  auto ok = [&](int e) -> int32_t {
    ++kernels;
    return e == 0 ? QWC_OK : status_of(static_cast<cudaError_t>(e));
  };
  auto gemm = [&](std::initializer_list<const MatMaps*> mats, std::initializer_list<const DevMat*> dms,
                  const uint8_t* bmap, uint32_t cols, uint32_t splits, float* out, uint32_t ld) -> int32_t {
    alignas(64) uint8_t cm[3][128];
    alignas(64) uint8_t sm[3][128];
    uint32_t rows[3], fmts[3], offs[3];
    uint32_t n = 0, off = 0;
    auto mi = mats.begin();
    for (const DevMat* d : dms) {
      std::memcpy(cm[n], (*mi)->codes, 128);
      std::memcpy(sm[n], (*mi)->scales, 128);
      rows[n] = d->rows;
      fmts[n] = d->format;
      offs[n] = off;
      off += d->rows;
      ++n;
      ++mi;
    }
    return ok(launch_gemm_jobs(cm, sm, rows, fmts, offs, n, bmap, cols, kMaxStreams, splits, out, ld, P.error, st, 1,
                               P.timeout_ns));
  };
  float* part = b.part0.as<float>();
  QWC_TRY(ok(launch_streams_norm(P, 1, m.layers[0].attn_norm, nullptr, 0, st)));
  for (uint32_t l = 0; l < m.n_layers; ++l) {
    const DevLayer& L = m.layers[l];
    if (l > 0) QWC_TRY(ok(launch_streams_norm(P, 0, L.attn_norm, part, b.splits_down, st)));
    QWC_TRY(gemm({&b.mq[l], &b.mk[l], &b.mv[l]}, {&L.q, &L.k, &L.v}, b.b_h, m.hidden, b.splits_qkv, part,
                 qw + 2 * kvw));
    QWC_TRY(ok(launch_streams_qkv(P, l, b.splits_qkv, m.kv_heads, st)));
    QWC_TRY(ok(launch_streams_attention(P, b.kv, l, b.attn_grid, st)));
    QWC_TRY(gemm({&b.mo[l]}, {&L.o}, b.b_q, qw, b.splits_o, part, m.hidden));
    QWC_TRY(ok(launch_streams_norm(P, 0, L.ffn_norm, part, b.splits_o, st)));
    QWC_TRY(gemm({&b.mg[l], &b.mu[l]}, {&L.gate, &L.up}, b.b_h, m.hidden, b.splits_gu, part, 2 * m.ffn));
    QWC_TRY(ok(launch_streams_swiglu(P, b.splits_gu, st)));
    QWC_TRY(gemm({&b.md[l]}, {&L.down}, b.b_f, m.ffn, b.splits_down, part, m.hidden));
  }
  if (!logits) {
    b.kernels_per_step_nologits = kernels;
    return QWC_OK;
  }
  QWC_TRY(ok(launch_streams_norm(P, 0, m.final_norm, part, b.splits_down, st)));
  QWC_TRY(gemm({&b.mlm}, {&m.lm_head}, b.b_h, m.hidden, 1, b.logits.as<float>(), m.vocab));
  QWC_TRY(ok(launch_streams_argmax(P, st)));
  QWC_TRY(ok(launch_streams_advance(P, b.history.as<uint32_t>(), b.counter.as<uint32_t>(), b.history_rows, st)));
  b.kernels_per_step = kernels;
  return QWC_OK;
}

// Records the step once as a CUDA graph (replayed every step), replacing any
// earlier recording; kernel parameters such as the wait bound are fixed at
// capture.
int32_t capture_one(Handle* h, bool logits, cudaGraph_t* graph_out, cudaGraphExec_t* exec_out) {
  if (*exec_out) cudaGraphExecDestroy(*exec_out);
  if (*graph_out) cudaGraphDestroy(*graph_out);
  *exec_out = nullptr;
  *graph_out = nullptr;
  QWC_CUDA(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
  const int32_t rec = record_step(h, logits);
  cudaGraph_t graph = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(h->stream, &graph);
  if (rec != QWC_OK || ce != cudaSuccess) {
    if (graph) cudaGraphDestroy(graph);
    cudaGetLastError();
    return rec != QWC_OK ? rec : status_of(ce);
  }
  *graph_out = graph;
  const cudaError_t ie = cudaGraphInstantiate(exec_out, graph, 0);
  if (ie != cudaSuccess) return status_of(ie);
  return QWC_OK;
}

int32_t capture_step(Handle* h) {
  Batched& b = *h->batched;
  QWC_TRY(capture_one(h, true, &b.graph, &b.exec));
  return capture_one(h, false, &b.graph_nologits, &b.exec_nologits);
}

int32_t build_batched(Handle* h) {
  const DevModel& m = h->host_model;
  const Config& c = h->config;
  auto bp = std::make_unique<Batched>();
  Batched& b = *bp;
  const uint32_t qw = m.q_heads * kHeadDim, kvw = m.kv_heads * kHeadDim;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, h->device);
  b.splits_qkv = gemm_splits(qw + 2 * kvw, m.hidden, sms);
  b.splits_o = gemm_splits(m.hidden, qw, sms);
  b.splits_gu = gemm_splits(2 * m.ffn, m.hidden, sms);
  b.splits_down = gemm_splits(m.hidden, m.ffn, sms);
  b.attn_grid = sms;  // one attention CTA per SM (its ring fills most of the shared memory)
  const size_t part_cols = std::max({size_t(b.splits_qkv) * (qw + 2 * kvw), size_t(b.splits_o) * m.hidden,
                                     size_t(b.splits_gu) * 2 * m.ffn, size_t(b.splits_down) * m.hidden});
  const size_t S = kMaxStreams;
  QWC_TRY(b.hidden.alloc(S * m.hidden * 4));
  QWC_TRY(b.xb_h.alloc(2 * S * m.hidden * 2));
  QWC_TRY(b.xb_q.alloc(2 * S * qw * 2));
  QWC_TRY(b.xb_f.alloc(2 * S * m.ffn * 2));
  QWC_TRY(b.part0.alloc(S * part_cols * 4));
  QWC_TRY(b.qrot.alloc(S * qw * 4));
  QWC_TRY(b.attn_part.alloc(S * m.q_heads * h->max_chunks * (kHeadDim + 4) * 4));
  QWC_TRY(b.attn_count.alloc(S * m.kv_heads * 4));
  QWC_TRY(b.logits.alloc(S * m.vocab * 4));
  QWC_TRY(b.qkv_rows.alloc(S * (qw + 2 * kvw) * 4));
  QWC_TRY(b.tokens.alloc(S * 4));
  QWC_TRY(b.desc.alloc(S * sizeof(SlotStep)));
  QWC_TRY(b.audio_ptrs.alloc(S * sizeof(float*)));
  QWC_TRY(b.err.alloc(256));
  b.history_rows = std::max<uint32_t>(c.max_positions, 1);
  QWC_TRY(b.history.alloc(size_t(b.history_rows) * S * 4));
  QWC_TRY(b.counter.alloc(256));
  for (DevBuf* z : {&b.hidden, &b.xb_h, &b.xb_q, &b.xb_f, &b.attn_count, &b.tokens, &b.desc, &b.audio_ptrs, &b.err,
                    &b.counter}) {
    QWC_CUDA(cudaMemset(z->ptr, 0, z->bytes));
  }
  // Attention partials: a NaN max marks "no segment starts at this chunk".
  QWC_CUDA(cudaMemset(b.attn_part.ptr, 0xFF, b.attn_part.bytes));
  if (cudaMallocHost(&b.host_desc, S * sizeof(SlotStep)) != cudaSuccess ||
      cudaMallocHost(&b.host_tokens, S * 4) != cudaSuccess || cudaMallocHost(&b.host_err, 64) != cudaSuccess) {
    cudaGetLastError();
    return QWC_OUT_OF_MEMORY;
  }
  const uint32_t L = m.n_layers;
  for (auto* v : {&b.mq, &b.mk, &b.mv, &b.mo, &b.mg, &b.mu, &b.md}) v->resize(L);
  for (uint32_t l = 0; l < L; ++l) {
    const DevLayer& D = m.layers[l];
    QWC_TRY(mat_maps(D.q, &b.mq[l]));
    QWC_TRY(mat_maps(D.k, &b.mk[l]));
    QWC_TRY(mat_maps(D.v, &b.mv[l]));
    QWC_TRY(mat_maps(D.o, &b.mo[l]));
    QWC_TRY(mat_maps(D.gate, &b.mg[l]));
    QWC_TRY(mat_maps(D.up, &b.mu[l]));
    QWC_TRY(mat_maps(D.down, &b.md[l]));
  }
  QWC_TRY(mat_maps(m.lm_head, &b.mlm));
  QWC_TRY(act_map(b.b_h, b.xb_h.ptr, m.hidden));
  QWC_TRY(act_map(b.b_q, b.xb_q.ptr, qw));
  QWC_TRY(act_map(b.b_f, b.xb_f.ptr, m.ffn));
  const uint64_t scale_row = uint64_t(kvw / kGroup) * 2;
  QWC_TRY(kv_map4(b.kv.k_codes, h->k_cache.as<uint8_t>() + m.cache_scales_bytes, kvw, m, h->streams, kHeadDim, true));
  QWC_TRY(kv_map4(b.kv.v_codes, h->v_cache.as<uint8_t>() + m.cache_scales_bytes, kvw, m, h->streams, kHeadDim, true));
  QWC_TRY(kv_map4(b.kv.k_scales, h->k_cache.as<uint8_t>(), scale_row, m, h->streams, 16, false));
  QWC_TRY(kv_map4(b.kv.v_scales, h->v_cache.as<uint8_t>(), scale_row, m, h->streams, 16, false));

  StreamsStep& P = b.P;
  P.model = h->model_buf.as<DevModel>();
  P.desc = b.desc.as<SlotStep>();
  P.audio = b.audio_ptrs.as<const float*>();
  P.hidden = b.hidden.as<float>();
  P.xb_h = b.xb_h.ptr;
  P.xb_q = b.xb_q.ptr;
  P.xb_f = b.xb_f.ptr;
  P.part0 = b.part0.as<float>();
  P.qrot = b.qrot.as<float>();
  P.attn_part = b.attn_part.as<float>();
  P.attn_count = b.attn_count.as<uint32_t>();
  P.k_cache = h->k_cache.as<uint8_t>();
  P.v_cache = h->v_cache.as<uint8_t>();
  P.logits = b.logits.as<float>();
  P.qkv_rows = b.qkv_rows.as<float>();
  P.tokens = b.tokens.as<uint32_t>();
  P.error = b.err.as<int32_t>();
  P.max_chunks = h->max_chunks;
  P.timeout_ns = h->wait_limit_ns ? h->wait_limit_ns : kBatchedWaitNs;

  int e = prepare_gemm_kernel();
  if (e == 0) e = prepare_stream_kernels();
  if (e != 0) return status_of(static_cast<cudaError_t>(e));
  h->batched = std::move(bp);
  const int32_t st = capture_step(h);
  if (st != QWC_OK) h->batched.reset();
  return st;
}

// Runs the captured step once for the columns in b.host_desc and, with
// `logits`, reads the argmax of every column back.
int32_t run_batched(Handle* h, bool logits = true) {
  Batched& b = *h->batched;
  cudaStream_t st = h->stream;
  QWC_CUDA(cudaMemcpyAsync(b.desc.ptr, b.host_desc, kMaxStreams * sizeof(SlotStep), cudaMemcpyHostToDevice, st));
  QWC_CUDA(cudaGraphLaunch(logits ? b.exec : b.exec_nologits, st));
  if (logits) QWC_CUDA(cudaMemcpyAsync(b.host_tokens, b.tokens.ptr, kMaxStreams * 4, cudaMemcpyDeviceToHost, st));
  QWC_CUDA(cudaMemcpyAsync(b.host_err, b.err.ptr, 16, cudaMemcpyDeviceToHost, st));
  QWC_CUDA(cudaStreamSynchronize(st));
  h->launches += logits ? b.kernels_per_step : b.kernels_per_step_nologits;
  if (*b.host_err != 0) {
    if (std::getenv("QWC_VERBOSE")) {
      std::fprintf(stderr, "qwc: batched step gave up waiting (code %d, detail %d %d %d)\n", b.host_err[0],
                   b.host_err[1], b.host_err[2], b.host_err[3]);
    }
    cudaMemsetAsync(b.err.ptr, 0, 16, st);
    cudaStreamSynchronize(st);
    return QWC_INVALID_STATE;
  }
  return QWC_OK;
}

// Decoder.prefill (decoder.zig:308-333) of one stream in 64-position steps:
// the columns of a step are consecutive positions of the stream, sharing its
// cache. Returns the prediction after the prompt's last position.
int32_t batched_prefill(Handle* h, uint32_t slot, const uint32_t* prompt, const std::vector<int32_t>& rows,
                        uint32_t prompt_len, uint32_t* next_out, uint32_t* column_out) {
  Batched& b = *h->batched;
  uint32_t last_col = 0;
  for (uint32_t c0 = 0; c0 < prompt_len; c0 += kMaxStreams) {
    const uint32_t n = std::min<uint32_t>(kMaxStreams, prompt_len - c0);
    for (uint32_t i = 0; i < kMaxStreams; ++i) {
      b.host_desc[i] = i < n ? SlotStep{1, c0 + i, static_cast<int32_t>(prompt[c0 + i]), rows[c0 + i],
                                        static_cast<int32_t>(slot), {0, 0, 0}}
                             : SlotStep{0, 0, 0, -1, 0, {0, 0, 0}};
    }
    // Decoder.prefill computes logits at the prompt's last position only (decoder.zig:308-333).
    QWC_TRY(run_batched(h, c0 + n == prompt_len));
    last_col = n - 1;
  }
  *next_out = b.host_tokens[last_col];
  *column_out = last_col;
  return QWC_OK;
}

// One batched decode step (streams > 1), the reference's decodeStep per slot
// (src/wasm/model.zig:423-451): each decoding slot emits its held token
// unless it ends the sequence, then the held token is fed through the step
// to predict the next. results[slot]: 1 token emitted, 0 finished or idle.
int32_t batched_step(Handle* h, uint32_t* tokens_out, int32_t* results) {
  Batched& b = *h->batched;
  const Config& c = h->config;
  const uint32_t n = static_cast<uint32_t>(h->slots.size());
  bool any = false;
  int32_t produced = 0;
  for (uint32_t slot = 0; slot < kMaxStreams; ++slot) {
    SlotStep d{0, 0, 0, -1, 0, {0, 0, 0}};
    if (slot < n) {
      StreamSlot& s = h->slots[slot];
      results[slot] = 0;
      if (s.decoding && !s.finished) {
        const uint32_t t = s.next_token;
        if (!h->ignore_eos && ends_sequence(c, t)) {
          s.finished = true;  // EOS ends the stream and is not emitted
        } else {
          tokens_out[slot] = t;
          s.generated.push_back(t);
          results[slot] = 1;
          ++produced;
          if (s.generated.size() >= s.max_tokens) {
            s.finished = true;
          } else if (s.position >= c.max_positions) {
            results[slot] = QWC_LIMIT_EXCEEDED;  // PositionExceeded (decoder.zig:142)
            s.finished = true;
          } else {
            d = SlotStep{1, s.position, static_cast<int32_t>(t), -1, static_cast<int32_t>(slot), {0, 0, 0}};
          }
        }
      }
    }
    b.host_desc[slot] = d;
    any = any || d.active;
  }
  if (!any) return produced;
  QWC_TRY(run_batched(h));
  for (uint32_t slot = 0; slot < n; ++slot) {
    if (!b.host_desc[slot].active) continue;
    StreamSlot& s = h->slots[slot];
    s.position += 1;
    s.next_token = b.host_tokens[slot];
    s.logits_batched = true;
    s.logits_col = slot;
  }
  return produced;
}

// `steps` device-chained decode steps of every decoding slot (streams > 1),
// timed with CUDA events: as `steps` qwc_streams_step calls without the stop
// rule, with the emitted tokens appended afterwards.
int32_t batched_run_timed(Handle* h, uint32_t steps, float* device_ms) {
  Batched& b = *h->batched;
  const uint32_t n = static_cast<uint32_t>(h->slots.size());
  bool any = false;
  for (uint32_t slot = 0; slot < kMaxStreams; ++slot) {
    SlotStep d{0, 0, 0, -1, 0, {0, 0, 0}};
    if (slot < n) {
      StreamSlot& s = h->slots[slot];
      if (s.decoding && !s.finished) {
        if (s.position + steps > h->config.max_positions) return QWC_LIMIT_EXCEEDED;
        if (s.generated.size() + steps > s.max_tokens) return QWC_LIMIT_EXCEEDED;
        d = SlotStep{1, s.position, static_cast<int32_t>(s.next_token), -1, static_cast<int32_t>(slot), {0, 0, 0}};
      }
    }
    b.host_desc[slot] = d;
    any = any || d.active;
  }
  if (!any || steps == 0 || steps > b.history_rows) return QWC_INVALID_ARGUMENT;
  cudaStream_t st = h->stream;
  QWC_CUDA(cudaMemcpyAsync(b.desc.ptr, b.host_desc, kMaxStreams * sizeof(SlotStep), cudaMemcpyHostToDevice, st));
  QWC_CUDA(cudaMemsetAsync(b.counter.ptr, 0, 4, st));
  cudaEvent_t e0, e1;
  QWC_CUDA(cudaEventCreate(&e0));
  QWC_CUDA(cudaEventCreate(&e1));
  cudaEventRecord(e0, st);
  cudaError_t le = cudaSuccess;
  for (uint32_t i = 0; i < steps && le == cudaSuccess; ++i) le = cudaGraphLaunch(b.exec, st);
  cudaEventRecord(e1, st);
  std::vector<uint32_t> hist(size_t(steps) * kMaxStreams);
  if (le == cudaSuccess) {
    le = cudaMemcpyAsync(hist.data(), b.history.ptr, hist.size() * 4, cudaMemcpyDeviceToHost, st);
  }
  if (le == cudaSuccess) le = cudaMemcpyAsync(b.host_err, b.err.ptr, 16, cudaMemcpyDeviceToHost, st);
  if (le == cudaSuccess) le = cudaStreamSynchronize(st);
  float ms = 0.0f;
  if (le == cudaSuccess) cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (le != cudaSuccess) return status_of(le);
  h->launches += uint64_t(b.kernels_per_step) * steps;
  if (*b.host_err != 0) {
    cudaMemsetAsync(b.err.ptr, 0, 16, st);
    cudaStreamSynchronize(st);
    return QWC_INVALID_STATE;
  }
  for (uint32_t slot = 0; slot < n; ++slot) {
    if (!b.host_desc[slot].active) continue;
    StreamSlot& s = h->slots[slot];
    for (uint32_t i = 0; i < steps; ++i) {
      s.generated.push_back(s.next_token);
      s.next_token = hist[size_t(i) * kMaxStreams + slot];
    }
    s.position += steps;
    s.logits_batched = true;
    s.logits_col = slot;
    if (s.generated.size() >= s.max_tokens) s.finished = true;
  }
  *device_ms = ms;
  return QWC_OK;
}

// `audio_on_device`: the audio rows are device memory (the tower's output)
// rather than host memory.
int32_t stream_begin(Handle* h, uint32_t slot, const uint32_t* prompt, uint32_t prompt_len, const float* audio,
                     uint32_t audio_steps, uint32_t max_tokens, bool audio_on_device = false) {
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (slot >= h->slots.size()) return QWC_INVALID_ARGUMENT;
  StreamSlot& s = h->slots[slot];
  if (s.decoding) return QWC_INVALID_STATE;
  const Config& c = h->config;
  if (max_tokens == 0 || max_tokens > c.max_decode_tokens) return QWC_LIMIT_EXCEEDED;  // model.zig:380-381
  if (!prompt || prompt_len == 0) return QWC_SHAPE_MISMATCH;                            // decoder.zig:317
  if (audio_steps > 0 && !audio) return QWC_INVALID_ARGUMENT;
  if (prompt_len > c.max_positions) return QWC_LIMIT_EXCEEDED;                          // decoder.zig:142
  std::vector<int32_t> rows(prompt_len);
  uint32_t audio_index = 0;
  for (uint32_t i = 0; i < prompt_len; ++i) {
    if (prompt[i] >= c.vocab_size) return QWC_SHAPE_MISMATCH;  // embeddingRow bounds (decoder.zig:365-367)
    if (prompt[i] == c.token_audio_pad) {
      if (audio_index >= audio_steps) return QWC_SHAPE_MISMATCH;  // PromptMismatch (decoder.zig:323)
      rows[i] = static_cast<int32_t>(audio_index++);
    } else {
      rows[i] = -1;
    }
  }
  if (audio_index != audio_steps) return QWC_SHAPE_MISMATCH;  // decoder.zig:331
  cudaSetDevice(h->device);
  // Decoder.reset (decoder.zig:109-121): the slot's cache goes back to zero.
  const uint64_t stride = h->host_model.cache_stream_stride;
  QWC_CUDA(cudaMemsetAsync(h->k_cache.as<uint8_t>() + stride * slot, 0, stride, h->stream));
  QWC_CUDA(cudaMemsetAsync(h->v_cache.as<uint8_t>() + stride * slot, 0, stride, h->stream));
  s = StreamSlot{};
  const float* dev_audio = nullptr;
  if (audio_steps) {
    s.audio = std::make_unique<DevBuf>();
    QWC_TRY(s.audio->alloc(size_t(audio_steps) * c.text_hidden_size * 4));
    QWC_CUDA(cudaMemcpyAsync(s.audio->ptr, audio, s.audio->bytes,
                             audio_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, h->stream));
    dev_audio = s.audio->as<float>();
  }
  if (h->batched) {
    QWC_CUDA(cudaMemcpyAsync(h->batched->audio_ptrs.as<const float*>() + slot, &dev_audio, sizeof(dev_audio),
                             cudaMemcpyHostToDevice, h->stream));
  }
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  uint32_t next = 0, col = 0;
  const bool serial = (h->prefill_serial || h->exact || !h->batched) && h->streams == 1;
  if (serial) {
    // Token by token through the persistent kernel (decoder.zig:308-333 as written).
    QWC_CUDA(cudaMemcpyAsync(h->prompt_ids.ptr, prompt, size_t(prompt_len) * 4, cudaMemcpyHostToDevice, h->stream));
    QWC_CUDA(cudaMemcpyAsync(h->prompt_rows.ptr, rows.data(), size_t(prompt_len) * 4, cudaMemcpyHostToDevice,
                             h->stream));
    if (audio_steps) {
      QWC_CUDA(cudaMemcpyAsync(h->audio_rows.ptr, audio, size_t(audio_steps) * c.text_hidden_size * 4,
                               audio_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, h->stream));
    }
    std::vector<uint32_t> tokens;
    QWC_TRY(run_decode(h, prompt_len, 0, prompt_len, 0, prompt_len - 1, &tokens));
    next = tokens[prompt_len - 1];
  } else {
    QWC_TRY(batched_prefill(h, slot, prompt, rows, prompt_len, &next, &col));
  }
  s.decoding = true;
  s.position = prompt_len;
  s.next_token = next;
  s.max_tokens = max_tokens;
  s.generated.reserve(max_tokens);
  s.logits_batched = !serial;
  s.logits_col = col;
  return QWC_OK;
}

// Computes the prediction that follows `token` (which sits at s.position),
// launching a chunk of steps ahead when none is buffered.
int32_t advance(Handle* h, StreamSlot& s, uint32_t token, uint32_t budget) {
  if (s.ahead.empty()) {
    const Config& c = h->config;
    if (s.position >= c.max_positions) return QWC_LIMIT_EXCEEDED;  // PositionExceeded (decoder.zig:142)
    uint32_t n = std::min<uint32_t>(h->step_chunk, budget);
    n = std::min<uint32_t>(n, c.max_positions - s.position);
    n = std::max<uint32_t>(n, 1);
    std::vector<uint32_t> tokens;
    QWC_TRY(run_decode(h, n, s.position, 0, token, 0, &tokens));
    for (uint32_t i = 0; i < n; ++i) s.ahead.push_back(tokens[i]);
    s.position += n;
    s.logits_batched = false;
  }
  s.next_token = s.ahead.front();
  s.ahead.pop_front();
  return QWC_OK;
}

// src/wasm/model.zig:423-451
int32_t stream_step(Handle* h, uint32_t slot, uint32_t* token_out) {
  if (h->state != State::kLoaded || slot >= h->slots.size()) return QWC_INVALID_STATE;
  if (h->streams > 1) return QWC_UNSUPPORTED;  // multi-stream handles advance with qwc_streams_step
  StreamSlot& s = h->slots[slot];
  if (!s.decoding) return QWC_INVALID_STATE;
  if (s.finished) return 0;
  if (!h->ignore_eos && ends_sequence(h->config, s.next_token)) {
    s.finished = true;
    return 0;
  }
  if (s.generated.size() >= s.max_tokens) {
    s.finished = true;
    return 0;
  }
  *token_out = s.next_token;
  s.generated.push_back(s.next_token);
  if (s.generated.size() >= s.max_tokens) {
    s.finished = true;
    return 1;
  }
  const uint32_t budget = s.max_tokens - static_cast<uint32_t>(s.generated.size());
  QWC_TRY(advance(h, s, s.next_token, budget));
  return 1;
}

}  // namespace
}  // namespace qwc

using namespace qwc;

namespace {

uint64_t audio_wait_ns(const Handle* h) { return h->wait_limit_ns ? h->wait_limit_ns : kBatchedWaitNs; }

// Uploads one clip's log-mel features and runs the tower and projector into
// h->audio_out. model.zig:380-386's checks: a whole number of mel columns,
// at least one frame, at most the mel capacity.
int32_t run_audio(Handle* h, const float* features, uint64_t floats, uint32_t* steps_out) {
  if (!h->audio) return QWC_NOT_FOUND;
  if (!features) return QWC_INVALID_ARGUMENT;
  const AudioGeometry& g = h->audio->g;
  if (floats == 0 || floats % g.mel_bins != 0) return QWC_SHAPE_MISMATCH;
  const uint64_t frames = floats / g.mel_bins;
  if (frames > g.max_frames) return QWC_AUDIO_TOO_LONG;
  cudaSetDevice(h->device);
  float* mel = h->audio->mel_buffer();
  QWC_CUDA(cudaMemcpyAsync(mel, features, floats * 4, cudaMemcpyHostToDevice, h->stream));
  const int32_t st = h->audio->run(mel, static_cast<uint32_t>(frames), h->audio_out.as<float>(), h->stream,
                                   audio_wait_ns(h), steps_out);
  h->launches += h->audio->launches();
  return st;
}

}  // namespace

extern "C" {

uint32_t qwc_abi_version(void) { return (QWC_ABI_MAJOR << 16) | QWC_ABI_MINOR; }

uint32_t qwc_features(void) { return QWC_FEATURE_MODEL | QWC_FEATURE_DECODE | QWC_FEATURE_STREAMS; }

const char* qwc_status_message(int32_t status) {
  switch (status) {
    case QWC_OK: return "ok";
    case QWC_INVALID_ARGUMENT: return "invalid argument";
    case QWC_OUT_OF_MEMORY: return "out of memory";
    case QWC_UNSUPPORTED: return "unsupported";
    case QWC_BAD_MAGIC: return "bad magic";
    case QWC_BAD_VERSION: return "bad version";
    case QWC_CHECKSUM_MISMATCH: return "checksum mismatch";
    case QWC_SHAPE_MISMATCH: return "shape mismatch";
    case QWC_INVALID_STATE: return "invalid state";
    case QWC_LIMIT_EXCEEDED: return "limit exceeded";
    case QWC_NOT_FOUND: return "not found";
    case QWC_TRUNCATED: return "truncated input";
    case QWC_INVALID_ENCODING: return "invalid encoding";
    case QWC_UNSUPPORTED_MODEL: return "unsupported model";
    case QWC_AUDIO_TOO_LONG: return "audio too long";
    default: return "unknown status";
  }
}

uint32_t qwc_create(int32_t device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  if (device < 0 || device >= count) return 0;
  if (cudaSetDevice(device) != cudaSuccess) return 0;
  auto h = std::make_unique<Handle>();
  h->device = device;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(g_mutex);
  const uint32_t id = g_next_handle++;
  g_handles[id] = std::move(h);
  return id;
}

int32_t qwc_destroy(uint32_t handle) {
  std::unique_ptr<Handle> h;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = g_handles.find(handle);
    if (it == g_handles.end()) return QWC_INVALID_ARGUMENT;
    h = std::move(it->second);
    g_handles.erase(it);
  }
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  release_model(h.get());
  return QWC_OK;
}

int32_t qwc_set_option(uint32_t handle, uint32_t option, uint32_t value) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  switch (option) {
    case QWC_OPTION_IGNORE_EOS: h->ignore_eos = value != 0; return QWC_OK;
    case QWC_OPTION_KEEP_LOGITS: h->keep_logits = value != 0; return QWC_OK;
    case QWC_OPTION_TRACE: h->trace = value != 0; return QWC_OK;
    case QWC_OPTION_PREFILL_SERIAL: h->prefill_serial = value != 0; return QWC_OK;
    case QWC_OPTION_EXACT: h->exact = value != 0; return QWC_OK;
    case QWC_OPTION_TEST_STALL: h->test_stall = value != 0; return QWC_OK;
    case QWC_OPTION_WAIT_LIMIT_US:
      h->wait_limit_ns = uint64_t(value) * 1000ull;
      if (h->batched) {
        cudaSetDevice(h->device);
        h->batched->P.timeout_ns = h->wait_limit_ns ? h->wait_limit_ns : kBatchedWaitNs;
        return capture_step(h);
      }
      return QWC_OK;
    case QWC_OPTION_STEP_CHUNK:
      if (value == 0 || value > 256) return QWC_INVALID_ARGUMENT;
      h->step_chunk = value;
      return QWC_OK;
    default: return QWC_INVALID_ARGUMENT;
  }
}

// src/wasm/model.zig:136-141: releases whatever the handle holds.
int32_t qwc_model_begin(uint32_t handle) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  release_model(h);
  h->cache_format = QWC_CACHE_F32;
  h->streams = 1;
  h->state = State::kReady;
  return QWC_OK;
}

}  // extern "C"

namespace {

// Copies one tensor's payload to the device and records it under (kind, layer).
int32_t add_tensor(Handle* h, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows, uint32_t cols,
                   const void* payload, uint64_t len) {
  if (h->state != State::kReady) return QWC_INVALID_STATE;
  if (!payload || rows == 0 || cols == 0) return QWC_INVALID_ARGUMENT;
  if (!is_audio_kind(kind) && (kind < QWC_KIND_DECODER_EMBED_TOKENS || kind > QWC_KIND_DECODER_DOWN)) {
    return QWC_UNSUPPORTED_MODEL;
  }
  if (h->tensors.count({kind, layer})) return QWC_INVALID_ARGUMENT;  // DuplicateTensor
  Tensor t;
  t.kind = kind;
  t.layer = layer;
  t.format = format;
  t.rows = rows;
  t.cols = cols;
  uint64_t need = 0;
  if (format == QWC_FORMAT_F32) {
    need = uint64_t(rows) * cols * 4;
  } else if (format == QWC_FORMAT_F16 && is_conv_kind(kind)) {
    need = uint64_t(rows) * cols * 2;  // layout.zig:150-175: the convolutions stay f16 (element_f16)
  } else if (format == QWC_FORMAT_Q4 || format == QWC_FORMAT_Q5 || format == QWC_FORMAT_Q8) {
    if (cols % kGroup != 0) return QWC_SHAPE_MISMATCH;  // RowNotGroupAligned (quant.zig:77-81)
    // quant.zig:144-176 with a 16-byte-aligned base.
    const uint64_t groups = uint64_t(rows) * (cols / kGroup);
    const uint64_t scales_len = groups * 2;
    t.scales_offset = 0;
    t.codes_offset = (scales_len + 15) / 16 * 16;
    need = t.codes_offset + groups * data_bytes_per_group(format);
  } else {
    return QWC_UNSUPPORTED_MODEL;
  }
  if (len < need) return QWC_TRUNCATED;
  cudaSetDevice(h->device);
  t.buf = std::make_unique<DevBuf>();
  QWC_TRY(t.buf->alloc(need));
  QWC_CUDA(cudaMemcpy(t.buf->ptr, payload, need, cudaMemcpyHostToDevice));
  h->weight_bytes += need;
  t.src_len = len;
  t.rank = (rows == 1 && (is_vector_kind(kind) || is_audio_vector_kind(kind))) ? 1u : 2u;
  t.dims[0] = t.rank == 1 ? cols : rows;
  if (t.rank == 2) t.dims[1] = cols;
  h->tensors.emplace(std::make_pair(kind, layer), std::move(t));
  return QWC_OK;
}

}  // namespace

extern "C" {

int32_t qwc_model_add_tensor(uint32_t handle, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows,
                             uint32_t cols, const void* payload, uint64_t len) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  QWC_TRY(add_tensor(h, kind, layer, format, rows, cols, payload, len));
  const Tensor& t = h->tensors.at({kind, layer});
  qwc_tensor_descriptor d{};
  d.offset_bytes = 0;
  d.len_bytes = t.src_len;
  d.kind = kind;
  d.layer = layer;
  d.format = format;
  d.rank = t.rank;
  for (int i = 0; i < 4; ++i) d.dims[i] = t.dims[i];
  d.shard_index = 0xFFFFFFFFu;
  h->descriptors.push_back(d);
  return QWC_OK;
}

int32_t qwc_model_add_shard(uint32_t handle, const void* bytes, uint64_t len) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kReady) return QWC_INVALID_STATE;
  if (h->shards.size() >= kShardCountMax) return QWC_LIMIT_EXCEEDED;
  ShardView v;
  QWC_TRY(parse_shard(bytes, len, &v));
  // DuplicateShard: the reference also compares buffer addresses, which here
  // can repeat legitimately (the caller may free a shard after the call and
  // reuse the memory), so only the payload checksum identifies a repeat.
  for (uint32_t c : h->shards) {
    if (c == v.checksum) return QWC_INVALID_ARGUMENT;
  }
  // Every tensor is checked before any is copied, so a rejected shard leaves
  // the handle as it was. Decoder, audio-tower and projector tensors are kept
  // on the device.
  auto kept_kind = [](uint32_t kind) {
    return is_audio_kind(kind) || (kind >= QWC_KIND_DECODER_EMBED_TOKENS && kind <= QWC_KIND_DECODER_DOWN);
  };
  for (uint32_t i = 0; i < v.count; ++i) {
    const ShardEntry e = shard_entry(v, i);
    if (!kept_kind(e.kind)) continue;
    const bool vec = e.rank == 1 && e.format == QWC_FORMAT_F32;
    const bool mat = e.rank == 2 && (e.format == QWC_FORMAT_Q4 || e.format == QWC_FORMAT_Q5 ||
                                     e.format == QWC_FORMAT_Q8 || e.format == QWC_FORMAT_F32);
    const bool conv = e.rank == 4 && e.format == QWC_FORMAT_F16 && is_conv_kind(e.kind);
    if (!vec && !mat && !conv) return QWC_UNSUPPORTED_MODEL;
    if (h->tensors.count({e.kind, e.layer})) return QWC_INVALID_ARGUMENT;  // DuplicateTensor
  }
  // A copy that fails part way (out of device memory) takes back the
  // tensors this shard added, so the handle is as it was and the same shard
  // may be added again.
  std::vector<std::pair<uint32_t, uint32_t>> added;
  const uint64_t weight_bytes0 = h->weight_bytes;
  for (uint32_t i = 0; i < v.count; ++i) {
    const ShardEntry e = shard_entry(v, i);
    if (!kept_kind(e.kind)) continue;
    // A convolution [out][in][3][3] is kept as out rows of in * 9 values.
    const uint32_t rows = e.rank == 1 ? 1u : e.dims[0];
    const uint32_t cols = e.rank == 1 ? e.dims[0] : e.rank == 4 ? e.dims[1] * e.dims[2] * e.dims[3] : e.dims[1];
    const int32_t st = add_tensor(h, e.kind, e.layer, e.format, rows, cols, v.payload + e.offset_bytes, e.len_bytes);
    if (st != QWC_OK) {
      for (const auto& key : added) h->tensors.erase(key);
      h->weight_bytes = weight_bytes0;
      return st;
    }
    added.emplace_back(e.kind, e.layer);
  }
  // model.zig:298-310: one descriptor per entry, the offset absolute within
  // the shard's bytes.
  const uint32_t shard_index = static_cast<uint32_t>(h->shards.size());
  for (uint32_t i = 0; i < v.count; ++i) {
    const ShardEntry e = shard_entry(v, i);
    qwc_tensor_descriptor d{};
    d.offset_bytes = uint64_t(v.payload - v.bytes) + e.offset_bytes;
    d.len_bytes = e.len_bytes;
    d.kind = e.kind;
    d.layer = e.layer;
    d.format = e.format;
    d.rank = e.rank;
    for (int k = 0; k < 4; ++k) d.dims[k] = e.dims[k];
    d.shard_index = shard_index;
    h->descriptors.push_back(d);
  }
  h->shards.push_back(v.checksum);
  return QWC_OK;
}

int32_t qwc_model_set_cache_format(uint32_t handle, uint32_t format) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (format != QWC_CACHE_F32 && format != QWC_CACHE_Q8) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kReady || (h->tensors.empty() && h->shards.empty())) {
    return QWC_INVALID_STATE;  // model.zig:184-188
  }
  h->cache_format = format;
  return QWC_OK;
}

int32_t qwc_model_set_streams(uint32_t handle, uint32_t streams) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kReady) return QWC_INVALID_STATE;
  if (streams == 0) return QWC_INVALID_ARGUMENT;
  if (streams > kMaxStreams) return QWC_LIMIT_EXCEEDED;
  h->streams = streams;
  return QWC_OK;
}

int32_t qwc_model_finish(uint32_t handle, const void* config, uint32_t config_len) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kReady) return QWC_INVALID_STATE;
  if (!config) return QWC_INVALID_ARGUMENT;
  if (config_len != sizeof(Config)) return QWC_TRUNCATED;  // model_config.zig:353-354
  Config c;
  std::memcpy(&c, config, sizeof(Config));
  QWC_TRY(validate_config(c));
  if (h->tensors.empty()) return QWC_INVALID_STATE;  // model.zig:208
  const int32_t st = finish_model(h, c);
  if (st != QWC_OK) {
    // model.zig:197-204: a failed load releases what it allocated; shards stay.
    for (DevBuf* b : {&h->model_buf, &h->rope_cos, &h->rope_sin, &h->k_cache, &h->v_cache, &h->qkv, &h->attn_out,
                      &h->hidden_g, &h->act, &h->attn_part, &h->attn_count, &h->amax_val, &h->amax_idx, &h->barrier,
                      &h->error, &h->tokens_out, &h->logits, &h->prompt_ids, &h->prompt_rows, &h->audio_rows,
                      &h->exact_scratch, &h->audio_out}) {
      b->alloc(0);
    }
    h->audio.reset();
    h->batched.reset();
    return st;
  }
  h->state = State::kLoaded;
  return QWC_OK;
}

int32_t qwc_model_requirements(uint32_t handle, qwc_requirements* out) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  qwc_requirements r{};
  r.weight_bytes = h->weight_bytes;
  r.cache_bytes = h->k_cache.bytes + h->v_cache.bytes;
  uint64_t scratch = 0;
  for (const DevBuf* b : {&h->model_buf, &h->rope_cos, &h->rope_sin, &h->qkv, &h->attn_out, &h->hidden_g, &h->act,
                          &h->attn_part, &h->attn_count, &h->amax_val, &h->amax_idx, &h->barrier, &h->error,
                          &h->tokens_out, &h->logits, &h->prompt_ids, &h->prompt_rows, &h->audio_rows,
                          &h->exact_scratch}) {
    scratch += b->bytes;
  }
  r.scratch_bytes = scratch;
  r.total_bytes = r.weight_bytes + r.cache_bytes + r.scratch_bytes;
  r.max_positions = h->config.max_positions;
  r.max_audio_frames = kCapacityFrames;
  r.max_decode_tokens = h->config.max_decode_tokens;
  r.reserved = 0;
  *out = r;
  return QWC_OK;
}

int32_t qwc_model_tensor_count(uint32_t handle, uint32_t* out) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  *out = static_cast<uint32_t>(h->descriptors.size());
  return QWC_OK;
}

static_assert(sizeof(qwc_tensor_descriptor) == 64, "abi.zig:391: the descriptor is 64 bytes");

int32_t qwc_model_tensor_descriptor(uint32_t handle, uint32_t index, qwc_tensor_descriptor* out) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (index >= h->descriptors.size()) return QWC_NOT_FOUND;  // model.zig:318
  *out = h->descriptors[index];
  return QWC_OK;
}

int32_t qwc_decode_begin(uint32_t handle, const uint32_t* prompt, uint32_t prompt_len, const float* audio,
                         uint32_t audio_steps, uint32_t max_tokens) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->streams > 1) return QWC_UNSUPPORTED;  // the stream family drives multi-stream handles
  return stream_begin(h, 0, prompt, prompt_len, audio, audio_steps, max_tokens);
}

int32_t qwc_decode_step(uint32_t handle, uint32_t* token_out) {
  Handle* h = lookup(handle);
  if (!h || !token_out) return QWC_INVALID_ARGUMENT;
  cudaSetDevice(h->device);
  return stream_step(h, 0, token_out);
}

int32_t qwc_stream_tokens(uint32_t handle, uint32_t slot, uint32_t* out, uint32_t capacity) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || slot >= h->slots.size() || !h->slots[slot].decoding) return QWC_INVALID_STATE;
  const StreamSlot& s = h->slots[slot];
  if (capacity < s.generated.size()) return QWC_LIMIT_EXCEEDED;  // model.zig:455-461
  if (!s.generated.empty() && !out) return QWC_INVALID_ARGUMENT;
  std::copy(s.generated.begin(), s.generated.end(), out);
  return static_cast<int32_t>(s.generated.size());
}

int32_t qwc_decode_tokens(uint32_t handle, uint32_t* out, uint32_t capacity) {
  return qwc_stream_tokens(handle, 0, out, capacity);
}

int32_t qwc_stream_end(uint32_t handle, uint32_t slot) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || slot >= h->slots.size() || !h->slots[slot].decoding) return QWC_INVALID_STATE;
  cudaSetDevice(h->device);
  const uint64_t stride = h->host_model.cache_stream_stride;
  QWC_CUDA(cudaMemsetAsync(h->k_cache.as<uint8_t>() + stride * slot, 0, stride, h->stream));
  QWC_CUDA(cudaMemsetAsync(h->v_cache.as<uint8_t>() + stride * slot, 0, stride, h->stream));
  if (h->batched) {
    const float* none = nullptr;
    QWC_CUDA(cudaMemcpyAsync(h->batched->audio_ptrs.as<const float*>() + slot, &none, sizeof(none),
                             cudaMemcpyHostToDevice, h->stream));
  }
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  h->slots[slot] = StreamSlot{};
  return QWC_OK;
}

int32_t qwc_decode_end(uint32_t handle) { return qwc_stream_end(handle, 0); }

int32_t qwc_stream_begin(uint32_t handle, uint32_t slot, const uint32_t* prompt, uint32_t prompt_len,
                         const float* audio, uint32_t audio_steps, uint32_t max_tokens) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  return stream_begin(h, slot, prompt, prompt_len, audio, audio_steps, max_tokens);
}

int32_t qwc_streams_step(uint32_t handle, uint32_t* tokens_out, int32_t* results) {
  Handle* h = lookup(handle);
  if (!h || !tokens_out || !results) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  cudaSetDevice(h->device);
  if (h->streams > 1) return batched_step(h, tokens_out, results);
  int32_t produced = 0;
  for (uint32_t slot = 0; slot < h->slots.size(); ++slot) {
    if (!h->slots[slot].decoding) {
      results[slot] = 0;
      continue;
    }
    const int32_t r = stream_step(h, slot, &tokens_out[slot]);
    results[slot] = r;
    if (r == 1) ++produced;
    if (r < 0) return r;
  }
  return produced;
}

int32_t qwc_streams_run_timed(uint32_t handle, uint32_t steps, float* device_ms) {
  Handle* h = lookup(handle);
  if (!h || !device_ms) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || h->streams < 2) return QWC_INVALID_STATE;
  cudaSetDevice(h->device);
  return batched_run_timed(h, steps, device_ms);
}

int32_t qwc_decode_run_timed(uint32_t handle, uint32_t steps, float* device_ms) {
  Handle* h = lookup(handle);
  if (!h || !device_ms) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || h->slots.empty() || !h->slots[0].decoding) return QWC_INVALID_STATE;
  StreamSlot& s = h->slots[0];
  if (s.generated.size() + steps > s.max_tokens) return QWC_LIMIT_EXCEEDED;
  if (s.position + steps > h->config.max_positions) return QWC_LIMIT_EXCEEDED;
  cudaSetDevice(h->device);
  s.ahead.clear();
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  float total = 0.0f;
  uint32_t token = s.next_token;
  uint32_t done = 0;
  std::vector<uint32_t> tokens;
  int32_t st = QWC_OK;
  while (done < steps && st == QWC_OK) {
    const uint32_t n = std::min<uint32_t>(h->step_chunk, steps - done);
    cudaEventRecord(e0, h->stream);
    st = run_decode(h, n, s.position, 0, token, 0, &tokens);
    if (st != QWC_OK) break;
    cudaEventRecord(e1, h->stream);
    cudaEventSynchronize(e1);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    total += ms;
    for (uint32_t i = 0; i < n; ++i) {
      s.generated.push_back(token);
      token = tokens[i];
    }
    s.position += n;
    done += n;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  s.next_token = token;
  *device_ms = total;
  return st;
}

int32_t qwc_debug_logits(uint32_t handle, uint32_t slot, float* out, uint32_t count) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || slot >= h->slots.size()) return QWC_INVALID_STATE;
  if (count < h->config.vocab_size) return QWC_LIMIT_EXCEEDED;
  cudaSetDevice(h->device);
  if (h->slots[slot].logits_batched) {
    const float* row = h->batched->logits.as<float>() + size_t(h->slots[slot].logits_col) * h->config.vocab_size;
    QWC_CUDA(cudaMemcpyAsync(out, row, size_t(h->config.vocab_size) * 4, cudaMemcpyDeviceToHost, h->stream));
    QWC_CUDA(cudaStreamSynchronize(h->stream));
    return QWC_OK;
  }
  if (!h->keep_logits) return QWC_INVALID_STATE;
  QWC_CUDA(cudaMemcpyAsync(out, h->logits.ptr, size_t(h->config.vocab_size) * 4, cudaMemcpyDeviceToHost, h->stream));
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  return QWC_OK;
}

int32_t qwc_debug_hold(uint32_t handle, uint32_t slot, int64_t force, uint32_t* held_out) {
  Handle* h = lookup(handle);
  if (!h || !held_out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || slot >= h->slots.size() || !h->slots[slot].decoding) return QWC_INVALID_STATE;
  StreamSlot& s = h->slots[slot];
  if (force >= 0) {
    if (!s.ahead.empty()) return QWC_INVALID_STATE;
    if (static_cast<uint64_t>(force) >= h->config.vocab_size) return QWC_INVALID_ARGUMENT;
    s.next_token = static_cast<uint32_t>(force);
  }
  *held_out = s.next_token;
  return QWC_OK;
}

int32_t qwc_debug_scratch(uint32_t handle, uint32_t which, float* out, uint32_t count) {
  Handle* h = lookup(handle);
  if (!h || !out || which > 4) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (which == 4 && !h->batched) return QWC_INVALID_STATE;
  const DevBuf* b = which == 0 ? &h->hidden_g : which == 1 ? &h->qkv : which == 2 ? &h->attn_out
                  : which == 3 ? &h->act : &h->batched->qkv_rows;
  if (uint64_t(count) * 4 < b->bytes) return QWC_LIMIT_EXCEEDED;
  cudaSetDevice(h->device);
  QWC_CUDA(cudaMemcpyAsync(out, b->ptr, b->bytes, cudaMemcpyDeviceToHost, h->stream));
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  return static_cast<int32_t>(b->bytes / 4);
}

int32_t qwc_debug_trace(uint32_t handle, uint64_t* out, uint32_t count) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->trace_buf.bytes == 0) return QWC_INVALID_STATE;
  const uint64_t n = h->trace_buf.bytes / 8;
  if (count < n) return QWC_LIMIT_EXCEEDED;
  cudaSetDevice(h->device);
  QWC_CUDA(cudaMemcpyAsync(out, h->trace_buf.ptr, h->trace_buf.bytes, cudaMemcpyDeviceToHost, h->stream));
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  return static_cast<int32_t>(n);
}

int32_t qwc_debug_cache(uint32_t handle, uint32_t slot, uint32_t which, void* out, uint64_t len) {
  Handle* h = lookup(handle);
  if (!h || !out || which > 1) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded || slot >= h->slots.size()) return QWC_INVALID_STATE;
  const uint64_t stride = h->host_model.cache_stream_stride;
  if (len < stride) return QWC_LIMIT_EXCEEDED;
  cudaSetDevice(h->device);
  const uint8_t* src = (which == 0 ? h->k_cache.as<uint8_t>() : h->v_cache.as<uint8_t>()) + stride * slot;
  QWC_CUDA(cudaMemcpyAsync(out, src, stride, cudaMemcpyDeviceToHost, h->stream));
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  return QWC_OK;
}

int32_t qwc_model_audio_config(uint32_t handle, qwc_audio_config* out) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  const AudioGeometry g = audio_geometry(h->config);
  qwc_audio_config a{};
  a.d_model = g.d_model;
  a.layers = g.layers;
  a.attention_heads = g.heads;
  a.head_dim = g.head_dim;
  a.ffn_dim = g.ffn;
  a.downsample_hidden_size = g.channels;
  a.n_window = g.n_window;
  a.n_window_infer = g.n_window_infer;
  a.chunk_frames = g.chunk_frames;
  a.frequency_bins = g.bins;
  a.conv_out_input_features = g.conv_features;
  a.chunk_steps = g.chunk_steps;
  a.max_position_steps = g.max_position_steps;
  a.output_dim = g.output_dim;
  a.mel_bins = g.mel_bins;
  a.layer_norm_eps = g.eps;
  *out = a;
  return QWC_OK;
}

int32_t qwc_audio_project(uint32_t handle, const float* log_mel, uint32_t frames, float* out,
                          uint64_t out_capacity_floats, uint32_t* steps_out) {
  Handle* h = lookup(handle);
  if (!h || !out) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (!h->audio) return QWC_NOT_FOUND;
  if (frames == 0) return QWC_SHAPE_MISMATCH;
  if (frames > h->audio->g.max_frames) return QWC_AUDIO_TOO_LONG;
  const uint32_t steps = audio_packed_steps(h->audio->g, frames);
  if (out_capacity_floats < uint64_t(steps) * h->audio->g.output_dim) return QWC_LIMIT_EXCEEDED;
  uint32_t got = 0;
  QWC_TRY(run_audio(h, log_mel, uint64_t(frames) * h->audio->g.mel_bins, &got));
  QWC_CUDA(cudaMemcpyAsync(out, h->audio_out.ptr, uint64_t(got) * h->audio->g.output_dim * 4, cudaMemcpyDeviceToHost,
                           h->stream));
  QWC_CUDA(cudaStreamSynchronize(h->stream));
  if (steps_out) *steps_out = got;
  return QWC_OK;
}

int32_t qwc_stream_begin_features(uint32_t handle, uint32_t slot, const uint32_t* prompt, uint32_t prompt_len,
                                  const float* features, uint64_t features_len, uint32_t max_tokens) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (slot >= h->slots.size()) return QWC_INVALID_ARGUMENT;
  if (h->slots[slot].decoding) return QWC_INVALID_STATE;
  if (max_tokens == 0 || max_tokens > h->config.max_decode_tokens) return QWC_LIMIT_EXCEEDED;  // model.zig:380-381
  if (features_len == 0 || features_len % 4 != 0) return QWC_INVALID_ARGUMENT;                 // exports.zig:450-451
  uint32_t steps = 0;
  QWC_TRY(run_audio(h, features, features_len / 4, &steps));
  return stream_begin(h, slot, prompt, prompt_len, h->audio_out.as<float>(), steps, max_tokens, true);
}

int32_t qwc_decode_begin_features(uint32_t handle, const uint32_t* prompt, uint32_t prompt_len, const float* features,
                                  uint64_t features_len, uint32_t max_tokens) {
  Handle* h = lookup(handle);
  if (!h) return QWC_INVALID_ARGUMENT;
  if (h->streams > 1) return QWC_UNSUPPORTED;
  return qwc_stream_begin_features(handle, 0, prompt, prompt_len, features, features_len, max_tokens);
}

int32_t qwc_debug_audio(uint32_t handle, uint32_t which, float* out, uint64_t count) {
  Handle* h = lookup(handle);
  if (!h || !out || which > 1) return QWC_INVALID_ARGUMENT;
  if (!h->audio) return QWC_NOT_FOUND;
  const uint64_t n = std::min<uint64_t>(count, uint64_t(h->audio->g.max_steps) * h->audio->g.d_model);
  const float* src = which == 0 ? h->audio->conv_stage() : h->audio->tower();
  QWC_CUDA(cudaMemcpy(out, src, n * 4, cudaMemcpyDeviceToHost));
  return static_cast<int32_t>(n);
}

int32_t qwc_audio_run_timed(uint32_t handle, const float* log_mel, uint32_t frames, uint32_t reps, float* device_ms,
                            uint32_t* launches_out) {
  Handle* h = lookup(handle);
  if (!h || !log_mel || !device_ms || reps == 0) return QWC_INVALID_ARGUMENT;
  if (h->state != State::kLoaded) return QWC_INVALID_STATE;
  if (!h->audio) return QWC_NOT_FOUND;
  if (frames == 0) return QWC_SHAPE_MISMATCH;
  if (frames > h->audio->g.max_frames) return QWC_AUDIO_TOO_LONG;
  cudaSetDevice(h->device);
  float* mel = h->audio->mel_buffer();
  QWC_CUDA(cudaMemcpyAsync(mel, log_mel, uint64_t(frames) * h->audio->g.mel_bins * 4, cudaMemcpyHostToDevice,
                           h->stream));
  cudaEvent_t e0, e1;
  QWC_CUDA(cudaEventCreate(&e0));
  QWC_CUDA(cudaEventCreate(&e1));
  int32_t st = QWC_OK;
  uint32_t steps = 0;
  cudaEventRecord(e0, h->stream);
  for (uint32_t r = 0; r < reps && st == QWC_OK; ++r) {
    st = h->audio->run(mel, frames, h->audio_out.as<float>(), h->stream, audio_wait_ns(h), &steps, false);
    h->launches += h->audio->launches();
  }
  cudaEventRecord(e1, h->stream);
  if (st == QWC_OK) st = h->audio->check_error(h->stream);
  cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *device_ms = ms;
  if (launches_out) *launches_out = static_cast<uint32_t>(h->audio->launches());
  return st;
}

uint64_t qwc_kernel_launches(uint32_t handle) {
  Handle* h = lookup(handle);
  return h ? h->launches : 0;
}

int32_t qwc_rope_tables(float theta, uint32_t head_dim, uint32_t max_positions, float* cos_out, float* sin_out) {
  if (!cos_out || !sin_out || head_dim == 0 || head_dim % 2 != 0) return QWC_INVALID_ARGUMENT;
  build_rope(theta, head_dim, max_positions, cos_out, sin_out);
  return QWC_OK;
}

}  // extern "C"

// qwc_internal.h -- structures shared by the host runtime (qwc_api.cpp) and
// the device code (qwc_decode.cu, qwc_ops.cu). Plain C++ so both nvcc and the
// host compiler read it.
#pragma once

#include <cstddef>
#include <cstdint>

namespace qwc {

constexpr uint32_t kGroup = 64;           // src/core/quant.zig:49
constexpr uint32_t kFormatF32 = 0;
constexpr uint32_t kFormatQ4 = 16;
constexpr uint32_t kFormatQ8 = 18;
constexpr uint32_t kMaxLayers = 64;
constexpr uint32_t kPositionLimit = 8192;  // src/core/qwen3_asr/model.zig:62
constexpr uint32_t kAttnChunk = 64;        // positions per split-K attention unit
constexpr uint32_t kHiddenMax = 4096;      // widest hidden vector of the decode kernel
constexpr uint32_t kHeadDim = 128;         // the kernels are written for head_dim 128

inline uint32_t data_bytes_per_group(uint32_t format) {
  return format == kFormatQ4 ? 32u : (format == kFormatQ8 ? 64u : 0u);
}

// One quantized matrix in HBM, in the reference's two-plane layout
// (src/core/quant.zig:8-41, 144-176): `scales` is rows x groups f16 values,
// `codes` rows x groups x data_bytes_per_group bytes; both 16-byte aligned.
struct DevMat {
  const uint8_t* scales;
  const uint8_t* codes;
  uint32_t rows;
  uint32_t cols;
  uint32_t format;
  uint32_t groups;      // cols / 64 per row
  uint32_t scale_row;   // bytes of scales per row (groups * 2)
  uint32_t code_row;    // bytes of codes per row
};

struct DevLayer {
  DevMat q, k, v, o, gate, up, down;
  const float* q_norm;
  const float* k_norm;
  const float* attn_norm;
  const float* ffn_norm;
};

// Static model description (lives in device memory for the decode kernel).
struct DevModel {
  DevLayer layers[kMaxLayers];
  DevMat embed;
  DevMat lm_head;
  const float* final_norm;
  const float* rope_cos;   // [max_positions][head_dim / 2]
  const float* rope_sin;
  uint32_t n_layers;
  uint32_t hidden;
  uint32_t q_heads;
  uint32_t kv_heads;
  uint32_t head_dim;
  uint32_t ffn;
  uint32_t vocab;
  uint32_t max_positions;
  float eps;
  float attn_scaling;      // 1 / sqrt(head_dim) in f32, as kernels.zig:727
  // q8 key/value cache of one stream: per layer [scales plane][codes plane]
  // (src/core/qwen3_asr/decoder.zig:58-65), keys and values in separate buffers.
  uint64_t cache_scales_bytes;  // max_positions * kv_groups * 2
  uint64_t cache_layer_stride;  // scales + codes bytes per layer
  uint64_t cache_stream_stride; // layers * layer stride
};

// One launch of the persistent B=1 decode kernel: `n_tokens` forward passes
// of stream 0, starting at `first_position`.
struct DecodeLaunch {
  const DevModel* model;
  uint8_t* k_cache;
  uint8_t* v_cache;
  uint32_t n_tokens;
  uint32_t first_position;
  // Inputs: token t < n_forced takes forced_token[t], or audio row
  // forced_row[t] when that is >= 0. Later tokens take the argmax of the
  // previous token (the greedy chain, decoder.zig:336-339).
  uint32_t n_forced;
  const uint32_t* forced_token;
  const int32_t* forced_row;
  const float* audio;        // [rows][hidden]
  uint32_t first_input;      // input of token 0 when n_forced == 0
  uint32_t logits_from;      // tokens t >= logits_from compute logits and argmax
  uint32_t* tokens_out;      // [n_tokens]: argmax of each token with logits
  float* logits_out;         // optional [vocab]: logits of the last token with logits
  // scratch (device)
  float* qkv;                // q_width + 2 * kv_width
  float* attn_out;           // q_width
  float* hidden_g;           // hidden
  float* act;                // ffn
  float* attn_part;          // [q_heads][max_chunks][head_dim + 2]
  uint32_t* attn_count;      // [kv_heads]
  float* amax_val;           // [grid]
  uint32_t* amax_idx;        // [grid]
  uint32_t* barrier;         // zeroed before every launch
  int32_t* error;            // nonzero after a bounded wait gave up
  uint64_t timeout_ns;
  uint32_t max_chunks;
  // Optional phase timeline: when non-null, thread 0 of every CTA stores
  // %globaltimer at each phase boundary of token `trace_token` into
  // trace[cta * kTraceEvents + event].
  uint64_t* trace;
  uint32_t trace_token;
};

// TMA descriptors (CUtensorMap, 128 opaque bytes each) of stream 0's q8
// key/value cache, viewed as 3-D u8 tensors [layer][position][bytes]: the
// codes planes (row = kv_width bytes) and the scales planes (row = kv_groups
// * 2 bytes). Built by the host with cuTensorMapEncodeTiled.
struct alignas(64) KvMaps {
  uint8_t k_codes[128];
  uint8_t k_scales[128];
  uint8_t v_codes[128];
  uint8_t v_scales[128];
};

constexpr uint32_t kTraceEvents = 512;
constexpr uint32_t kTraceEventsPerLayer = 11;

}  // namespace qwc

// Launchers implemented in the .cu files (host-callable).
namespace qwc {
int decode_kernel_smem_bytes();
// Returns cudaError_t as int.
int launch_decode(const DecodeLaunch& launch, const KvMaps& maps, int grid, void* stream);
int decode_grid_size(int device);

// cuTensorMapEncodeTiled through the runtime's driver entry point. `strides`
// holds rank - 1 byte strides (dimension 1 up); `swizzle128` selects the
// 128-byte swizzle. Returns a QWC_* status.
enum MapType : int { kMapU8 = 0, kMapF16 = 1 };
int32_t encode_tensor_map(uint8_t* out128, int type, uint32_t rank, void* base, const uint64_t* dims,
                          const uint64_t* strides, const uint32_t* box, bool swizzle128);
int gemm_smem_bytes();
}  // namespace qwc

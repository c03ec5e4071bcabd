// qwc_internal.h -- structures shared by the host runtime (qwc_api.cpp) and
// the device code (qwc_decode.cu, qwc_ops.cu). Plain C++ so both nvcc and the
// host compiler read it.
#pragma once

#include <cstddef>
#include <cstdint>

#ifdef __CUDACC__
#define QWC_HOST_DEVICE __host__ __device__
#else
#define QWC_HOST_DEVICE
#endif

namespace qwc {

constexpr uint32_t kGroup = 64;           // src/core/quant.zig:49
constexpr uint32_t kFormatF32 = 0;
constexpr uint32_t kFormatQ4 = 16;
constexpr uint32_t kFormatQ5 = 17;
constexpr uint32_t kFormatQ8 = 18;
constexpr uint32_t kMaxLayers = 64;
constexpr uint32_t kPositionLimit = 8192;  // src/core/qwen3_asr/model.zig:62
constexpr uint32_t kAttnChunk = 64;        // positions per split-K attention unit
constexpr uint32_t kHiddenMax = 4096;      // widest hidden vector of the decode kernel
constexpr uint32_t kHeadDim = 128;         // the kernels are written for head_dim 128
// Floats per attention chunk partial of the decode kernel: o[head_dim], max,
// sum, two pad words (16-byte aligned rows for float4 loads).
constexpr uint32_t kAttnPartStride = kHeadDim + 4;

// Code bytes per 64-value group (quant.zig:47-59): q4 32, q5 40 (32 bytes of
// low nibbles, then an 8-byte plane of fifth bits), q8 64.
QWC_HOST_DEVICE inline uint32_t data_bytes_per_group(uint32_t format) {
  return format == kFormatQ4 ? 32u : format == kFormatQ5 ? 40u : (format == kFormatQ8 ? 64u : 0u);
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
  float* attn_part;          // [q_heads][max_chunks][kAttnPartStride]
  uint32_t* attn_count;      // [kv_heads]
  float* amax_val;           // [grid]
  uint32_t* amax_idx;        // [grid]
  uint32_t* barrier;         // zeroed before every launch
  int32_t* error;            // nonzero after a bounded wait gave up
  uint64_t timeout_ns;
  uint32_t max_chunks;
  // Nonzero: every f32 operation in the reference's order (QWC_OPTION_EXACT):
  // sequential dot-product lanes and sums of squares, whole-history
  // attention per kv head, the host C library's exp. exact_scratch holds the
  // attention scores and value weights, [q_heads][3][max_positions] floats.
  uint32_t exact;
  float* exact_scratch;
  // Failure-path testing (QWC_OPTION_TEST_STALL): added to every grid
  // barrier's target, so with 1 the barriers wait for a CTA that does not
  // exist and end only when their bound runs out.
  uint32_t stall;
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

constexpr uint32_t kBarrierBytes = 1024;   // grid-barrier counters of the decode kernel, zeroed per launch
constexpr uint32_t kTraceEvents = 512;
constexpr uint32_t kTraceEventsPerStage = 3;  // input ready, output done, barrier passed

}  // namespace qwc

// Launchers implemented in the .cu files (host-callable).
namespace qwc {
// Returns cudaError_t as int.
int launch_decode(const DecodeLaunch& launch, const KvMaps& maps, int grid, void* stream);
// The same kernel with three 57 KB ring slots instead of five of 34 KB
// (qwc_decode_wide.cu), for models whose down-projection share per CTA fits
// one wide slot but not one narrow slot.
int launch_decode_wide(const DecodeLaunch& launch, const KvMaps& maps, int grid, void* stream);
constexpr uint32_t kDecodeSlotBytes = 34 * 1024;
constexpr uint32_t kDecodeWideSlotBytes = 453 * 128;
int decode_grid_size(int device);

// ---- batched multi-stream step (qwc_streams.cu) ----

constexpr uint32_t kMaxStreams = 64;  // stream columns of the tensor-core GEMM
// One consumer warp's state at the end of a batched-attention segment:
// max[2], sum[2], o[2][head_dim] of the two query heads of a kv head.
constexpr uint32_t kStreamsPartFloats = 4 + 2 * kHeadDim;

// What one GEMM column does in the next batched step: consume `token`
// (embedding row) or, when `audio_row` >= 0, that row of the stream's audio,
// at `position` of the stream whose cache is slot `cache`. Decode steps use
// one column per stream; a prefill uses up to 64 columns of one stream
// (consecutive positions, causal through the shared cache).
struct SlotStep {
  int32_t active;
  uint32_t position;
  int32_t token;
  int32_t audio_row;
  int32_t cache;
  int32_t pad[3];
};

// Device buffers and shapes shared by the step's kernels. All [slot] arrays
// have kMaxStreams rows; inactive slots are skipped (their rows hold zeros).
struct StreamsStep {
  const DevModel* model;
  const SlotStep* desc;          // [kMaxStreams]
  const float* const* audio;     // [kMaxStreams] per-slot audio rows (device pointers, may be null)
  float* hidden;                 // [slot][hidden]
  void* xb_h;                    // f16 [2 x slot][hidden]: hi rows, then lo rows (GEMM activation layout)
  void* xb_q;                    // f16 [2 x slot][q width]
  void* xb_f;                    // f16 [2 x slot][ffn]
  float* part0;                  // [split][slot][rows] projection partials
  float* qrot;                   // [slot][q width]: normed, rotated queries
  float* attn_part;              // [slot][q head][chunk][head_dim + 4]: o, max, sum of a CTA's segment
  uint32_t* attn_count;          // [slot][kv head]
  uint8_t* k_cache;
  uint8_t* v_cache;
  float* logits;                 // [slot][vocab]
  float* qkv_rows;               // [slot][q width + 2 kv width]: the last layer's pre-norm q/k/v rows of the step
  uint32_t* tokens;              // [slot]
  int32_t* error;
  uint32_t max_chunks;
  uint64_t timeout_ns;
};

// 4-D TMA descriptors over every slot's q8 cache: [slot][layer][position][row bytes].
struct alignas(64) KvMaps4 {
  uint8_t k_codes[128];
  uint8_t k_scales[128];
  uint8_t v_codes[128];
  uint8_t v_scales[128];
};

// One tensor-core GEMM launch over up to three matrices sharing K and the
// activations: out[split][streams][out_ld], matrix j's rows at column
// out_offsets[j]. Maps are 128-byte CUtensorMaps. `streams` columns are
// taken 64 per column block (grid z), block b reading activation rows
// [128 b, 128 b + 128).
int launch_gemm_jobs(const uint8_t (*codes_maps)[128], const uint8_t (*scale_maps)[128], const uint32_t* rows,
                     const uint32_t* formats, const uint32_t* out_offsets, uint32_t njobs, const uint8_t* map_b,
                     uint32_t cols, uint32_t streams, uint32_t splits, float* out, uint32_t out_ld, int32_t* error,
                     void* stream, uint32_t col_blocks = 1, uint64_t timeout_ns = 2000000000ull);
int launch_gemm_streams(const uint8_t* map_codes, const uint8_t* map_scales, const uint8_t* map_b, uint32_t rows,
                        uint32_t cols, uint32_t format, uint32_t splits, float* out, int32_t* error, void* stream);
// TMA descriptors for the stream GEMM: a weight matrix (codes and scales
// planes) and an activation buffer of 128 f16 rows (hi, then lo) x cols.
// `scale_stride`: bytes between scale rows when the plane is padded (a
// multiple of 16); 0 for the container's packed plane (cols / 32 bytes,
// which must then be a multiple of 16).
int32_t gemm_weight_maps(uint32_t format, const void* codes, const void* scales, uint32_t rows, uint32_t cols,
                         uint8_t* codes_map, uint8_t* scales_map, uint32_t scale_stride = 0);
int32_t gemm_act_map(void* base, uint32_t cols, uint8_t* out, uint32_t col_blocks = 1);
// Split count for a GEMM of `rows` x `cols` (times `col_blocks` blocks of 64
// columns) on `sms` SMs.
uint32_t gemm_splits(uint32_t rows, uint32_t cols, int sms, uint32_t col_blocks = 1);
// Dense f16-weight GEMM (the audio convolutions): out[split][columns][rows]
// = W[rows][kpad] X^T over the split's K blocks, X packed like the stream
// GEMM's activations but in natural K order; map_a from
// gemm_dense_weight_map, map_b from gemm_act_map(…, kpad, …, column blocks).
int32_t gemm_dense_weight_map(const void* weights, uint32_t rows, uint32_t kpad, uint8_t* out);
int launch_gemm_dense(const uint8_t* map_a, const uint8_t* map_b, uint32_t rows, uint32_t kpad, uint32_t columns,
                      uint32_t splits, float* out, int32_t* error, uint64_t timeout_ns, void* stream);
int prepare_gemm_dense_kernel();
// Audio tower kernels (qwc_audio.cu); each returns cudaError_t as int.
int launch_audio_conv1(const float* mel, uint32_t frames, uint32_t mel_bins, uint32_t chunk_frames, uint32_t chunks,
                       const void* w, const float* bias, uint32_t channels, float* out, void* stream);
int launch_audio_im2col(const float* in, uint32_t chunks, uint32_t ih, uint32_t iw, uint32_t channels, uint32_t kpad,
                        void* out, void* stream);
int launch_audio_conv_epilogue(const float* parts, uint32_t splits, uint32_t columns, uint32_t channels,
                               const float* bias, float* out, void* stream);
int launch_audio_flatten(const float* conv3, uint32_t steps, uint32_t chunk_steps, uint32_t bins, uint32_t channels,
                         void* out, void* stream);
// mode: 0 position, 1 bias, 2 residual, 3 GELU into GEMM activation rows.
int launch_audio_epilogue(int mode, const float* parts, uint32_t splits, uint32_t steps, uint32_t ld, uint32_t width,
                          const float* add, uint32_t chunk_steps, float* x, uint32_t x_ld, void* packed, void* stream);
// LayerNorm of each of `steps` rows of x, after x += sum of `splits`
// partials [split][steps][width] + rbias when `parts` is given.
int launch_audio_layernorm(float* x, const float* parts, uint32_t splits, const float* rbias, const float* weight,
                           const float* bias, uint32_t width, float eps, uint32_t steps, float* out, void* packed,
                           void* stream);
// Windowed attention over the Q|K|V GEMM's partials [split][steps][3 width]
// plus the q|k|v biases, into the O GEMM's activation rows.
int launch_audio_attention(const float* parts, uint32_t splits, const float* qkv_bias, uint32_t steps,
                           uint32_t width, uint32_t heads, uint32_t head_dim, uint32_t window, void* packed,
                           void* stream);
size_t audio_attention_smem(uint32_t window, uint32_t head_dim);
int prepare_audio_kernels(uint32_t window, uint32_t head_dim);
// x[columns][cols] f32 -> the GEMM's activation rows (f16 hi and lo, 128 rows
// per 64-column block, K chunks in the weight order) at `out`.
int launch_pack_activations(const float* x, uint32_t columns, uint32_t cols, void* out, void* stream);
// Step kernels; each returns cudaError_t as int.
int launch_streams_norm(const StreamsStep& P, int input_mode, const float* weight, const float* parts,
                        uint32_t splits, void* stream);
int launch_streams_qkv(const StreamsStep& P, uint32_t layer, uint32_t splits, uint32_t kv_heads, void* stream);
int launch_streams_attention(const StreamsStep& P, const KvMaps4& maps, uint32_t layer, int grid, void* stream);
int launch_streams_swiglu(const StreamsStep& P, uint32_t splits, void* stream);
int launch_streams_argmax(const StreamsStep& P, void* stream);
int launch_streams_advance(const StreamsStep& P, uint32_t* history, uint32_t* counter, uint32_t rows, void* stream);
// Kernel attributes (dynamic shared memory) set once, outside stream capture.
int prepare_stream_kernels();
int prepare_gemm_kernel();

// cuTensorMapEncodeTiled through the runtime's driver entry point. `strides`
// holds rank - 1 byte strides (dimension 1 up); `swizzle128` selects the
// 128-byte swizzle. Returns a QWC_* status.
enum MapType : int { kMapU8 = 0, kMapF16 = 1 };
int32_t encode_tensor_map(uint8_t* out128, int type, uint32_t rank, void* base, const uint64_t* dims,
                          const uint64_t* strides, const uint32_t* box, bool swizzle128);
int gemm_smem_bytes();
}  // namespace qwc

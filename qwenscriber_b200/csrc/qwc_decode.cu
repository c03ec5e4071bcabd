// qwc_decode.cu -- the persistent sm_100a decode kernel for one stream.
//
// One launch runs `n_tokens` forward passes of Decoder.forwardToken
// (src/core/qwen3_asr/decoder.zig:133-287) followed, where logits are wanted,
// by the argmax (decoder.zig:290-301). One CTA per SM, co-resident
// (cooperative launch):
//
//   * the producer warp streams this CTA's fixed share of every weight matrix
//     -- whole rows, in the reference's two-plane q4/q8 layout -- from HBM into
//     a ring of shared-memory slots with cp.async.bulk, tracked by mbarriers.
//     Weights never depend on activations, so it runs ahead across phase
//     boundaries, layers and tokens while the consumers wait at barriers.
//   * eight consumer warps dequantize in registers and reduce with warp
//     shuffles (the dot products of kernels.zig:118-158); the activation
//     vector sits in shared memory, read once per 16-byte code chunk and
//     shared by the four rows a warp works on at a time. The lm_head (the
//     one stage with many tiles per CTA) runs on the integer tensor cores
//     instead: exact integer group sums of the codes against byte limbs of
//     the activations (gemv_tiles_mma). Fused epilogues:
//     QK-RMSNorm + RoPE + q8 KV append inside the attention phase, residual
//     adds, SwiGLU, and the argmax.
//
// Phases per layer, separated by grid barriers: QKV -> attention (split-K
// flash decode over the q8 cache, last-arriver combine) -> O + residual ->
// RMSNorm + gate/up + SwiGLU -> down + residual. Every CTA recomputes the
// RMSNorm of the full hidden vector redundantly instead of taking another
// barrier. Every wait is bounded by `timeout_ns`; on expiry the kernel
// records an error, drains its in-flight copies and returns.

#include <cuda_runtime.h>

#include <cstddef>

#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kRowsPerPass = 4;                // rows one warp works on at a time
// The weight ring: five slots of 34 KB (32 rows of a q4 matrix with K = 2048),
// or, in the copy of this kernel that qwc_decode_wide.cu compiles, three of
// 57 KB, for models whose down-projection share fits one wide slot but not one
// narrow slot (one tile instead of two per CTA). The host picks the copy per
// model (launch_decode / launch_decode_wide).
#ifndef QWC_DECODE_WIDE_SLOTS
#define QWC_DECODE_WIDE_SLOTS 0
#endif
constexpr int kSlots = QWC_DECODE_WIDE_SLOTS ? 3 : 5;
constexpr uint32_t kSlotBytes = QWC_DECODE_WIDE_SLOTS ? kDecodeWideSlotBytes : kDecodeSlotBytes;
constexpr uint32_t kXMax = 8192;               // floats in the activation buffer (max K)
constexpr uint32_t kRowsMax = 256;             // rows of one stage per CTA (non-LM stages)
constexpr uint32_t kResidMax = 256;            // hidden rows owned by one CTA
static_assert(kConsumerThreads == 2 * kHeadDim, "attention maps (query head, dimension) onto the consumer threads");
static_assert(kConsumerWarps == 8, "attention splits a chunk into eight warps of positions");

// Attention tile: one ring slot per (kv head, position chunk) unit.
constexpr uint32_t kTileKCodes = 0;                                     // [kAttnChunk][kHeadDim] key codes
constexpr uint32_t kTileVCodes = kTileKCodes + kAttnChunk * kHeadDim;   // [kAttnChunk][kHeadDim] value codes
constexpr uint32_t kTileKScales = kTileVCodes + kAttnChunk * kHeadDim;  // [kAttnChunk][16 B]: scales of 4 kv heads
constexpr uint32_t kTileVScales = kTileKScales + kAttnChunk * 16;
constexpr uint32_t kTileQNorm = kTileVScales + kAttnChunk * 16;         // [kHeadDim] f32
constexpr uint32_t kTileKNorm = kTileQNorm + kHeadDim * 4;
constexpr uint32_t kTileCos = kTileKNorm + kHeadDim * 4;                // [kHeadDim / 2] f32 for this position
constexpr uint32_t kTileSin = kTileCos + kHeadDim * 2;
constexpr uint32_t kAttnTileBytes = kTileSin + kHeadDim * 2;
static_assert(kTileVCodes % 128 == 0 && kTileKScales % 128 == 0 && kTileVScales % 128 == 0 && kTileQNorm % 16 == 0 &&
                  kTileCos % 16 == 0 && kTileSin % 16 == 0,
              "TMA boxes land on 128-byte boundaries, bulk copies on 16-byte boundaries");

enum Stage : int { kStQKV = 0, kStO = 1, kStGateUp = 2, kStDown = 4, kStLM = 5, kStAttn = 6 };

// A token is a walk over stages: five per layer in this order, then the
// lm_head stage for tokens with logits. The producer and the consumers run
// the same walk, each with one code path per kind of stage, so the code a
// layer executes stays small enough to remain in the instruction cache.
constexpr int kStagesPerLayer = 5;
__device__ __forceinline__ int layer_stage(uint32_t i) {
  // QKV, attention, O, gate and up, down (decoder.zig:165-271).
  return i == 0 ? kStQKV : i == 1 ? kStAttn : i == 2 ? kStO : i == 3 ? kStGateUp : kStDown;
}

enum ErrorCode : int32_t { kErrBarrier = 1, kErrFull = 2, kErrEmpty = 3, kErrShape = 4 };

struct Smem {
  uint8_t ring[kSlots][kSlotBytes];
  uint64_t full[kSlots];
  uint64_t empty[kSlots];
  float x[kXMax];                 // activation vector, swizzled (x_index), q4-prescaled when asked
  float part[kRowsMax];           // per-row dot products of the current stage
  float chunk_part[kSlotBytes / 512];  // per (row, 512-byte chunk) dot products of the current tile
  float resid[kResidMax];         // this CTA's rows of the residual stream
  float red[kConsumerWarps * 2];  // block reductions
  float amax_v[kConsumerWarps];
  uint32_t amax_i[kConsumerWarps];
  uint32_t flag;
  uint32_t abort;  // set by any consumer thread whose bounded wait gave up
  // The model description, copied from device memory at launch: every stage
  // reads matrix shapes and pointers from it, and shared-memory loads keep
  // those reads off the stage's critical path.
  alignas(16) uint8_t model[sizeof(DevModel)];
};

// Attention scratch overlays the activation buffer (never live together).
// Members read or written with 128-bit accesses are 16-byte aligned.
struct AttnSmem {
  alignas(16) float q[2][4][36];  // rotated query heads, 32-dimension quarters padded against bank conflicts
  alignas(16) float tmp[2][kHeadDim];
  alignas(16) float ktmp[kHeadDim];
  alignas(16) float prob[2][kAttnChunk];
  alignas(16) float lsum[2][8];
  alignas(16) float mx[2];
  alignas(16) float vpart[8][2][kHeadDim];
  alignas(16) uint32_t new_codes[2][kHeadDim / 4];  // the appended key (0) / value (1) row, packed q8 codes
  alignas(16) uint32_t new_scales[2][2];            // f16 scale bits of its two groups
};
static_assert(offsetof(AttnSmem, q) % 16 == 0 && offsetof(AttnSmem, vpart) % 16 == 0 &&
                  offsetof(AttnSmem, new_codes) % 16 == 0 && (sizeof(float) * 36) % 16 == 0,
              "vector accesses in the attention scratch need 16-byte alignment");
static_assert(offsetof(Smem, x) % 16 == 0 && offsetof(Smem, ring) % 128 == 0 && kSlotBytes % 128 == 0,
              "activation buffer and TMA destinations alignment");
static_assert(sizeof(AttnSmem) <= sizeof(float) * kXMax, "attention scratch must fit the activation buffer");
static_assert(sizeof(Smem) <= 227 * 1024, "one CTA per SM: the shared memory fits the 227 KB opt-in limit");
static_assert(kAttnTileBytes <= kSlotBytes, "an attention tile fills one ring slot");
static_assert(kHiddenMax * 4 <= kSlotBytes, "a norm weight vector fills one ring slot");

// Float4-granular XOR swizzle so a lane's 32 (or 16) consecutive activations
// load conflict-free with 128-bit shared loads.
__device__ __forceinline__ uint32_t x_index(uint32_t k) {
  const uint32_t q = k >> 2;
  return ((q ^ ((q >> 3) & 7u)) << 2) | (k & 3u);
}

struct Span {
  uint32_t begin, end;
};

__device__ __forceinline__ Span split_rows(uint32_t rows, uint32_t c, uint32_t n) {
  return {static_cast<uint32_t>((uint64_t(rows) * c) / n), static_cast<uint32_t>((uint64_t(rows) * (c + 1)) / n)};
}

// One matrix's rows within a CTA's share of a stage. The plane pointers and
// row pitches are copied out of the model description so the streaming loops
// keep them in registers.
struct Piece {
  const uint8_t* scales;  // first row's scales
  const uint8_t* codes;   // first row's codes
  uint32_t scale_row;     // bytes of scales per row
  uint32_t code_row;      // bytes of codes per row
  uint32_t rows;          // rows in this piece
  uint32_t local0;        // index of the first row within the CTA's share of the stage
  uint32_t out0;          // index of the first row in the stage's output vector
};

// The CTA's share of a stage: identical for the producer and the consumers.
__device__ int stage_pieces(const DevModel& m, uint32_t layer, int stage, uint32_t c, uint32_t n, Piece* out) {
  const DevLayer& L = m.layers[layer];
  int count = 0;
  auto add = [&](const DevMat* mat, uint32_t r0, uint32_t r1, uint32_t local0, uint32_t out0) {
    if (r1 > r0) {
      const uint32_t sr = mat->scale_row, cr = mat->code_row;
      out[count++] = Piece{mat->scales + size_t(r0) * sr, mat->codes + size_t(r0) * cr, sr, cr, r1 - r0, local0, out0};
    }
  };
  switch (stage) {
    case kStQKV: {
      const uint32_t qr = L.q.rows, kr = L.k.rows, vr = L.v.rows;
      const Span s = split_rows(qr + kr + vr, c, n);
      const uint32_t b = s.begin, e = s.end;
      // [0, qr) q rows, [qr, qr + kr) k rows, then v rows.
      add(&L.q, min(b, qr), min(e, qr), 0, min(b, qr));
      add(&L.k, min(max(b, qr), qr + kr) - qr, min(max(e, qr), qr + kr) - qr, min(max(b, qr), qr + kr) - b,
          min(max(b, qr), qr + kr));
      add(&L.v, max(b, qr + kr) - (qr + kr), max(e, qr + kr) - (qr + kr), max(b, qr + kr) - b, max(b, qr + kr));
      break;
    }
    case kStO: {
      const Span s = split_rows(L.o.rows, c, n);
      add(&L.o, s.begin, s.end, 0, s.begin);
      break;
    }
    case kStGateUp: {
      // This CTA's gate rows, then the same rows of up: one stage, so its
      // tiles run across the two matrices.
      const Span s = split_rows(L.gate.rows, c, n);
      add(&L.gate, s.begin, s.end, 0, s.begin);
      add(&L.up, s.begin, s.end, s.end - s.begin, s.begin);
      break;
    }
    case kStDown: {
      const Span s = split_rows(L.down.rows, c, n);
      add(&L.down, s.begin, s.end, 0, s.begin);
      break;
    }
    default: {
      const Span s = split_rows(m.lm_head.rows, c, n);
      add(&m.lm_head, s.begin, s.end, 0, s.begin);
      break;
    }
  }
  return count;
}

// Rows per ring slot; an integer-GEMV tile (`regions`) leaves 64 bytes for
// the gap between its two code regions (Producer::issue).
__device__ __forceinline__ uint32_t rows_per_tile(const Piece& p, bool regions = false) {
  return (kSlotBytes - (regions ? 64u : 0u)) / (p.scale_row + p.code_row);
}

__device__ __forceinline__ uint32_t stage_format(const DevModel& m, uint32_t layer, int stage) {
  const DevLayer& L = m.layers[layer];
  return stage == kStLM ? m.lm_head.format
       : stage == kStQKV ? L.q.format
       : stage == kStO ? L.o.format
       : stage == kStGateUp ? L.gate.format
                        : L.down.format;
}

// Length of the stage's input vector (the GEMV's K).
__device__ __forceinline__ uint32_t stage_width(const DevModel& m, int stage) {
  return stage == kStO ? m.q_heads * kHeadDim : stage == kStDown ? m.ffn : m.hidden;
}

// Stages the integer tensor-core GEMV takes (gemv_tiles_mma): the lm_head,
// for q4 and q8 matrices whose K is a multiple of 256 and fits its side
// arrays. (The layer stages have one to three tiles per CTA, too few to give
// whole 16-row blocks to every warp; split over the warps, with a block
// barrier and a reduction per stage plus the conversion of their inputs,
// they measured slower than the CUDA-core GEMV.)
constexpr uint32_t kMmaKMax = 6144;
__device__ __forceinline__ bool mma_gemv(int stage, uint32_t format, uint32_t width) {
  return stage == kStLM && (format == kFormatQ4 || format == kFormatQ8) && width % 256 == 0 && width <= kMmaKMax;
}

// ---------------------------------------------------------------------------
// Producer
// ---------------------------------------------------------------------------

struct Producer {
  Smem* s;
  uint32_t it = 0;
  int32_t* error;
  uint64_t timeout_ns;
  bool ok = true;

  // Waits for the next free slot, arms its full barrier for `bytes` and
  // returns it (nullptr after an error).
  __device__ uint8_t* begin_tile(uint32_t bytes, uint64_t** bar) {
    const uint32_t slot = it % kSlots;
    const uint32_t parity = ((it / kSlots) & 1u) ^ 1u;
    if (!mbar_wait_bounded(&s->empty[slot], parity, error, timeout_ns, kErrEmpty)) {
      ok = false;
      return nullptr;
    }
    mbar_arrive_expect_tx(&s->full[slot], bytes);
    *bar = &s->full[slot];
    ++it;
    return s->ring[slot];
  }

  // `nr` whole rows of one matrix: their scales, then their codes. For the
  // integer GEMV (`regions`) the codes go in two regions, the first
  // (nr + 1) / 2 rows and the rest, the second starting 64 bytes further on
  // (mod 128) so that rows of the two regions fall in different banks.
  __device__ void issue(const Piece& pc, uint32_t r0, uint32_t nr, bool regions) {
    const uint32_t bytes_s = nr * pc.scale_row;
    const uint32_t bytes_c = nr * pc.code_row;
    uint64_t* bar;
    uint8_t* dst = begin_tile(bytes_s + bytes_c, &bar);
    if (!dst) return;
    bulk_g2s(dst, pc.scales + size_t(r0) * pc.scale_row, bytes_s, bar);
    const uint8_t* src = pc.codes + size_t(r0) * pc.code_row;
    if (!regions || nr < 2) {
      bulk_g2s(dst + bytes_s, src, bytes_c, bar);
      return;
    }
    const uint32_t ha = (nr + 1) / 2;
    bulk_g2s(dst + bytes_s, src, ha * pc.code_row, bar);
    bulk_g2s(dst + bytes_s + ha * pc.code_row + 64, src + size_t(ha) * pc.code_row, (nr - ha) * pc.code_row, bar);
  }

  // A norm weight vector of n floats.
  __device__ void vector_tile(const float* v, uint32_t n) {
    uint64_t* bar;
    uint8_t* dst = begin_tile(n * 4, &bar);
    if (!dst) return;
    bulk_g2s(dst, v, n * 4, bar);
  }

  // This CTA's attention units at `position` (the same walk as attention_stage).
  __device__ void attention_tiles(const DevModel& m, const KvMaps& maps, uint32_t layer, uint32_t position) {
    const uint32_t cached = (position + kAttnChunk - 1) / kAttnChunk;  // chunks of cached positions
    const uint32_t slots = cached + 1;                                 // + the new row's unit
    const uint32_t units = m.kv_heads * slots;
    const DevLayer& L = m.layers[layer];
    const float* cos_row = m.rope_cos + size_t(position) * (kHeadDim / 2);
    const float* sin_row = m.rope_sin + size_t(position) * (kHeadDim / 2);
    for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const uint32_t h = u / slots;
      const uint32_t ch = u % slots;
      uint64_t* bar;
      if (ch == cached) {
        // The new row's unit: the norm weights and the RoPE row only.
        uint8_t* dst = begin_tile(kHeadDim * 4 * 2 + kHeadDim * 2 * 2, &bar);
        if (!dst) return;
        bulk_g2s(dst + kTileQNorm, L.q_norm, kHeadDim * 4, bar);
        bulk_g2s(dst + kTileKNorm, L.k_norm, kHeadDim * 4, bar);
        bulk_g2s(dst + kTileCos, cos_row, kHeadDim * 2, bar);
        bulk_g2s(dst + kTileSin, sin_row, kHeadDim * 2, bar);
        continue;
      }
      uint8_t* dst = begin_tile(kAttnTileBytes, &bar);
      if (!dst) return;
      // The cache rows were written with ordinary stores by earlier tokens;
      // order them before this async-proxy read.
      fence_proxy_async_global();
      const int32_t y = static_cast<int32_t>(ch * kAttnChunk);
      const int32_t z = static_cast<int32_t>(layer);
      const int32_t xs = static_cast<int32_t>((h * 4u) & ~15u);  // 16-byte box holding kv head h's two f16 scales
      tma_load_3d(dst + kTileKCodes, maps.k_codes, static_cast<int32_t>(h * kHeadDim), y, z, bar);
      tma_load_3d(dst + kTileVCodes, maps.v_codes, static_cast<int32_t>(h * kHeadDim), y, z, bar);
      tma_load_3d(dst + kTileKScales, maps.k_scales, xs, y, z, bar);
      tma_load_3d(dst + kTileVScales, maps.v_scales, xs, y, z, bar);
      bulk_g2s(dst + kTileQNorm, L.q_norm, kHeadDim * 4, bar);
      bulk_g2s(dst + kTileKNorm, L.k_norm, kHeadDim * 4, bar);
      bulk_g2s(dst + kTileCos, cos_row, kHeadDim * 2, bar);
      bulk_g2s(dst + kTileSin, sin_row, kHeadDim * 2, bar);
    }
  }

  // Rows t0 .. t0 + nr of the stage's pieces taken end to end (one K and one
  // format per stage), as one tile: each piece's segment in two bulk copies,
  // its scales and its codes, at the segment's place in the tile.
  __device__ void issue_span(const Piece* pieces, int np, uint32_t t0, uint32_t nr) {
    const uint32_t sr = pieces[0].scale_row, cr = pieces[0].code_row;
    uint64_t* bar;
    uint8_t* dst = begin_tile(nr * (sr + cr), &bar);
    if (!dst) return;
    uint32_t first = 0;  // stage row of the piece's first row
    for (int p = 0; p < np; ++p) {
      const uint32_t b = max(t0, first), e = min(t0 + nr, first + pieces[p].rows);
      if (b < e) {
        const uint32_t r = b - first, k = b - t0, n = e - b;
        bulk_g2s(dst + k * sr, pieces[p].scales + size_t(r) * sr, n * sr, bar);
        bulk_g2s(dst + nr * sr + k * cr, pieces[p].codes + size_t(r) * cr, n * cr, bar);
      }
      first += pieces[p].rows;
    }
  }

  __device__ void stage(const DevModel& m, uint32_t layer, int st, bool regions) {
    Piece pieces[3];
    const int np = stage_pieces(m, layer, st, blockIdx.x, gridDim.x, pieces);
    if (np == 0) return;
    if (regions) {  // the integer lm_head: one piece
      const uint32_t per = rows_per_tile(pieces[0], true);
      for (uint32_t r = 0; r < pieces[0].rows && ok; r += per) issue(pieces[0], r, min(per, pieces[0].rows - r), true);
      return;
    }
    uint32_t total = 0;
    for (int p = 0; p < np; ++p) total += pieces[p].rows;
    const uint32_t per = rows_per_tile(pieces[0]);
    for (uint32_t t0 = 0; t0 < total && ok; t0 += per) issue_span(pieces, np, t0, min(per, total - t0));
  }

  // After an error: wait (bounded) for every copy still in flight so no bulk
  // write lands in shared memory after the CTA exits.
  __device__ void drain() {
    const uint64_t deadline = global_timer_ns() + 1000000000ull;
    for (uint32_t slot = 0; slot < kSlots; ++slot) {
      if (it <= slot) continue;
      const uint32_t last = it - 1 - ((it - 1 - slot) % kSlots);
      const uint32_t parity = (last / kSlots) & 1u;
      while (!mbar_try_wait(&s->full[slot], parity)) {
        if (global_timer_ns() > deadline) break;
      }
    }
  }
};

// The producer's stream, in the consumers' order: per layer the attention
// norm, QKV rows, attention tiles, O rows, the FFN norm, gate, up and down
// rows; then, for tokens with logits, the final norm and the lm_head rows.
__device__ void run_producer(const DecodeLaunch& P, const KvMaps& maps, Smem* s) {
  if ((threadIdx.x & 31) != 0) return;
  const DevModel& m = *reinterpret_cast<const DevModel*>(s->model);
  Producer pr{s, 0, P.error, P.timeout_ns, true};
  for (uint32_t t = 0; t < P.n_tokens && pr.ok; ++t) {
    const uint32_t position = P.first_position + t;
    const uint32_t walk = m.n_layers * kStagesPerLayer + (t >= P.logits_from ? 1u : 0u);
    for (uint32_t q = 0; q < walk && pr.ok; ++q) {
      const uint32_t l = q / kStagesPerLayer;
      const int st = l < m.n_layers ? layer_stage(q % kStagesPerLayer) : kStLM;
      if (st == kStQKV || st == kStGateUp || st == kStLM) {
        const float* norm = st == kStQKV ? m.layers[l].attn_norm : st == kStGateUp ? m.layers[l].ffn_norm : m.final_norm;
        pr.vector_tile(norm, m.hidden);
      }
      if (!pr.ok) break;
      if (st == kStAttn) {
        if (!P.exact) pr.attention_tiles(m, maps, l, position);  // exact mode reads the cache with plain loads
      } else {
        const uint32_t lq = st == kStLM ? 0 : l;
        pr.stage(m, lq, st, st == kStLM && !P.exact && mma_gemv(st, stage_format(m, lq, st), stage_width(m, st)));
      }
    }
  }
  if (!pr.ok) pr.drain();
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------

struct Ctx {
  const DecodeLaunch* P;
  const DevModel* m;
  Smem* s;
  uint32_t it;        // tile counter, in step with the producer
  uint32_t barriers;  // grid barriers passed
  bool ok;
  int warp, lane, tid;
  bool tracing;           // this token's phase timeline is being recorded
  uint64_t full_wait_ns;  // thread 0: time spent waiting for streamed tiles
  uint64_t bar_wait_ns;   // thread 0: time between barrier arrival and release
  uint64_t tile_ns;       // thread 0: time from a tile's arrival to its release
  uint64_t tile_t0;
};

__device__ bool error_set(const int32_t* e) { return *reinterpret_cast<const volatile int32_t*>(e) != 0; }

// Phase timeline (DecodeLaunch::trace): event e of the traced token.
__device__ __forceinline__ void trace_mark(const Ctx& c, uint32_t e) {
  if (c.tracing && c.tid == 0 && e < kTraceEvents - 3) c.P->trace[blockIdx.x * kTraceEvents + e] = global_timer_ns();
}

// Waits (bounded) for the next streamed tile and returns its slot. Every
// consumer warp acquires and releases every tile, in stream order.
__device__ const uint8_t* acquire_tile(Ctx& c) {
  const uint32_t slot = c.it % kSlots;
  const uint32_t parity = (c.it / kSlots) & 1u;
  const uint64_t w0 = (c.tracing && c.tid == 0) ? global_timer_ns() : 0;
  if (c.ok && !mbar_wait_bounded(&c.s->full[slot], parity, c.P->error, c.P->timeout_ns, kErrFull)) {
    c.ok = false;
  }
  if (c.tracing && c.tid == 0) {
    c.tile_t0 = global_timer_ns();
    c.full_wait_ns += c.tile_t0 - w0;
  }
  return c.s->ring[slot];
}

// Hands the current slot back to the producer once this warp is done with it.
__device__ void release_tile(Ctx& c) {
  __syncwarp();
  if (c.tracing && c.tid == 0) c.tile_ns += global_timer_ns() - c.tile_t0;
  if (c.lane == 0) mbar_arrive(&c.s->empty[c.it % kSlots]);
  ++c.it;
}

// Grid-wide barrier among the consumer warps of every CTA. The counter is
// monotonic within a launch (zeroed by the host before it). It is also where
// a CTA decides, for all its consumer threads at once, to stop after a
// bounded wait gave up: a thread whose own wait ran out must not leave the
// stage walk while the others go on to the next block-wide barrier.
__device__ void grid_barrier(Ctx& c) {
  if (!c.ok) c.s->abort = 1u;
  consumer_sync(kConsumerThreads);
  if (c.tid == 0 && c.s->abort) {
    // This CTA stops without arriving; the others see the error word (set by
    // the wait that gave up) or run out their own bounded waits.
    c.s->flag = 1u;
  } else if (c.tid == 0) {
    c.barriers += 1;
    const uint32_t target = c.barriers * gridDim.x + c.P->stall;
    const uint64_t arrive = c.tracing ? global_timer_ns() : 0;
    // The release is cumulative: it publishes every write the CTA's threads
    // made before the bar.sync above.
    red_release_add(c.P->barrier, 1);
    uint64_t deadline = 0;  // set on the first check, so a barrier that opens quickly never reads the clock
    uint32_t spins = 0;
    bool failed = false;
    // The error word is read only while waiting: a barrier that opens costs
    // no extra L2 round trip. An error raised by a CTA that still arrives is
    // seen by the host after the launch, and by the next barrier that waits.
    while (ld_acquire(c.P->barrier) < target) {
      if ((++spins & 63u) == 0) {
        if (error_set(c.P->error)) {
          failed = true;
          break;
        }
        const uint64_t now = global_timer_ns();
        if (deadline == 0) {
          deadline = now + c.P->timeout_ns;
        } else if (now > deadline) {
          atomicCAS(c.P->error, 0, kErrBarrier);
          failed = true;
          break;
        }
      }
    }
    c.s->flag = failed ? 1u : 0u;
    if (c.tracing) c.bar_wait_ns += global_timer_ns() - arrive;
  }
  consumer_sync(kConsumerThreads);
  c.ok = c.s->flag == 0u;
}

// Block-wide sum over the consumer threads.
__device__ float block_sum(Ctx& c, float v) {
  v = warp_sum(v);
  if (c.lane == 0) c.s->red[c.warp] = v;
  consumer_sync(kConsumerThreads);
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) total += c.s->red[w];
  consumer_sync(kConsumerThreads);
  return total;
}

// x holds activations multiplied by 2^74 * 16^-(nibble position) for q4
// stages (q4_chunk_dot_sub, qwc_device.cuh), so the GEMV can mask nibbles
// straight into floats.

constexpr int kMaxPer4 = (kHiddenMax / 4 + kConsumerThreads - 1) / kConsumerThreads;  // float4 groups per thread

// Exact mode keeps x as four lane arrays, the reference dotF32's lanes
// (kernels.zig:39-51): lane array j holds x[j], x[4 + j], x[8 + j], ... at
// s->x[j * xs + i], so the thread that runs lane j of a row reads its
// activations as consecutive float4s. The 16-byte pad between the arrays
// keeps the four lanes' reads in different banks.
__device__ __forceinline__ uint32_t x_lane_stride(uint32_t width) {
  return width / 4 + ((width + 16 <= kXMax) ? 4u : 0u);
}

// x[k .. k + 3] <- v, prescaled for q4 stages; k is a multiple of 4 and
// `width` the length of the vector x holds.
template <bool E>
__device__ __forceinline__ void store_x4(Ctx& c, uint32_t k, float4 v, bool q4, uint32_t width) {
  if constexpr (E) {
    const uint32_t xs = x_lane_stride(width);
    float* x = c.s->x + (k >> 2);
    x[0] = v.x;
    x[xs] = v.y;
    x[2 * xs] = v.z;
    x[3 * xs] = v.w;
    return;
  }
  if (q4) {
    // kQ4SubScale * q4_xscale over k & 7 = 0..3 or 4..7 (powers of two: exact).
    const bool hi = (k & 4u) != 0;
    v.x *= hi ? kQ4SubScale * q4_xscale(4) : kQ4SubScale * q4_xscale(0);
    v.y *= hi ? kQ4SubScale * q4_xscale(5) : kQ4SubScale * q4_xscale(1);
    v.z *= hi ? kQ4SubScale * q4_xscale(6) : kQ4SubScale * q4_xscale(2);
    v.w *= hi ? kQ4SubScale * q4_xscale(7) : kQ4SubScale * q4_xscale(3);
  }
  *reinterpret_cast<float4*>(&c.s->x[x_index(k)]) = v;
}

// x <- rmsnorm(raw) * weight (math.zig:120-130: value * inverse_rms * weight),
// stored prescaled for q4 stages. `raw` holds this thread's float4 groups
// (k = 4 * (tid + i * kConsumerThreads)); the weight vector is the next
// streamed tile.
template <bool E>
__device__ void normalize_into_x(Ctx& c, const float4 (&raw)[kMaxPer4], uint32_t width, bool q4) {
  if constexpr (E) {
    // The raw vector goes to shared memory in index order, and one thread
    // sums its squares in that order (math.zig:123); every CTA does this
    // itself, so no grid-wide exchange is added.
#pragma unroll
    for (int i = 0; i < kMaxPer4; ++i) {
      const uint32_t k4 = c.tid + i * kConsumerThreads;
      if (k4 < width / 4) reinterpret_cast<float4*>(c.s->x)[k4] = raw[i];
    }
    consumer_sync(kConsumerThreads);
    if (c.tid == 0) c.s->red[0] = rms_inverse(sum_squares_seq(c.s->x, width), width, c.m->eps);
    consumer_sync(kConsumerThreads);
    const float inv = c.s->red[0];
    const float4* weight = reinterpret_cast<const float4*>(acquire_tile(c));
#pragma unroll
    for (int i = 0; i < kMaxPer4; ++i) {
      const uint32_t k4 = c.tid + i * kConsumerThreads;
      if (k4 < width / 4) {
        const float4 w = weight[k4];
        store_x4<true>(c, 4 * k4,
                 make_float4(__fmul_rn(__fmul_rn(raw[i].x, inv), w.x), __fmul_rn(__fmul_rn(raw[i].y, inv), w.y),
                             __fmul_rn(__fmul_rn(raw[i].z, inv), w.z), __fmul_rn(__fmul_rn(raw[i].w, inv), w.w)),
                 false, width);
      }
    }
    release_tile(c);
    consumer_sync(kConsumerThreads);
    return;
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kMaxPer4; ++i) {
    if (c.tid + i * kConsumerThreads < width / 4) {
      ss = fmaf(raw[i].x, raw[i].x, ss);
      ss = fmaf(raw[i].y, raw[i].y, ss);
      ss = fmaf(raw[i].z, raw[i].z, ss);
      ss = fmaf(raw[i].w, raw[i].w, ss);
    }
  }
  const float total = block_sum(c, ss);
  const float inv = 1.0f / sqrtf(total / static_cast<float>(width) + c.m->eps);
  const float4* weight = reinterpret_cast<const float4*>(acquire_tile(c));
#pragma unroll
  for (int i = 0; i < kMaxPer4; ++i) {
    const uint32_t k4 = c.tid + i * kConsumerThreads;
    if (k4 < width / 4) {
      const float4 w = weight[k4];
      store_x4<false>(c, 4 * k4,
               make_float4(raw[i].x * inv * w.x, raw[i].y * inv * w.y, raw[i].z * inv * w.z, raw[i].w * inv * w.w),
               q4, width);
    }
  }
  release_tile(c);
  consumer_sync(kConsumerThreads);
}

// x <- rmsnorm(hidden) * weight for a hidden vector other CTAs wrote (L2 loads).
template <bool E>
__device__ void norm_global_into_x(Ctx& c, const float* src, uint32_t width, bool q4) {
  float4 raw[kMaxPer4];
#pragma unroll
  for (int i = 0; i < kMaxPer4; ++i) {
    const uint32_t k4 = c.tid + i * kConsumerThreads;
    raw[i] = k4 < width / 4 ? ld_cg4(reinterpret_cast<const float4*>(src) + k4) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  normalize_into_x<E>(c, raw, width, q4);
}

// Copies a vector other CTAs wrote into x (L2-coherent loads), prescaled for q4.
template <bool E>
__device__ void load_x_global(Ctx& c, const float* src, uint32_t width, bool q4) {
  for (uint32_t k4 = c.tid; k4 < width / 4; k4 += kConsumerThreads) {
    store_x4<E>(c, 4 * k4, ld_cg4(reinterpret_cast<const float4*>(src) + k4), q4, width);
  }
  consumer_sync(kConsumerThreads);
}

// The O projection's input: the attention output of every query head,
// merged from its chunk partials (flash-decode rescale: each chunk's o and
// sum scaled by exp(max_chunk - max_all), then o / sum). A thread owns
// kMergeGroups float4 groups of the output and issues the loads of eight
// chunks for all of them together, one L2 round trip per eight chunks.
constexpr int kMergeGroups = 2;
__device__ void attention_into_x(Ctx& c, const float* parts, uint32_t chunks, bool q4) {
  const uint32_t qw4 = c.m->q_heads * kHeadDim / 4;
  const uint32_t stride = c.P->max_chunks * kAttnPartStride;  // floats per query head
  for (uint32_t g0 = c.tid; g0 < qw4; g0 += kMergeGroups * kConsumerThreads) {
    const float* base[kMergeGroups];
    uint32_t k4[kMergeGroups];
    bool on[kMergeGroups];
    float mx[kMergeGroups], l[kMergeGroups];
    float4 o[kMergeGroups];
#pragma unroll
    for (int g = 0; g < kMergeGroups; ++g) {
      k4[g] = g0 + g * kConsumerThreads;
      on[g] = k4[g] < qw4;
      const uint32_t k = on[g] ? k4[g] * 4 : 0u;
      base[g] = parts + size_t(k / kHeadDim) * stride + k % kHeadDim;
      mx[g] = -INFINITY;
      l[g] = 0.0f;
      o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (uint32_t c0 = 0; c0 < chunks; c0 += 8) {
      float pm[kMergeGroups][8], pl[kMergeGroups][8];
      float4 po[kMergeGroups][8];
#pragma unroll
      for (int g = 0; g < kMergeGroups; ++g) {
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          pm[g][q] = -INFINITY;
          pl[g][q] = 0.0f;
          po[g][q] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (on[g] && c0 + q < chunks) {
            const float* src = base[g] + size_t(c0 + q) * kAttnPartStride;
            const uint32_t d = static_cast<uint32_t>(k4[g] * 4 % kHeadDim);
            pm[g][q] = ld_cg(src - d + kHeadDim);
            pl[g][q] = ld_cg(src - d + kHeadDim + 1);
            po[g][q] = ld_cg4(reinterpret_cast<const float4*>(src));
          }
        }
      }
#pragma unroll
      for (int g = 0; g < kMergeGroups; ++g) {
        float bm = mx[g];
#pragma unroll
        for (int q = 0; q < 8; ++q) bm = fmaxf(bm, pm[g][q]);
        const float rescale = (mx[g] == -INFINITY) ? 0.0f : expf(mx[g] - bm);
        float4 acc = make_float4(o[g].x * rescale, o[g].y * rescale, o[g].z * rescale, o[g].w * rescale);
        float ls = l[g] * rescale;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float f = (pm[g][q] == -INFINITY) ? 0.0f : expf(pm[g][q] - bm);
          acc = make_float4(fmaf(po[g][q].x, f, acc.x), fmaf(po[g][q].y, f, acc.y), fmaf(po[g][q].z, f, acc.z),
                            fmaf(po[g][q].w, f, acc.w));
          ls = fmaf(pl[g][q], f, ls);
        }
        o[g] = acc;
        l[g] = ls;
        mx[g] = bm;
      }
    }
#pragma unroll
    for (int g = 0; g < kMergeGroups; ++g) {
      if (!on[g]) continue;
      const float4 out = make_float4(o[g].x / l[g], o[g].y / l[g], o[g].z / l[g], o[g].w / l[g]);
      // Every CTA merges the same partials in the same order; CTA 0 also
      // keeps the attention output for qwc_debug_scratch.
      if (blockIdx.x == 0) reinterpret_cast<float4*>(c.P->attn_out)[k4[g]] = out;
      store_x4<false>(c, 4 * k4[g], out, q4, 4 * qw4);
    }
  }
  consumer_sync(kConsumerThreads);
}

// Layer-0 input: the token's embedding row (decoder.zig:346-376, quant.zig:348-364)
// or an audio row; this CTA's residual rows keep the raw values, x the normed.
template <bool E>
__device__ void input_into_x(Ctx& c, uint32_t token, int32_t audio_row, Span own, bool q4) {
  const DevModel& m = *c.m;
  const uint32_t hidden = m.hidden;
  float4 raw[kMaxPer4];
  const DevMat& e = m.embed;
  const uint8_t* srow = e.scales + size_t(token) * e.scale_row;
  const uint8_t* crow = e.codes + size_t(token) * e.code_row;
  const float* arow = c.P->audio + size_t(audio_row < 0 ? 0 : audio_row) * hidden;
#pragma unroll
  for (int i = 0; i < kMaxPer4; ++i) {
    const uint32_t k4 = c.tid + i * kConsumerThreads;
    float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (k4 < hidden / 4) {
      const uint32_t k = 4 * k4;
      if (audio_row >= 0) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(arow) + k4);
        v[0] = a.x;
        v[1] = a.y;
        v[2] = a.z;
        v[3] = a.w;
      } else {
        // The four values share one group: code (u - bias) times the group's scale.
        const float scale = f16_bits_to_f32_fast(__ldg(reinterpret_cast<const uint16_t*>(srow) + k / kGroup));
        if (e.format == kFormatQ4) {
          const uint32_t b = __ldg(reinterpret_cast<const uint16_t*>(crow + k / 2));
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = static_cast<float>(static_cast<int>((b >> (4 * t)) & 0xFu) - 8) * scale;
        } else if (e.format == kFormatQ5) {
          const uint8_t* grp = crow + (k / kGroup) * 40u;
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = static_cast<float>(q5_code(grp, (k + t) % kGroup)) * scale;
        } else {
          const uint32_t b = __ldg(reinterpret_cast<const uint32_t*>(crow + k));
#pragma unroll
          for (int t = 0; t < 4; ++t) v[t] = static_cast<float>(static_cast<int>((b >> (8 * t)) & 0xFFu) - 128) * scale;
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        if (k + t >= own.begin && k + t < own.end) c.s->resid[k + t - own.begin] = v[t];
      }
    }
    raw[i] = make_float4(v[0], v[1], v[2], v[3]);
  }
  normalize_into_x<E>(c, raw, hidden, q4);
}

// ---- GEMV over the streamed tiles ----

template <uint32_t FMT>
struct Fmt;
template <>
struct Fmt<kFormatQ4> {
  static constexpr int kPairs = 16;    // packed activation pairs per 16-byte chunk
  static constexpr uint32_t kDB = 32;  // code bytes per group
  static constexpr uint32_t kKPerByte = 2;
};
template <>
struct Fmt<kFormatQ8> {
  static constexpr int kPairs = 8;
  static constexpr uint32_t kDB = 64;
  static constexpr uint32_t kKPerByte = 1;
};
template <>
struct Fmt<kFormatQ5> {  // its chunks are 16 groups (640 bytes); a lane takes half a group
  static constexpr int kPairs = 16;
  static constexpr uint32_t kDB = 40;
  static constexpr uint32_t kKPerByte = 0;
};

// Code bytes a warp covers per chunk step: 32 lanes x 16 bytes, or for q5
// 16 whole groups (a lane's 32 weights: 16 bytes of nibbles + 4 of fifth bits).
template <uint32_t FMT>
__host__ __device__ constexpr uint32_t chunk_bytes() {
  return FMT == kFormatQ5 ? 16u * 40u : 512u;
}

struct Best {
  float v;
  uint32_t i;
};

// The value a logit competes with in the argmax. decoder.zig:290-301 seeds
// the running maximum with values[0] and replaces it only on a strict `>`:
// a NaN at index 0 is never replaced (the answer is 0), and a NaN elsewhere
// never wins. Ranking a NaN logit 0 as +inf (ties go to the lowest index) and
// skipping every other NaN (all comparisons with NaN are false) gives the
// same answer from any order of reduction.
__device__ __forceinline__ float argmax_key(float v, uint32_t index) {
  return (index == 0 && v != v) ? __int_as_float(0x7F800000) : v;
}

// Consumes the stage's tiles. Non-LM stages leave per-row dot products in
// s->part[local]; the LM stage keeps a running argmax per lane and optionally
// stores the logits. A warp pass covers four rows: lane l takes the 16 bytes
// at l * 16 of each 512-byte chunk, the matching activations from x are
// loaded once per chunk for the four rows, and the four dot products reduce
// together (warp_sum4). Rows past the tile repeat the last row so the pass
// has no branches; their sums are dropped.
template <uint32_t FMT>
__device__ void gemv_tiles(Ctx& c, const Piece* pieces, int np, bool lm, Best& best, float* logits_out) {
  for (int p = 0; p < np; ++p) {
    const Piece pc = pieces[p];
    const uint32_t per = rows_per_tile(pc);
    const uint32_t chunks = pc.code_row / chunk_bytes<FMT>();
    // Rows of at most two chunks are taken whole by one pass, and their sums
    // go straight to their rows; longer rows are split into one-chunk passes
    // whose sums are added after the tile.
    const bool whole = chunks <= 2;
    const uint32_t span = whole ? chunks : 1u;  // chunks per pass
    for (uint32_t r = 0; r < pc.rows; r += per) {
      const uint32_t nr = min(per, pc.rows - r);
      const uint32_t quads = (nr + kRowsPerPass - 1) / kRowsPerPass;
      const uint32_t passes = whole ? quads : quads * chunks;
      const uint8_t* base = acquire_tile(c);
      if (c.ok) {
        const uint8_t* codes = base + nr * pc.scale_row;
        for (uint32_t ps = c.warp; ps < passes; ps += kConsumerWarps) {
          const uint32_t r0 = (whole ? ps : ps / chunks) * kRowsPerPass, j0 = whole ? 0u : ps % chunks;
          float acc[kRowsPerPass] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (uint32_t j = j0; j < j0 + span; ++j) {
            if constexpr (FMT == kFormatQ5) {
              // Lane l: half (l & 1) of group 16 j + l / 2. The activations
              // are stored as for q4 (prescaled), so the low nibbles go through
              // q4_chunk_dot_sub; each set fifth bit adds its activation, and
              // sum((u - 16) x) = sum(nib x) + 16 sum(bit x) - 16 sum(x).
              const uint32_t g = 16u * j + (static_cast<uint32_t>(c.lane) >> 1);
              const uint32_t h = static_cast<uint32_t>(c.lane) & 1u;
              uint64_t x2[16];
              float xp[32];  // the activations themselves, for the fifth bits
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(&c.s->x[x_index(64u * g + 32u * h + 4 * q)]);
                x2[2 * q] = pack2(v.x, v.y);
                x2[2 * q + 1] = pack2(v.z, v.w);
                const int p0 = (4 * q) % 8;  // nibble position of v.x
                xp[4 * q] = v.x * q4_unscale(p0);
                xp[4 * q + 1] = v.y * q4_unscale(p0 + 1);
                xp[4 * q + 2] = v.z * q4_unscale(p0 + 2);
                xp[4 * q + 3] = v.w * q4_unscale(p0 + 3);
              }
              const float xbias = 16.0f * q4_chunk_xsum(x2);
#pragma unroll
              for (int q = 0; q < kRowsPerPass; ++q) {
                const uint32_t row = min(r0 + q, nr - 1);
                const uint8_t* grp = codes + row * pc.code_row + 40u * g;
                const uint2 l0 = *reinterpret_cast<const uint2*>(grp + 16u * h);
                const uint2 l1 = *reinterpret_cast<const uint2*>(grp + 16u * h + 8u);
                const uint32_t fifth = *reinterpret_cast<const uint32_t*>(grp + 32u + 4u * h);
                const float scale =
                    f16_bits_to_f32_fast(*reinterpret_cast<const uint16_t*>(base + row * pc.scale_row + g * 2));
                float b0 = 0.0f, b1 = 0.0f;
#pragma unroll
                for (int i = 0; i < 32; i += 2) {
                  if (fifth & (1u << i)) b0 += xp[i];
                  if (fifth & (2u << i)) b1 += xp[i + 1];
                }
                const float nib = q4_chunk_dot_sub(make_uint4(l0.x, l0.y, l1.x, l1.y), x2);
                const float d = fmaf(nib, kQ4SubUnscale, fmaf(16.0f, b0 + b1, -xbias));
                acc[q] = fmaf(d, scale, acc[q]);
              }
              continue;
            }
            const uint32_t off = 16u * c.lane + 512u * j;
            const uint32_t kbase = off * Fmt<FMT>::kKPerByte;
            uint64_t x2[Fmt<FMT>::kPairs];
#pragma unroll
            for (int q = 0; q < Fmt<FMT>::kPairs / 2; ++q) {
              const float4 v = *reinterpret_cast<const float4*>(&c.s->x[x_index(kbase + 4 * q)]);
              x2[2 * q] = pack2(v.x, v.y);
              x2[2 * q + 1] = pack2(v.z, v.w);
            }
            // q4: the chunk's 8 * sum(x), shared by the pass's four rows.
            float xbias = 0.0f;
            if constexpr (FMT == kFormatQ4) xbias = 8.0f * q4_chunk_xsum(x2);
#pragma unroll
            for (int q = 0; q < kRowsPerPass; ++q) {
              const uint32_t row = min(r0 + q, nr - 1);
              const uint4 w = *reinterpret_cast<const uint4*>(codes + row * pc.code_row + off);
              const float scale = f16_bits_to_f32_fast(
                  *reinterpret_cast<const uint16_t*>(base + row * pc.scale_row + (off / Fmt<FMT>::kDB) * 2));
              float d;
              if constexpr (FMT == kFormatQ4) {
                d = fmaf(q4_chunk_dot_sub(w, x2), kQ4SubUnscale, -xbias);  // sum((u - 8) * x)
              } else {
                d = q8_chunk_dot(w, x2);
              }
              acc[q] = fmaf(d, scale, acc[q]);
            }
          }
          const float total = warp_sum4(acc[0], acc[1], acc[2], acc[3]);
          const uint32_t i = r0 + (static_cast<uint32_t>(c.lane) >> 3);
          if ((c.lane & 7) == 0 && i < nr) {
            if (!whole) {
              c.s->chunk_part[i * chunks + j0] = total;
            } else if (!lm) {
              c.s->part[pc.local0 + r + i] = total;
            } else {
              const uint32_t row = pc.out0 + r + i;
              if (logits_out) logits_out[row] = total;
              const float key = argmax_key(total, row);
              if (key > best.v || (key == best.v && row < best.i)) best = Best{key, row};
            }
          }
        }
      }
      release_tile(c);
      if (whole) continue;
      consumer_sync(kConsumerThreads);
      for (uint32_t i = c.tid; i < nr; i += kConsumerThreads) {
        float total = c.s->chunk_part[i * chunks];
        for (uint32_t j = 1; j < chunks; ++j) total += c.s->chunk_part[i * chunks + j];
        if (!lm) {
          c.s->part[pc.local0 + r + i] = total;
        } else {
          const uint32_t row = pc.out0 + r + i;
          if (logits_out) logits_out[row] = total;
          const float key = argmax_key(total, row);
          if (key > best.v || (key == best.v && row < best.i)) best = Best{key, row};
        }
      }
      consumer_sync(kConsumerThreads);  // chunk_part is reused by the next tile
    }
  }
}

// ---- GEMV on the integer tensor cores (default mode, the q4/q8 lm_head) ----
//
// The activation vector becomes integers: per quad of 256 activations,
// x_int = rint(x * 2^e') with |x_int| < 2^30 (e' = e - 4 for q4, below),
// written as four signed byte limbs (x_int = sum_j limb_j * 256^j). A warp
// multiplies 16 weight rows by the limb columns with mma.sync m16n8k32
// (s8 x s8, s32 accumulators), so a group's 64 products and their sum are
// exact integers. The weights enter already centred, in one or two logic
// operations per four codes: a q8 code u as u ^ 0x80 = u - 128; a q4 nibble
// as 16 (u - 8) = (16 u) ^ 0x80, the high nibble masked in place and the low
// one shifted up first (the factor 16 is why q4 activations are taken at
// 2^(e - 4)). The per-group integers are combined two limbs at a time,
// converted to f32 once and scaled by the group's f16 scale; per quad by
// 2^-e.
//
// q4: an MMA covers a pair of groups, the first group's limbs in B columns
// 0-3 and the second's in columns 4-7 (lanes t < 2 load the first group's
// codes, t >= 2 the second's, 16 bytes each, and B is zero where a column and
// a k belong to different groups). q8: an MMA pair covers one group; columns
// 4-7 repeat 0-3.
//
// Shared-memory banks: a tile's codes sit in two regions (Producer::issue)
// 64 bytes apart mod 128, and MMA row m reads region m & 1, so the eight lanes
// of a 16-byte load phase read two rows in different banks.
//
// Limb layout (written over the quad's own 256 floats of x, 256 bytes per
// group): q4 [limb j][half t'][32 bytes: the B registers of the four MMAs of
// that half-group], q8 [limb j][t][16 bytes: k 0-3, 16-19 of the first MMA,
// then the second's]. The side arrays follow the limb planes in x.
constexpr uint32_t kMmaScaleOff = kMmaKMax;  // f32 [kMmaKMax / 256]: 2^-e per quad, floats of x
constexpr uint32_t kMmaZeroOff = 6180;       // 32 zero bytes, 16 mod 128 bytes from x
static_assert(kMmaScaleOff + kMmaKMax / 256 <= kMmaZeroOff && kMmaZeroOff + 8 <= kXMax,
              "the integer GEMV's side arrays fit in x");
static_assert(kMmaScaleOff % 4 == 0 && (kMmaZeroOff * 4) % 128 == 16,
              "16-byte aligned side arrays; the zero block in banks the limb loads leave free");

__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, int c0, int c1, int c2, int c3) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

// out[j] byte i = in[i] byte j.
__device__ __forceinline__ void transpose_bytes(const uint32_t (&in)[4], uint32_t (&out)[4]) {
  const uint32_t a = __byte_perm(in[0], in[1], 0x5140), b = __byte_perm(in[0], in[1], 0x7362);
  const uint32_t c = __byte_perm(in[2], in[3], 0x5140), d = __byte_perm(in[2], in[3], 0x7362);
  out[0] = __byte_perm(a, c, 0x5410);
  out[1] = __byte_perm(a, c, 0x7632);
  out[2] = __byte_perm(b, d, 0x5410);
  out[3] = __byte_perm(b, d, 0x7632);
}

// Four q4 codes of a word as 16 (u - 8) in s8: the high nibbles in place, the
// low ones shifted up (lop3 LUT 0x6A = (a & b) ^ c).
__device__ __forceinline__ uint32_t q4_high16(uint32_t w) {
  uint32_t r;
  asm("lop3.b32 %0, %1, 0xF0F0F0F0, 0x80808080, 0x6A;" : "=r"(r) : "r"(w));
  return r;
}
__device__ __forceinline__ uint32_t q4_low16(uint32_t w) { return q4_high16(w << 4); }

// Writes quad qd's limb planes and scale from this lane's eight activations:
// lane (gi, t, h) holds activations 64 gi + 16 t + 8 h .. + 7 of the quad.
// Warp-collective; the caller orders any reads of the quad's bytes before it.
template <uint32_t FMT>
__device__ __forceinline__ void limbs_store(Ctx& c, uint32_t qd, const float (&xs)[8]) {
  const uint32_t lane = static_cast<uint32_t>(c.lane);
  const uint32_t gi = lane >> 3, t = (lane >> 1) & 3u, h = lane & 1u;
  uint32_t mb = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(xs[i]) & 0x7FFFFFFFu);
  mb = __reduce_max_sync(0xffffffffu, mb);
  // e = 156 - biased exponent of the quad's largest |x|, so |x| * 2^e < 2^30;
  // capped so 2^-e stays a normal float. A non-finite quad yields NaN sums.
  const uint32_t eb = mb >> 23;
  const int e = eb == 255u ? 0 : min(156 - static_cast<int>(eb), 126);
  const float up = __uint_as_float(static_cast<uint32_t>(127 + e) << 23);
  const float sc = FMT == kFormatQ4 ? up * 0.0625f : up;  // q4 codes enter as 16 (u - 8): 2^(e - 4)
  uint32_t lw[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int xi = __float2int_rn(xs[i] * sc);
    // Signed base-256 digits: bytes of xi + 0x808080, the low three re-centred.
    lw[i] = (static_cast<uint32_t>(xi) + 0x00808080u) ^ 0x00808080u;
  }
  uint32_t first[4], second[4];
  if constexpr (FMT == kFormatQ4) {
    const uint32_t lo[4] = {lw[0], lw[2], lw[4], lw[6]}, hi[4] = {lw[1], lw[3], lw[5], lw[7]};
    transpose_bytes(lo, first);
    transpose_bytes(hi, second);
  } else {
    const uint32_t a[4] = {lw[0], lw[1], lw[2], lw[3]}, b[4] = {lw[4], lw[5], lw[6], lw[7]};
    transpose_bytes(a, first);
    transpose_bytes(b, second);
  }
  uint8_t* grp = reinterpret_cast<uint8_t*>(c.s->x) + qd * 1024 + gi * 256;
  if constexpr (FMT == kFormatQ4) {
    // This lane's eight activations are block m = 2 (t & 1) + h of the 32 in
    // half t >> 1: low nibbles in register (m & 1) + 4 (m >> 1) of the half's
    // eight, high nibbles two registers later.
    const uint32_t m = 2 * (t & 1u) + h;
    uint8_t* dst = grp + (t >> 1) * 32 + 4 * ((m & 1u) + 4 * (m >> 1));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *reinterpret_cast<uint32_t*>(dst + 64 * j) = first[j];
      *reinterpret_cast<uint32_t*>(dst + 64 * j + 8) = second[j];
    }
  } else {
    uint8_t* dst = grp + t * 16 + h * 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) *reinterpret_cast<uint2*>(dst + 64 * j) = make_uint2(first[j], second[j]);
  }
  if (lane == 0) {
    c.s->x[kMmaScaleOff + qd] =
        eb == 255u ? __uint_as_float(0x7FC00000u) : __uint_as_float(static_cast<uint32_t>(127 - e) << 23);
  }
}

// The first of the eight activations a lane converts in quad qd.
__device__ __forceinline__ uint32_t limb_k0(const Ctx& c, uint32_t qd) {
  const uint32_t lane = static_cast<uint32_t>(c.lane);
  return qd * 256 + (lane >> 3) * 64 + 16 * ((lane >> 1) & 3u) + 8 * (lane & 1u);
}

// Rewrites x (plain f32, x_index order, `width` values) as limb planes in
// place: a warp takes whole quads and writes a quad once it has read all of it.
// Also writes the zero block q4 lanes read for B columns of the other group
// (f32 inputs of other stages overwrite it).
template <uint32_t FMT>
__device__ void limbs_from_x(Ctx& c, uint32_t width) {
  for (uint32_t qd = static_cast<uint32_t>(c.warp); qd < width / 256; qd += kConsumerWarps) {
    const uint32_t k0 = limb_k0(c, qd);
    const float4 v0 = *reinterpret_cast<const float4*>(&c.s->x[x_index(k0)]);
    const float4 v1 = *reinterpret_cast<const float4*>(&c.s->x[x_index(k0 + 4)]);
    const float xs[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    __syncwarp();  // every lane has read its activations before the quad is overwritten
    limbs_store<FMT>(c, qd, xs);
  }
  if (c.warp == 0 && c.lane < 8) c.s->x[kMmaZeroOff + c.lane] = 0.0f;
  consumer_sync(kConsumerThreads);
}

// Per-lane constants of the integer GEMV.
struct MmaLane {
  const uint8_t* lb;  // B fragments of pair / group 0
  uint32_t lstride;   // bytes per pair (q4) / group (q8)
  uint32_t sh;        // q4: this lane's group within a pair's scale halfwords
};

template <uint32_t FMT>
__device__ __forceinline__ MmaLane mma_lane(const Ctx& c) {
  const uint32_t lane = static_cast<uint32_t>(c.lane);
  const uint32_t g = lane >> 2, t = lane & 3u;
  const uint8_t* xb = reinterpret_cast<const uint8_t*>(c.s->x);
  // q4: lane (g, t) holds B column g; its k belong to group t >> 1 of the
  // pair, so it loads limb g & 3 of that half-group where (t < 2) == (g < 4),
  // else zeros (stride 0 keeps it on the zero block).
  const bool active = FMT == kFormatQ8 || ((t < 2) == (g < 4));
  MmaLane L;
  L.lb = FMT == kFormatQ4 ? (active ? xb + (t >> 1) * 256 + (g & 3u) * 64 + (t & 1u) * 32 : xb + kMmaZeroOff * 4)
                          : xb + (g & 3u) * 64 + t * 16;
  L.lstride = FMT == kFormatQ4 ? (active ? 512u : 0u) : 256u;
  L.sh = 16 * (t >> 1);
  return L;
}

// Dot products of the 16 rows of block b of a tile (MMA row m: row
// 8 b + (m >> 1) of code region m & 1, clamped) over every quad; lane (g, 0)
// returns MMA rows g and g + 8 in out_g, out_8.
template <uint32_t FMT>
__device__ __forceinline__ void block_dot(const Ctx& c, const MmaLane& L, const uint8_t* base, const Piece& pc,
                                          uint32_t nr, uint32_t b, float& out_g, float& out_8) {
  const uint32_t lane = static_cast<uint32_t>(c.lane);
  const uint32_t g = lane >> 2, t = lane & 3u;
  const uint32_t ha = (nr + 1) / 2, hb = nr - ha;
  const uint32_t quads = pc.code_row / (FMT == kFormatQ4 ? 128u : 256u);
  const bool second = (g & 1u) && hb > 0;  // a tile of one row has no second region
  const uint32_t rsize = second ? hb : ha, row0 = second ? ha : 0;
  const uint32_t lg = min(8 * b + (g >> 1), rsize - 1), l8 = min(8 * b + 4 + (g >> 1), rsize - 1);
  const uint8_t* codes = base + nr * pc.scale_row + (second ? ha * pc.code_row + 64 : 0) + 16 * t;
  const uint8_t* cg = codes + lg * pc.code_row;
  const uint8_t* c8 = codes + l8 * pc.code_row;
  const uint8_t* sg = base + (row0 + lg) * pc.scale_row;
  const uint8_t* s8 = base + (row0 + l8) * pc.scale_row;
  const float* qscale = c.s->x + kMmaScaleOff;
  float acc_g = 0.0f, acc_8 = 0.0f;
  for (uint32_t qd = 0; qd < quads; ++qd) {
    const uint2 sgw = *reinterpret_cast<const uint2*>(sg + qd * 8);
    const uint2 s8w = *reinterpret_cast<const uint2*>(s8 + qd * 8);
    float fg = 0.0f, f8 = 0.0f;
    if constexpr (FMT == kFormatQ4) {
#pragma unroll
      for (uint32_t pp = 0; pp < 2; ++pp) {
        const uint32_t pr = 2 * qd + pp;
        const uint4 wg = *reinterpret_cast<const uint4*>(cg + pr * 64);
        const uint4 w8 = *reinterpret_cast<const uint4*>(c8 + pr * 64);
        const uint4 b0 = *reinterpret_cast<const uint4*>(L.lb + pr * L.lstride);
        const uint4 b1 = *reinterpret_cast<const uint4*>(L.lb + pr * L.lstride + 16);
        int d[4];
        mma_s8s8(d, q4_low16(wg.x), q4_low16(w8.x), q4_low16(wg.y), q4_low16(w8.y), b0.x, b0.y, 0, 0, 0, 0);
        mma_s8s8(d, q4_high16(wg.x), q4_high16(w8.x), q4_high16(wg.y), q4_high16(w8.y), b0.z, b0.w, d[0], d[1], d[2],
                 d[3]);
        mma_s8s8(d, q4_low16(wg.z), q4_low16(w8.z), q4_low16(wg.w), q4_low16(w8.w), b1.x, b1.y, d[0], d[1], d[2], d[3]);
        mma_s8s8(d, q4_high16(wg.z), q4_high16(w8.z), q4_high16(wg.w), q4_high16(w8.w), b1.z, b1.w, d[0], d[1], d[2],
                 d[3]);
        // Lane t: group t >> 1 of the pair, limbs 2 (t & 1) and 2 (t & 1) + 1.
        const int eg = d[0] + 256 * d[1], e8 = d[2] + 256 * d[3];
        const uint32_t hg = ((pp ? sgw.y : sgw.x) >> L.sh) & 0xFFFFu;
        const uint32_t h8 = ((pp ? s8w.y : s8w.x) >> L.sh) & 0xFFFFu;
        fg = fmaf(static_cast<float>(eg), __half2float(__ushort_as_half(static_cast<unsigned short>(hg))), fg);
        f8 = fmaf(static_cast<float>(e8), __half2float(__ushort_as_half(static_cast<unsigned short>(h8))), f8);
      }
    } else {
      const uint32_t sgv[4] = {sgw.x & 0xFFFFu, sgw.x >> 16, sgw.y & 0xFFFFu, sgw.y >> 16};
      const uint32_t s8v[4] = {s8w.x & 0xFFFFu, s8w.x >> 16, s8w.y & 0xFFFFu, s8w.y >> 16};
#pragma unroll
      for (uint32_t q = 0; q < 4; ++q) {
        const uint32_t grp = 4 * qd + q;
        const uint4 wg = *reinterpret_cast<const uint4*>(cg + grp * 64);
        const uint4 w8 = *reinterpret_cast<const uint4*>(c8 + grp * 64);
        const uint4 bl = *reinterpret_cast<const uint4*>(L.lb + grp * L.lstride);
        constexpr uint32_t kC = 0x80808080u;  // u - 128 as s8
        int d[4];
        mma_s8s8(d, wg.x ^ kC, w8.x ^ kC, wg.y ^ kC, w8.y ^ kC, bl.x, bl.y, 0, 0, 0, 0);
        mma_s8s8(d, wg.z ^ kC, w8.z ^ kC, wg.w ^ kC, w8.w ^ kC, bl.z, bl.w, d[0], d[1], d[2], d[3]);
        // Lane t holds limbs 2t and 2t + 1 (t < 2; lanes t >= 2 repeat them).
        const int eg = d[0] + 256 * d[1], e8 = d[2] + 256 * d[3];
        fg = fmaf(static_cast<float>(eg), __half2float(__ushort_as_half(static_cast<unsigned short>(sgv[q]))), fg);
        f8 = fmaf(static_cast<float>(e8), __half2float(__ushort_as_half(static_cast<unsigned short>(s8v[q]))), f8);
      }
    }
    const float qs = qscale[qd];
    acc_g = fmaf(fg, qs, acc_g);
    acc_8 = fmaf(f8, qs, acc_8);
  }
  if constexpr (FMT == kFormatQ4) {
    // The pair's two groups (lanes t and t ^ 2) add up.
    acc_g += __shfl_xor_sync(0xffffffffu, acc_g, 2);
    acc_8 += __shfl_xor_sync(0xffffffffu, acc_8, 2);
  }
  // Limbs 2 and 3 (lane t = 1) weigh 65536 against limbs 0 and 1.
  out_g = fmaf(__shfl_xor_sync(0xffffffffu, acc_g, 1), 65536.0f, acc_g);
  out_8 = fmaf(__shfl_xor_sync(0xffffffffu, acc_8, 1), 65536.0f, acc_8);
}

// Consumes the lm_head's tiles with the limb planes in x. A tile's rows
// form blocks of 16 (8 from each code region); warps take the stage's blocks
// in turn, each covering every quad of its block, so no block barrier or
// reduction is needed per tile. Each lane keeps its running argmax (and
// stores the logits where asked), as the CUDA-core GEMV does.
template <uint32_t FMT>
__device__ void gemv_tiles_mma(Ctx& c, const Piece* pieces, int np, Best& best, float* logits_out) {
  const uint32_t lane = static_cast<uint32_t>(c.lane), warp = static_cast<uint32_t>(c.warp);
  const uint32_t g = lane >> 2, t = lane & 3u;
  const MmaLane L = mma_lane<FMT>(c);
  uint32_t unit = 0;
  for (int p = 0; p < np; ++p) {
    const Piece pc = pieces[p];
    const uint32_t per = rows_per_tile(pc, true);
    for (uint32_t r = 0; r < pc.rows; r += per) {
      const uint32_t nr = min(per, pc.rows - r);
      const uint32_t ha = (nr + 1) / 2, hb = nr - ha;
      const uint32_t blocks = (ha + 7) / 8;
      const uint8_t* base = acquire_tile(c);
      for (uint32_t b = 0; b < blocks; ++b, ++unit) {
        if (unit % kConsumerWarps != warp || !c.ok) continue;
        float tg, t8;
        block_dot<FMT>(c, L, base, pc, nr, b, tg, t8);
        // MMA rows g and g + 8: local rows 8 b + (g >> 1) and + 4 of region g & 1.
        const uint32_t region = g & 1u, size = region ? hb : ha;
        const uint32_t l0 = 8 * b + (g >> 1);
        const float tot[2] = {tg, t8};
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (t != 0 || l0 + 4 * k >= size) continue;
          const uint32_t row = pc.out0 + r + region * ha + l0 + 4 * k;
          if (logits_out) logits_out[row] = tot[k];
          const float key = argmax_key(tot[k], row);
          if (key > best.v || (key == best.v && row < best.i)) best = Best{key, row};
        }
      }
      release_tile(c);
    }
  }
}

// The lm_head on the integer tensor cores and the conversion of its input,
// out of line and with plain-value arguments: inlined, they changed the
// register allocation of the layer stages' walk and slowed those stages more
// than the lm_head gained.
struct LmResult {
  uint32_t it;
  uint32_t ok;
  float v;
  uint32_t i;
};
template <uint32_t FMT>
__device__ __noinline__ LmResult lm_head_mma(const DecodeLaunch* P, const DevModel* m, Smem* s, uint32_t it, Piece pc,
                                             float* logits_out, float best_v, uint32_t best_i) {
  Ctx c{P, m, s, it, 0, true, static_cast<int>(threadIdx.x / 32), static_cast<int>(threadIdx.x % 32),
        static_cast<int>(threadIdx.x), false, 0, 0, 0, 0};
  Best best{best_v, best_i};
  gemv_tiles_mma<FMT>(c, &pc, 1, best, logits_out);
  return LmResult{c.it, c.ok ? 1u : 0u, best.v, best.i};
}
template <uint32_t FMT>
__device__ __noinline__ void lm_input_limbs(const DecodeLaunch* P, const DevModel* m, Smem* s, uint32_t width) {
  Ctx c{P, m, s, 0, 0, true, static_cast<int>(threadIdx.x / 32), static_cast<int>(threadIdx.x % 32),
        static_cast<int>(threadIdx.x), false, 0, 0, 0, 0};
  limbs_from_x<FMT>(c, width);
}

// ---- exact mode: dot products in the reference's order ----
//
// One lane of dotF32 (kernels.zig:39-51) over a row that linearQuantized
// dequantizes first (kernels.zig:118-158, quant.zig:315-345): lane j sums
// w[4 i + j] * x[4 i + j] for i = 0, 1, 2, ... with every product and sum
// rounded, where w = (code - bias) * scale exactly. `xl` is lane array j of x.
template <uint32_t FMT>
__device__ __forceinline__ float lane_dot(const uint8_t* scales, const uint8_t* codes, uint32_t groups, const float* xl,
                                          uint32_t j) {
  float l = 0.0f;
  for (uint32_t g = 0; g < groups; ++g) {
    const float s = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(scales)[g]);
    if constexpr (FMT == kFormatQ8) {
      // Word q of the group's codes holds elements 4 q .. 4 q + 3; lane j takes byte j.
      const uint4* cw = reinterpret_cast<const uint4*>(codes + 64u * g);
      const float4* xg = reinterpret_cast<const float4*>(xl + 16u * g);
      const uint32_t sel = 0x7440u | j;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 w = cw[q];
        const float4 xv = xg[q];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        const float xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float cv = __fadd_rn(bits_f32(__byte_perm(ws[e], kMagic, sel)), kNegQ8);  // code - 128, exact
          l = __fadd_rn(l, __fmul_rn(__fmul_rn(cv, s), xs[e]));
        }
      }
    } else if constexpr (FMT == kFormatQ4) {
      // Word q holds elements 8 q .. 8 q + 7 at nibble positions 0..7; lane j
      // takes positions j and j + 4 (lane indices 2 q and 2 q + 1).
      const uint4* cw = reinterpret_cast<const uint4*>(codes + 32u * g);
      const float2* xg = reinterpret_cast<const float2*>(xl + 16u * g);
      const uint32_t sh = 4u * j;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 w = cw[h];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 xv = xg[4 * h + e];
          const float c0 = __fadd_rn(bits_f32(((ws[e] >> sh) & 0xFu) | kMagic), kNegM0);  // u - 8, exact
          const float c1 = __fadd_rn(bits_f32(((ws[e] >> (sh + 16u)) & 0xFu) | kMagic), kNegM0);
          l = __fadd_rn(l, __fmul_rn(__fmul_rn(c0, s), xv.x));
          l = __fadd_rn(l, __fmul_rn(__fmul_rn(c1, s), xv.y));
        }
      }
    } else {
      const uint8_t* grp = codes + 40u * g;
      for (uint32_t i = 0; i < 16; ++i) {
        const float cv = static_cast<float>(q5_code(grp, 4u * i + j));
        l = __fadd_rn(l, __fmul_rn(__fmul_rn(cv, s), xl[16u * g + i]));
      }
    }
  }
  return l;
}

// Consumes the stage's tiles in exact mode. Warps 0-3 take the stage's even
// tiles and warps 4-7 its odd ones; in a tile, thread 4 r + j of the group
// runs lane j of rows r, r + 32, ..., and the row's sum is
// ((l0 + l1) + l2) + l3 as @reduce(.Add) forms it.
template <uint32_t FMT>
__device__ void gemv_tiles_exact(Ctx& c, const Piece* pieces, int np, bool lm, Best& best, float* logits_out) {
  const uint32_t grp = static_cast<uint32_t>(c.warp) >> 2;
  const uint32_t t = static_cast<uint32_t>(c.tid) & 127u;
  const uint32_t j = t & 3u;
  const float* xl = c.s->x + j * x_lane_stride(pieces[0].scale_row / 2 * kGroup);
  uint32_t n = 0;
  for (int p = 0; p < np; ++p) {
    const Piece pc = pieces[p];
    const uint32_t per = rows_per_tile(pc);
    const uint32_t groups = pc.scale_row / 2;
    for (uint32_t r = 0; r < pc.rows; r += per, ++n) {
      const uint32_t nr = min(per, pc.rows - r);
      const uint8_t* base = acquire_tile(c);
      if (c.ok && (n & 1u) == grp) {
        const uint8_t* codes = base + nr * pc.scale_row;
        for (uint32_t i0 = 0; i0 < nr; i0 += 32) {
          const uint32_t i = i0 + (t >> 2);
          const uint32_t row = min(i, nr - 1);
          const float l = lane_dot<FMT>(base + row * pc.scale_row, codes + row * pc.code_row, groups, xl, j);
          const float l1 = __shfl_down_sync(0xffffffffu, l, 1);
          const float l2 = __shfl_down_sync(0xffffffffu, l, 2);
          const float l3 = __shfl_down_sync(0xffffffffu, l, 3);
          if (j == 0 && i < nr) {
            const float total = __fadd_rn(__fadd_rn(__fadd_rn(l, l1), l2), l3);
            if (!lm) {
              c.s->part[pc.local0 + r + i] = total;
            } else {
              const uint32_t out = pc.out0 + r + i;
              if (logits_out) logits_out[out] = total;
              const float key = argmax_key(total, out);
              if (key > best.v || (key == best.v && out < best.i)) best = Best{key, out};
            }
          }
        }
      }
      release_tile(c);
    }
  }
}

// Runs one GEMV stage over the CTA's pieces.
template <bool E>
__device__ void gemv_stage(Ctx& c, const Piece* pieces_in, int np, uint32_t format, bool mma, bool lm, Best& best,
                           float* logits_out) {
  // The CUDA-core GEMVs see a stage's pieces end to end as one: the pieces
  // share K and format, their stage-local rows (local0) run on from one to
  // the next, and the producer cuts the tiles across them (issue_span). Only
  // the lm_head, a single piece, reads out0.
  Piece whole = pieces_in[0];
  for (int p = 1; p < np; ++p) whole.rows += pieces_in[p].rows;
  whole.local0 = 0;
  const Piece* pieces = mma ? pieces_in : &whole;
  if (!mma) np = np > 0 ? 1 : 0;
  if constexpr (E) {
    if (format == kFormatQ4) {
      gemv_tiles_exact<kFormatQ4>(c, pieces, np, lm, best, logits_out);
    } else if (format == kFormatQ5) {
      gemv_tiles_exact<kFormatQ5>(c, pieces, np, lm, best, logits_out);
    } else {
      gemv_tiles_exact<kFormatQ8>(c, pieces, np, lm, best, logits_out);
    }
    consumer_sync(kConsumerThreads);
    return;
  }
  if (mma) {
    // The lm_head stage is one piece (or none: a CTA without rows).
    if (np > 0 && c.ok) {
      const LmResult o = format == kFormatQ4
                             ? lm_head_mma<kFormatQ4>(c.P, c.m, c.s, c.it, pieces[0], logits_out, best.v, best.i)
                             : lm_head_mma<kFormatQ8>(c.P, c.m, c.s, c.it, pieces[0], logits_out, best.v, best.i);
      c.it = o.it;
      c.ok = o.ok != 0;
      best = Best{o.v, o.i};
    }
  } else if (format == kFormatQ4) {
    gemv_tiles<kFormatQ4>(c, pieces, np, lm, best, logits_out);
  } else if (format == kFormatQ5) {
    gemv_tiles<kFormatQ5>(c, pieces, np, lm, best, logits_out);
  } else {
    gemv_tiles<kFormatQ8>(c, pieces, np, lm, best, logits_out);
  }
  consumer_sync(kConsumerThreads);
}

// ---- attention (decodeAttentionStepQ8, kernels.zig:697-767, split-K) ----
//
// Units per kv head h: one per chunk of kAttnChunk cached positions
// (0 .. position - 1), then the new row's unit; CTA b takes units b,
// b + grid, ... The producer streams each unit's tile: for a chunk, its cached
// key/value rows (codes and scales, TMA boxes of the q8 cache); for every
// unit the layer's q/k RMSNorm weights and this position's RoPE row. The new
// row's unit computes and appends the new key/value row and its one-position
// partial; the chunk units, which no longer wait for that work, run beside it.

__device__ void attention_stage(Ctx& c, uint32_t layer, uint32_t position) {
  const DevModel& m = *c.m;
  AttnSmem* a = reinterpret_cast<AttnSmem*>(c.s->x);
  // Units per kv head: one per chunk of cached positions (0 .. position - 1),
  // then the new row's unit.
  const uint32_t cached = (position + kAttnChunk - 1) / kAttnChunk;
  const uint32_t slots = cached + 1;
  const uint32_t units = m.kv_heads * slots;
  const uint32_t kvw = m.kv_heads * kHeadDim;
  const uint32_t qw = m.q_heads * kHeadDim;
  const uint32_t kv_groups = kvw / kGroup;
  uint8_t* kl = c.P->k_cache + size_t(layer) * m.cache_layer_stride;
  uint8_t* vl = c.P->v_cache + size_t(layer) * m.cache_layer_stride;
  const int tid = c.tid;
  const int j = tid / kHeadDim;  // query head 2h + j; for the appended row, key (0) / value (1)
  const int d = tid % kHeadDim;
  const uint32_t newest = position;

  for (uint32_t u = blockIdx.x; u < units; u += gridDim.x) {
    const uint32_t h = u / slots;
    const uint32_t ch = u % slots;
    const bool last = ch == cached;  // the new row's unit
    // 1. Query rows 2h, 2h+1 (and for the new row's unit the new key/value
    // rows) from L2, issued before waiting for the tile.
    const float qraw = ld_cg(c.P->qkv + (2 * h + j) * kHeadDim + d);
    const float kvraw = last ? ld_cg(c.P->qkv + qw + size_t(j) * kvw + h * kHeadDim + d) : 0.0f;
    const uint8_t* tile = acquire_tile(c);
    const float* q_norm = reinterpret_cast<const float*>(tile + kTileQNorm);
    const float* k_norm = reinterpret_cast<const float*>(tile + kTileKNorm);
    const float* cos_row = reinterpret_cast<const float*>(tile + kTileCos);
    const float* sin_row = reinterpret_cast<const float*>(tile + kTileSin);
    // 2. Per-head RMSNorm of the queries and the new key (decoder.zig:180-195,
    // math.zig:120-130). The key's sum of squares runs in dimension order on
    // one thread and value * inverse_rms * weight rounds each product, so the
    // appended row equals the reference's on the same inputs. The queries are
    // never stored: their sums are warp reductions (head j on warps 4j..4j+3).
    {
      if (last && j == 0) a->ktmp[d] = kvraw;
      const float qss = warp_sum(qraw * qraw);
      if (c.lane == 0) c.s->red[c.warp] = qss;
      consumer_sync(kConsumerThreads);
      if (last && tid == 64) c.s->red[kConsumerWarps] = rms_inverse(sum_squares_seq(a->ktmp, kHeadDim), kHeadDim, m.eps);
      consumer_sync(kConsumerThreads);
      const float* r4 = c.s->red + 4 * j;
      const float inv = 1.0f / sqrtf(((r4[0] + r4[1]) + (r4[2] + r4[3])) / static_cast<float>(kHeadDim) + m.eps);
      const float qn = qraw * inv * q_norm[d];
      const float kn =
          (last && j == 0) ? __fmul_rn(__fmul_rn(kvraw, c.s->red[kConsumerWarps]), k_norm[d]) : 0.0f;
      a->tmp[j][d] = qn;
      if (last && j == 0) a->ktmp[d] = kn;
      consumer_sync(kConsumerThreads);
    }
    // 3. RoPE (rotate_half, kernels.zig:495-527) of the queries and the new key.
    const int pair = d % (kHeadDim / 2);
    const float cs = cos_row[pair], sn = sin_row[pair];
    a->q[j][d / 32][d % 32] = rope_rn(d < kHeadDim / 2, a->tmp[j][pair], a->tmp[j][pair + kHeadDim / 2], cs, sn);
    // 4. The new row's unit appends the new key (normed, rotated) and value
    // rows as q8 (decoder.zig:187-216, quant.zig:197-227): one 64-value group
    // per two warps. The codes also stay in shared memory for this unit.
    if (last) {
      float val = kvraw;
      if (j == 0) val = rope_rn(d < kHeadDim / 2, a->ktmp[pair], a->ktmp[pair + kHeadDim / 2], cs, sn);
      const float amax = warp_max(fabsf(val));
      consumer_sync(kConsumerThreads);
      if (c.lane == 0) c.s->red[c.warp] = amax;
      consumer_sync(kConsumerThreads);
      const int gw = (c.warp / 2) * 2;
      const float gmax = fmaxf(c.s->red[gw], c.s->red[gw + 1]);
      const __half sh = __float2half_rn(gmax / 128.0f);
      const uint8_t code = q8_code(val, __half2float(sh));
      uint8_t* plane = j == 0 ? kl : vl;
      plane[m.cache_scales_bytes + size_t(position) * kvw + h * kHeadDim + d] = code;
      reinterpret_cast<uint8_t*>(a->new_codes[j])[d] = code;
      if ((d % kGroup) == 0) {
        reinterpret_cast<uint16_t*>(plane + size_t(position) * kv_groups * 2)[h * 2 + d / kGroup] = __half_as_ushort(sh);
        a->new_scales[j][d / kGroup] = __half_as_ushort(sh);
      }
      // Later tokens read this row through TMA (the async proxy).
      fence_proxy_async_global();
    }
    consumer_sync(kConsumerThreads);
    if (last) {
      // The new row's attention: one position, so its softmax weight is 1
      // and the partial is (value row, score, 1). Query head j's score is
      // q . k over the two 64-value groups, each group's sum times its scale
      // (q8GroupDot, kernels.zig:636-661); warps 4j .. 4j + 3 hold head j.
      const float kc = static_cast<float>(reinterpret_cast<const uint8_t*>(a->new_codes[0])[d]) - 128.0f;
      const float part = warp_sum(a->q[j][d / 32][d % 32] * kc);
      if (c.lane == 0) c.s->red[c.warp] = part;
      consumer_sync(kConsumerThreads);
      const float* r4 = c.s->red + 4 * j;
      const float score = m.attn_scaling * ((r4[0] + r4[1]) * f16_bits_to_f32_fast(a->new_scales[0][0]) +
                                            (r4[2] + r4[3]) * f16_bits_to_f32_fast(a->new_scales[0][1]));
      const float vc = static_cast<float>(reinterpret_cast<const uint8_t*>(a->new_codes[1])[d]) - 128.0f;
      float* dst = c.P->attn_part + (size_t(2 * h + j) * c.P->max_chunks + ch) * kAttnPartStride;
      dst[d] = vc * f16_bits_to_f32_fast(a->new_scales[1][d / kGroup]);
      if (d == 0) {
        dst[kHeadDim] = score;
        dst[kHeadDim + 1] = 1.0f;
      }
      release_tile(c);
      consumer_sync(kConsumerThreads);  // the scratch is reused by the next unit
      continue;
    }
    // 5. Scores (q8GroupDot, kernels.zig:636-661): four lanes per position,
    // 32 dimensions each; the two lanes of a 64-value group add their sums
    // before the group scale.
    const uint32_t r = static_cast<uint32_t>(tid) / 4;
    const uint32_t qd = static_cast<uint32_t>(tid) % 4;
    float p0, p1;
    {
      const uint32_t pos = ch * kAttnChunk + r;
      const bool valid = pos < newest;  // the cached positions; the new row has its own unit
      const uint4* src = reinterpret_cast<const uint4*>(tile + kTileKCodes + r * kHeadDim + qd * 32);
      const uint4 kw0 = src[0], kw1 = src[1];
      const uint32_t kbits =
          *reinterpret_cast<const uint16_t*>(tile + kTileKScales + r * 16 + (h % 4) * 4 + (qd / 2) * 2);
      const uint32_t words[8] = {kw0.x, kw0.y, kw0.z, kw0.w, kw1.x, kw1.y, kw1.z, kw1.w};
      const uint64_t bias = pack2(kNegQ8, kNegQ8);
      uint64_t acc0 = 0, acc1 = 0;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float4 q0 = *reinterpret_cast<const float4*>(&a->q[0][qd][4 * w]);
        const float4 q1 = *reinterpret_cast<const float4*>(&a->q[1][qd][4 * w]);
        const uint64_t c01 = add2(pack2(bits_f32(__byte_perm(words[w], kMagic, 0x7440)),
                                        bits_f32(__byte_perm(words[w], kMagic, 0x7441))), bias);
        const uint64_t c23 = add2(pack2(bits_f32(__byte_perm(words[w], kMagic, 0x7442)),
                                        bits_f32(__byte_perm(words[w], kMagic, 0x7443))), bias);
        acc0 = fma2(c01, pack2(q0.x, q0.y), acc0);
        acc0 = fma2(c23, pack2(q0.z, q0.w), acc0);
        acc1 = fma2(c01, pack2(q1.x, q1.y), acc1);
        acc1 = fma2(c23, pack2(q1.z, q1.w), acc1);
      }
      const float2 f0 = unpack2(acc0), f1 = unpack2(acc1);
      float g0 = f0.x + f0.y, g1 = f1.x + f1.y;
      g0 += __shfl_xor_sync(0xffffffffu, g0, 1);
      g1 += __shfl_xor_sync(0xffffffffu, g1, 1);
      const float scale = f16_bits_to_f32_fast(kbits);
      g0 *= scale;
      g1 *= scale;
      g0 += __shfl_xor_sync(0xffffffffu, g0, 2);
      g1 += __shfl_xor_sync(0xffffffffu, g1, 2);
      const float sc0 = valid ? m.attn_scaling * g0 : -INFINITY;
      const float sc1 = valid ? m.attn_scaling * g1 : -INFINITY;
      // Chunk maxima (math.zig:77-93 subtracts the row max before exp).
      const float w0 = warp_max(sc0), w1 = warp_max(sc1);
      if (c.lane == 0) {
        c.s->red[c.warp] = w0;
        c.s->red[kConsumerWarps + c.warp] = w1;
      }
      consumer_sync(kConsumerThreads);
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        m0 = fmaxf(m0, c.s->red[w]);
        m1 = fmaxf(m1, c.s->red[kConsumerWarps + w]);
      }
      p0 = valid ? expf(sc0 - m0) : 0.0f;
      p1 = valid ? expf(sc1 - m1) : 0.0f;
      if (qd == 0) {
        a->prob[0][r] = p0;
        a->prob[1][r] = p1;
      }
      const float l0 = warp_sum(qd == 0 ? p0 : 0.0f), l1 = warp_sum(qd == 0 ? p1 : 0.0f);
      if (c.lane == 0) {
        a->lsum[0][c.warp] = l0;
        a->lsum[1][c.warp] = l1;
      }
      a->mx[j] = j == 0 ? m0 : m1;
      consumer_sync(kConsumerThreads);
    }
    // 6. Values (q8GroupAccumulate, kernels.zig:665-688): lane = 4
    // dimensions, warp = 8 positions.
    {
      float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      const uint32_t grp = static_cast<uint32_t>(c.lane) / 16;
#pragma unroll
      for (int i = 0; i < kAttnChunk / kConsumerWarps; ++i) {
        const uint32_t rr = c.warp * (kAttnChunk / kConsumerWarps) + i;
        const uint32_t pos = ch * kAttnChunk + rr;
        const uint32_t word = *reinterpret_cast<const uint32_t*>(tile + kTileVCodes + rr * kHeadDim + 4 * c.lane);
        const uint32_t bits = *reinterpret_cast<const uint16_t*>(tile + kTileVScales + rr * 16 + (h % 4) * 4 + grp * 2);
        const float scale = f16_bits_to_f32_fast(bits);
        const bool valid = pos < newest;
        const float sw0 = valid ? scale * a->prob[0][rr] : 0.0f;
        const float sw1 = valid ? scale * a->prob[1][rr] : 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float cv = bits_f32(__byte_perm(word, kMagic, 0x7440 + t)) + kNegQ8;  // code - 128, exact
          acc[0][t] = fmaf(cv, sw0, acc[0][t]);
          acc[1][t] = fmaf(cv, sw1, acc[1][t]);
        }
      }
      release_tile(c);
      *reinterpret_cast<float4*>(&a->vpart[c.warp][0][4 * c.lane]) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
      *reinterpret_cast<float4*>(&a->vpart[c.warp][1][4 * c.lane]) = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
    }
    consumer_sync(kConsumerThreads);
    // 7. One chunk: the output directly. Several: a chunk partial (o[d], max,
    // sum) to global, then the last unit of this kv head to finish combines
    // them (flash-decode rescale).
    float o = 0.0f, l = 0.0f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      o += a->vpart[w][j][d];
      l += a->lsum[j][w];
    }
    const float mj = a->mx[j];
    // 7. The chunk's partial (o[d], max, sum) goes to global memory; the O
    // stage merges the partials of every chunk of every head while it loads
    // its input (attention_into_x), so no unit waits for another here.
    {
      float* dst = c.P->attn_part + (size_t(2 * h + j) * c.P->max_chunks + ch) * kAttnPartStride;
      dst[d] = o;
      if (d == 0) {
        dst[kHeadDim] = mj;
        dst[kHeadDim + 1] = l;
      }
    }
    consumer_sync(kConsumerThreads);  // the scratch is reused by the next unit
  }
}

// ---- exact mode: attention in the reference's order ----
//
// decodeAttentionStepQ8 (kernels.zig:697-767) with its softmax
// (math.zig:77-93) as written: per query head, the scores of every cached
// position (q8GroupDot: four lanes per 64-value group, sums rounded in
// order), the maximum, exp of each difference, their sum in position order,
// one reciprocal, and the outputs summed over positions in order
// (q8GroupAccumulate). CTA h < kv_heads takes kv head h (query heads 2h and
// 2h + 1); the other CTAs have no attention work. Scores and value weights go
// through exact_scratch; the cache rows, including the one this stage
// appends, are read with ordinary loads.
struct AttnExact {
  alignas(16) float raw[4][kHeadDim];  // pre-norm query heads 2h, 2h + 1, then the new key and value rows
  alignas(16) float rot[3][kHeadDim];  // normed, rotated query heads and key
  float inv[4];
  float red[2][kConsumerWarps];
  float amax[kConsumerWarps];
};
static_assert(sizeof(AttnExact) <= sizeof(float) * kXMax, "exact attention scratch must fit the activation buffer");

__device__ void attention_stage_exact(const DecodeLaunch* P, const DevModel* mp_, Smem* s, uint32_t layer,
                                                   uint32_t position) {
  const DevModel& m = *mp_;
  const uint32_t h = blockIdx.x;
  if (h >= m.kv_heads) return;
  AttnExact* a = reinterpret_cast<AttnExact*>(s->x);
  const int warp = static_cast<int>(threadIdx.x / 32), lane = static_cast<int>(threadIdx.x % 32);
  const DevLayer& L = m.layers[layer];
  const uint32_t qw = m.q_heads * kHeadDim, kvw = m.kv_heads * kHeadDim, kv_groups = kvw / kGroup;
  const uint32_t mp = m.max_positions, n = position + 1;
  uint8_t* kl = P->k_cache + size_t(layer) * m.cache_layer_stride;
  uint8_t* vl = P->v_cache + size_t(layer) * m.cache_layer_stride;
  const int tid = static_cast<int>(threadIdx.x), j = tid / kHeadDim, d = tid % kHeadDim;
  // 1. The pre-norm rows: queries 2h + j, and the new key (j = 0) or value (j = 1).
  a->raw[j][d] = ld_cg(P->qkv + (2 * h + j) * kHeadDim + d);
  a->raw[2 + j][d] = ld_cg(P->qkv + qw + size_t(j) * kvw + h * kHeadDim + d);
  consumer_sync(kConsumerThreads);
  // 2. QK-RMSNorm (decoder.zig:180-195): sequential sums on three warps.
  if (tid == 0 || tid == 32 || tid == 64) {
    a->inv[tid / 32] = rms_inverse(sum_squares_seq(a->raw[tid / 32], kHeadDim), kHeadDim, m.eps);
  }
  consumer_sync(kConsumerThreads);
  a->rot[j][d] = __fmul_rn(__fmul_rn(a->raw[j][d], a->inv[j]), L.q_norm[d]);
  if (j == 0) a->rot[2][d] = __fmul_rn(__fmul_rn(a->raw[2][d], a->inv[2]), L.k_norm[d]);
  consumer_sync(kConsumerThreads);
  // 3. RoPE at this position (kernels.zig:495-527).
  const int pair = d % (kHeadDim / 2);
  const float cs = m.rope_cos[size_t(position) * (kHeadDim / 2) + pair];
  const float sn = m.rope_sin[size_t(position) * (kHeadDim / 2) + pair];
  const float qr = rope_rn(d < kHeadDim / 2, a->rot[j][pair], a->rot[j][pair + kHeadDim / 2], cs, sn);
  const float kr = j == 0 ? rope_rn(d < kHeadDim / 2, a->rot[2][pair], a->rot[2][pair + kHeadDim / 2], cs, sn) : 0.0f;
  consumer_sync(kConsumerThreads);
  a->rot[j][d] = qr;
  if (j == 0) a->rot[2][d] = kr;
  // 4. appendCacheRow (decoder.zig:68-106): the key (j = 0) and value
  // (j = 1) rows as q8, one 64-value group per two warps (quant.zig:197-227).
  {
    const float val = j == 0 ? kr : a->raw[3][d];
    const float amax = warp_max(fabsf(val));
    if (lane == 0) a->amax[warp] = amax;
    consumer_sync(kConsumerThreads);
    const int gw = (warp / 2) * 2;
    const __half sh = __float2half_rn(__fdiv_rn(fmaxf(a->amax[gw], a->amax[gw + 1]), 128.0f));
    uint8_t* plane = j == 0 ? kl : vl;
    plane[m.cache_scales_bytes + size_t(position) * kvw + h * kHeadDim + d] = q8_code(val, __half2float(sh));
    if ((d % kGroup) == 0) {
      reinterpret_cast<uint16_t*>(plane + size_t(position) * kv_groups * 2)[h * 2 + d / kGroup] = __half_as_ushort(sh);
    }
    // Later fast-mode tokens read this row through TMA (the async proxy).
    fence_proxy_async_global();
  }
  consumer_sync(kConsumerThreads);  // the appended row is visible to this CTA's loads below
  // 5. Scores (q8GroupDot, kernels.zig:636-661), both query heads per position.
  float* sc0 = P->exact_scratch + size_t(2 * h) * 3 * mp;  // [3][mp]: scores / exp, value weights of groups 0, 1
  float* sc1 = sc0 + size_t(3) * mp;
  for (uint32_t p = tid; p < n; p += kConsumerThreads) {
    const uint4* krow = reinterpret_cast<const uint4*>(kl + m.cache_scales_bytes + size_t(p) * kvw + h * kHeadDim);
    const uint16_t* ks = reinterpret_cast<const uint16_t*>(kl + size_t(p) * kv_groups * 2) + h * 2;
    float tot[2] = {0.0f, 0.0f};
#pragma unroll 1
    for (uint32_t g = 0; g < 2; ++g) {
      const float scale = f16_bits_to_f32(ks[g]);
      float lanes[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll 1
      for (int q = 0; q < 4; ++q) {
        const uint4 w = krow[4 * g + q];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const float cv = __fadd_rn(bits_f32(__byte_perm(ws[e], kMagic, 0x7440 + b)), kNegQ8);
            const uint32_t dim = 64 * g + 16 * q + 4 * e + b;
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) lanes[hh][b] = __fadd_rn(lanes[hh][b], __fmul_rn(cv, a->rot[hh][dim]));
          }
        }
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const float group = __fadd_rn(__fadd_rn(__fadd_rn(lanes[hh][0], lanes[hh][1]), lanes[hh][2]), lanes[hh][3]);
        tot[hh] = __fadd_rn(tot[hh], __fmul_rn(group, scale));
      }
    }
    sc0[p] = __fmul_rn(m.attn_scaling, tot[0]);
    sc1[p] = __fmul_rn(m.attn_scaling, tot[1]);
  }
  consumer_sync(kConsumerThreads);
  // 6. Row maxima (the order does not change a maximum).
  {
    float m0 = -INFINITY, m1 = -INFINITY;
    for (uint32_t p = tid; p < n; p += kConsumerThreads) {
      m0 = fmaxf(m0, sc0[p]);
      m1 = fmaxf(m1, sc1[p]);
    }
    m0 = warp_max(m0);
    m1 = warp_max(m1);
    if (lane == 0) {
      a->red[0][warp] = m0;
      a->red[1][warp] = m1;
    }
    consumer_sync(kConsumerThreads);
    m0 = -INFINITY;
    m1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      m0 = fmaxf(m0, a->red[0][w]);
      m1 = fmaxf(m1, a->red[1][w]);
    }
    // 7. exp(score - max) in place.
    for (uint32_t p = tid; p < n; p += kConsumerThreads) {
      sc0[p] = exp_ref(__fsub_rn(sc0[p], m0));
      sc1[p] = exp_ref(__fsub_rn(sc1[p], m1));
    }
  }
  consumer_sync(kConsumerThreads);
  // 8. The sums in position order, then one reciprocal each.
  if (tid == 0 || tid == 32) {
    const float* e = tid == 0 ? sc0 : sc1;
    float total = 0.0f;
    uint32_t p = 0;
    for (; p + 8 <= n; p += 8) {
      float t[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) t[i] = e[p + i];
#pragma unroll
      for (int i = 0; i < 8; ++i) total = __fadd_rn(total, t[i]);
    }
    for (; p < n; ++p) total = __fadd_rn(total, e[p]);
    a->inv[tid / 32] = __fdiv_rn(1.0f, total);
  }
  consumer_sync(kConsumerThreads);
  // 9. Value weights: scale of the position's value group times its
  // probability (q8GroupAccumulate's scaled_weight), for both groups.
  for (uint32_t q = tid; q < 2 * n; q += kConsumerThreads) {
    const uint32_t hh = q / n, p = q % n;
    float* sc = hh == 0 ? sc0 : sc1;
    const float prob = __fmul_rn(sc[p], a->inv[hh]);
    const uint16_t* vs = reinterpret_cast<const uint16_t*>(vl + size_t(p) * kv_groups * 2) + h * 2;
    sc[mp + p] = __fmul_rn(f16_bits_to_f32(vs[0]), prob);
    sc[2 * mp + p] = __fmul_rn(f16_bits_to_f32(vs[1]), prob);
  }
  consumer_sync(kConsumerThreads);
  // 10. Output dimension d of query head 2h + j: the sum over positions in order.
  {
    const float* sw = (j == 0 ? sc0 : sc1) + size_t(1 + d / kGroup) * mp;
    const uint8_t* vcol = vl + m.cache_scales_bytes + h * kHeadDim + d;
    float out = 0.0f;
    uint32_t p = 0;
    for (; p + 8 <= n; p += 8) {
      float cv[8], w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        cv[i] = __fadd_rn(static_cast<float>(vcol[size_t(p + i) * kvw]), -128.0f);
        w[i] = sw[p + i];
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) out = __fadd_rn(out, __fmul_rn(cv[i], w[i]));
    }
    for (; p < n; ++p) out = __fadd_rn(out, __fmul_rn(__fadd_rn(static_cast<float>(vcol[size_t(p) * kvw]), -128.0f), sw[p]));
    P->attn_out[(2 * h + j) * kHeadDim + d] = out;
  }
  consumer_sync(kConsumerThreads);  // the activation buffer is reused by the next stage
}

// ---- the consumer program ----

template <bool E>
__device__ void run_consumers(const DecodeLaunch& P, Smem* s) {
  const DevModel& m = *reinterpret_cast<const DevModel*>(s->model);
  Ctx c{&P, &m, s, 0, 0, true, static_cast<int>(threadIdx.x / 32), static_cast<int>(threadIdx.x % 32),
        static_cast<int>(threadIdx.x), false, 0, 0, 0, 0};
  const Span own = split_rows(m.hidden, blockIdx.x, gridDim.x);  // hidden rows of O and down
  const Span fr = split_rows(m.ffn, blockIdx.x, gridDim.x);      // ffn rows of gate and up
  uint32_t input = P.first_input;

  for (uint32_t t = 0; t < P.n_tokens && c.ok; ++t) {
    const uint32_t position = P.first_position + t;
    int32_t row = -1;
    if (t < P.n_forced) {
      input = P.forced_token[t];
      row = P.forced_row ? P.forced_row[t] : -1;
    }
    c.tracing = P.trace != nullptr && t == P.trace_token;
    const bool logits = t >= P.logits_from;
    const uint32_t walk = m.n_layers * kStagesPerLayer + (logits ? 1u : 0u);
    for (uint32_t q = 0; q < walk; ++q) {
      const uint32_t l = q / kStagesPerLayer;
      const int st = l < m.n_layers ? layer_stage(q % kStagesPerLayer) : kStLM;
      const uint32_t e0 = q * kTraceEventsPerStage;
      if (st == kStAttn) {
        // -- attention over position + 1 cached rows (decoder.zig:216-253)
        trace_mark(c, e0);
        if constexpr (E) {
          attention_stage_exact(&P, &m, s, l, position);
        } else {
          attention_stage(c, l, position);
        }
      } else {
        const uint32_t lq = st == kStLM ? 0 : l;
        const uint32_t format = stage_format(m, lq, st);
        // The default-mode q4/q8 lm_head multiplies on the integer tensor
        // cores (gemv_tiles_mma) and takes x unscaled; the other stages mask
        // nibbles against a prescaled x (store_x4).
        const bool mma = !E && st == kStLM && mma_gemv(st, format, m.hidden);
        const bool q4 = !mma && (format == kFormatQ4 || format == kFormatQ5);
        // -- stage input into x: the layer-0 input row, an RMSNorm of the
        // residual stream (decoder.zig:165-176, 259-262, 277-283), or the
        // attention output / SwiGLU activations; gate and up share one input.
        if (st == kStQKV && l == 0) {
          input_into_x<E>(c, input, row, own, q4);
        } else if (st == kStQKV || st == kStGateUp || st == kStLM) {
          norm_global_into_x<E>(c, P.hidden_g, m.hidden, q4);
        } else if (st == kStO) {
          if constexpr (E) {
            load_x_global<E>(c, P.attn_out, m.q_heads * kHeadDim, q4);
          } else {
            // Partials: one per chunk of cached positions, then the new row's.
            attention_into_x(c, P.attn_part, (position + kAttnChunk - 1) / kAttnChunk + 1, q4);
          }
        } else if (st == kStDown) {
          load_x_global<E>(c, P.act, m.ffn, q4);
        }
        // The integer lm_head takes its input as limb planes.
        if (mma) {
          if (format == kFormatQ4) {
            lm_input_limbs<kFormatQ4>(c.P, c.m, c.s, m.hidden);
          } else {
            lm_input_limbs<kFormatQ8>(c.P, c.m, c.s, m.hidden);
          }
        }
        trace_mark(c, e0);
        Piece pieces[3];
        const int np = stage_pieces(m, lq, st, blockIdx.x, gridDim.x, pieces);
        Best best{-INFINITY, 0xFFFFFFFFu};
        float* logits_out = (st == kStLM && P.logits_out && t + 1 == P.n_tokens) ? P.logits_out : nullptr;
        gemv_stage<E>(c, pieces, np, format, mma, st == kStLM, best, logits_out);
        // -- stage output
        if (st == kStQKV) {
          for (int p = 0; p < np; ++p) {
            for (uint32_t i = c.tid; i < pieces[p].rows; i += kConsumerThreads) {
              P.qkv[pieces[p].out0 + i] = s->part[pieces[p].local0 + i];
            }
          }
        } else if (st == kStO || st == kStDown) {
          // Residual adds (decoder.zig:256-257, 270-271) on this CTA's rows.
          for (uint32_t r = own.begin + c.tid; r < own.end; r += kConsumerThreads) {
            const float h = s->resid[r - own.begin] + s->part[r - own.begin];
            s->resid[r - own.begin] = h;
            P.hidden_g[r] = h;
          }
        } else if (st == kStGateUp) {
          // SwiGLU (kernels.zig:233-239): gate rows, then up rows, in part.
          const uint32_t nf = fr.end - fr.begin;
          for (uint32_t i = c.tid; i < nf; i += kConsumerThreads) {
            const float g = s->part[i];
            if constexpr (E) {
              const float silu = __fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g)));  // math.zig:69-71
              P.act[fr.begin + i] = __fmul_rn(silu, s->part[nf + i]);
            } else {
              const float silu = g / (1.0f + expf(-g));
              P.act[fr.begin + i] = silu * s->part[nf + i];
            }
          }
        } else {
          // lm_head: this CTA's first maximum (decoder.zig:290-301).
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
            const uint32_t oi = __shfl_xor_sync(0xffffffffu, best.i, o);
            if (ov > best.v || (ov == best.v && oi < best.i)) best = Best{ov, oi};
          }
          if (c.lane == 0) {
            s->amax_v[c.warp] = best.v;
            s->amax_i[c.warp] = best.i;
          }
          consumer_sync(kConsumerThreads);
          if (c.tid == 0) {
            Best b{s->amax_v[0], s->amax_i[0]};
            for (int w = 1; w < kConsumerWarps; ++w) {
              const Best o{s->amax_v[w], s->amax_i[w]};
              if (o.v > b.v || (o.v == b.v && o.i < b.i)) b = o;
            }
            P.amax_val[blockIdx.x] = b.v;
            P.amax_idx[blockIdx.x] = b.i;
          }
        }
      }
      trace_mark(c, e0 + 1);
      grid_barrier(c);
      if (!c.ok) break;
      trace_mark(c, e0 + 2);
    }
    if (!c.ok) break;
    if (c.tracing && c.tid == 0) {
      P.trace[blockIdx.x * kTraceEvents + kTraceEvents - 3] = c.tile_ns;
      P.trace[blockIdx.x * kTraceEvents + kTraceEvents - 2] = c.full_wait_ns;
      P.trace[blockIdx.x * kTraceEvents + kTraceEvents - 1] = c.bar_wait_ns;
    }
    if (logits) {
      // Every CTA combines the per-CTA maxima (one L2 round trip, then a
      // block reduction). CTA row ranges ascend, so lowest-index-on-tie over
      // (value, index) pairs is the reference's first-maximum rule.
      Best b{-INFINITY, 0xFFFFFFFFu};
      for (uint32_t q = c.tid; q < gridDim.x; q += kConsumerThreads) {
        const Best o{ld_cg(P.amax_val + q), __ldcg(P.amax_idx + q)};
        if (o.v > b.v || (o.v == b.v && o.i < b.i)) b = o;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, b.v, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, b.i, o);
        if (ov > b.v || (ov == b.v && oi < b.i)) b = Best{ov, oi};
      }
      if (c.lane == 0) {
        s->amax_v[c.warp] = b.v;
        s->amax_i[c.warp] = b.i;
      }
      consumer_sync(kConsumerThreads);
      if (c.tid == 0) {
        Best f{s->amax_v[0], s->amax_i[0]};
        for (int w = 1; w < kConsumerWarps; ++w) {
          const Best o{s->amax_v[w], s->amax_i[w]};
          if (o.v > f.v || (o.v == f.v && o.i < f.i)) f = o;
        }
        s->flag = f.i;
        if (blockIdx.x == 0) P.tokens_out[t] = f.i;
      }
      consumer_sync(kConsumerThreads);
      input = s->flag;
      consumer_sync(kConsumerThreads);
    }
  }
}

// E = exact mode (DecodeLaunch::exact): a separate instantiation, so the
// default kernel carries none of its code or register demands.
template <bool E>
__global__ void __launch_bounds__(kThreads, 1)
    decode_kernel(const __grid_constant__ DecodeLaunch P, const __grid_constant__ KvMaps maps) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem* s = reinterpret_cast<Smem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], kConsumerWarps);
    }
    fence_mbar_init();
    s->abort = 0u;
  }
  static_assert(sizeof(DevModel) % 8 == 0, "the model description copies as 8-byte words");
  for (uint32_t i = threadIdx.x; i < sizeof(DevModel) / 8; i += blockDim.x) {
    reinterpret_cast<uint64_t*>(s->model)[i] = __ldg(reinterpret_cast<const uint64_t*>(P.model) + i);
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerThreads) {
    run_producer(P, maps, s);
  } else {
    run_consumers<E>(P, s);
  }
}

}  // namespace

#if QWC_DECODE_WIDE_SLOTS
int launch_decode_wide(const DecodeLaunch& launch, const KvMaps& maps, int grid, void* stream) {
#else
int decode_grid_size(int device) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms;
}

int launch_decode(const DecodeLaunch& launch, const KvMaps& maps, int grid, void* stream) {
#endif
  const int smem = static_cast<int>(sizeof(Smem));
  const void* fn = launch.exact ? reinterpret_cast<const void*>(decode_kernel<true>)
                                : reinterpret_cast<const void*>(decode_kernel<false>);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return static_cast<int>(e);
  DecodeLaunch copy = launch;
  KvMaps maps_copy = maps;
  void* args[] = {&copy, &maps_copy};
  return static_cast<int>(cudaLaunchCooperativeKernel(fn, dim3(grid), dim3(kThreads), args, static_cast<size_t>(smem),
                                                      static_cast<cudaStream_t>(stream)));
}

}  // namespace qwc

// qwc_decode.cu -- the persistent sm_100a decode kernel for one stream.
//
// One launch runs `n_tokens` forward passes of Decoder.forwardToken
// (src/core/qwen3_asr/decoder.zig:133-287) followed, where logits are wanted,
// by the argmax (decoder.zig:290-301). One CTA per SM, co-resident
// (cooperative launch):
//
//   * warp 8 (producer) streams this CTA's fixed share of every weight matrix
//     -- whole rows, in the reference's two-plane q4/q8 layout -- from HBM into
//     a ring of shared-memory slots with cp.async.bulk, tracked by mbarriers.
//     Weights never depend on activations, so it runs ahead across phase
//     boundaries, layers and tokens and keeps HBM busy while the consumers
//     wait at barriers.
//   * warps 0-7 (consumers) dequantize in registers and reduce with warp
//     shuffles (the dot products of kernels.zig:118-158), then run the fused
//     epilogues: QK-RMSNorm + RoPE + q8 KV append inside the attention phase,
//     residual adds, SwiGLU, and the argmax.
//
// Phases per layer, separated by grid barriers: QKV -> attention (split-K
// flash decode over the q8 cache, last-arriver combine) -> O + residual ->
// RMSNorm + gate/up + SwiGLU -> down + residual. Every CTA recomputes the
// RMSNorm of the full hidden vector redundantly instead of taking another
// barrier. Every wait is bounded by `timeout_ns`; on expiry the kernel
// records an error, drains its in-flight copies and returns.

#include <cuda_runtime.h>

#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kSlots = 6;
constexpr uint32_t kSlotBytes = 28 * 1024;
constexpr uint32_t kXMax = 8192;        // floats in the activation buffer (max K)
constexpr uint32_t kRowsMax = 256;      // rows of one stage per CTA (non-LM stages)
constexpr uint32_t kResidMax = 256;     // hidden rows owned by one CTA

enum Stage : int { kStQKV = 0, kStO = 1, kStGate = 2, kStUp = 3, kStDown = 4, kStLM = 5 };

enum ErrorCode : int32_t { kErrBarrier = 1, kErrFull = 2, kErrEmpty = 3, kErrShape = 4 };

struct Smem {
  uint8_t ring[kSlots][kSlotBytes];
  uint64_t full[kSlots];
  uint64_t empty[kSlots];
  float x[kXMax];                 // activation vector, swizzled (x_index)
  float part[2][kRowsMax];        // per-row partial dot products (K segments)
  float gate[kRowsMax];           // gate outputs waiting for the up rows
  float resid[kResidMax];         // this CTA's rows of the residual stream
  float red[kConsumerWarps * 2];  // block reductions
  float amax_v[kConsumerWarps];
  uint32_t amax_i[kConsumerWarps];
  uint32_t flag;
};

// Attention scratch overlays the activation buffer (never live together).
struct AttnSmem {
  float q[2][kHeadDim];
  float tmp[2][kHeadDim];
  float prob[2][kAttnChunk];
  float vpart[kConsumerWarps][2][kHeadDim];
  float kv_new[2][kHeadDim];
};
static_assert(sizeof(AttnSmem) <= sizeof(float) * kXMax, "attention scratch must fit the activation buffer");

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

struct Piece {
  const DevMat* mat;
  uint32_t row0;     // first matrix row
  uint32_t rows;     // rows in this piece
  uint32_t local0;   // index of row0 within the CTA's share of the stage
  uint32_t out0;     // index of row0 in the stage's output vector
};

// The CTA's share of a stage: identical for the producer and the consumers.
__device__ int stage_pieces(const DevModel& m, uint32_t layer, int stage, uint32_t c, uint32_t n, Piece* out) {
  const DevLayer& L = m.layers[layer];
  int count = 0;
  auto add = [&](const DevMat* mat, uint32_t r0, uint32_t r1, uint32_t local0, uint32_t out0) {
    if (r1 > r0) out[count++] = Piece{mat, r0, r1 - r0, local0, out0};
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
    case kStGate: {
      const Span s = split_rows(L.gate.rows, c, n);
      add(&L.gate, s.begin, s.end, 0, s.begin);
      break;
    }
    case kStUp: {
      const Span s = split_rows(L.up.rows, c, n);
      add(&L.up, s.begin, s.end, 0, s.begin);
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

__device__ __forceinline__ uint32_t rows_per_tile(const DevMat& mat) { return kSlotBytes / (mat.scale_row + mat.code_row); }

// ---------------------------------------------------------------------------
// Producer
// ---------------------------------------------------------------------------

struct Producer {
  Smem* s;
  uint32_t it = 0;
  int32_t* error;
  uint64_t timeout_ns;
  bool ok = true;

  __device__ void issue(const DevMat& mat, uint32_t r0, uint32_t nr) {
    const uint32_t slot = it % kSlots;
    const uint32_t parity = ((it / kSlots) & 1u) ^ 1u;
    if (!mbar_wait_bounded(&s->empty[slot], parity, error, global_timer_ns() + timeout_ns, kErrEmpty)) {
      ok = false;
      return;
    }
    const uint32_t bytes_s = nr * mat.scale_row;
    const uint32_t bytes_c = nr * mat.code_row;
    mbar_arrive_expect_tx(&s->full[slot], bytes_s + bytes_c);
    bulk_g2s(s->ring[slot], mat.scales + size_t(r0) * mat.scale_row, bytes_s, &s->full[slot]);
    bulk_g2s(s->ring[slot] + bytes_s, mat.codes + size_t(r0) * mat.code_row, bytes_c, &s->full[slot]);
    ++it;
  }

  __device__ void stage(const DevModel& m, uint32_t layer, int st) {
    Piece pieces[3];
    const int np = stage_pieces(m, layer, st, blockIdx.x, gridDim.x, pieces);
    for (int p = 0; p < np && ok; ++p) {
      const uint32_t per = rows_per_tile(*pieces[p].mat);
      for (uint32_t r = 0; r < pieces[p].rows && ok; r += per) {
        issue(*pieces[p].mat, pieces[p].row0 + r, min(per, pieces[p].rows - r));
      }
    }
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

__device__ void run_producer(const DecodeLaunch& P, Smem* s) {
  if ((threadIdx.x & 31) != 0) return;
  const DevModel& m = *P.model;
  Producer pr{s, 0, P.error, P.timeout_ns, true};
  for (uint32_t t = 0; t < P.n_tokens && pr.ok; ++t) {
    for (uint32_t l = 0; l < m.n_layers && pr.ok; ++l) {
      for (int st = kStQKV; st <= kStDown && pr.ok; ++st) pr.stage(m, l, st);
    }
    if (t >= P.logits_from && pr.ok) pr.stage(m, 0, kStLM);
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
  uint64_t deadline;
  bool ok;
  int warp, lane, tid;
};

__device__ bool error_set(const int32_t* e) { return *reinterpret_cast<const volatile int32_t*>(e) != 0; }

// Grid-wide barrier among the consumer warps of every CTA. The counter is
// monotonic within a launch (zeroed by the host before it).
__device__ void grid_barrier(Ctx& c) {
  consumer_sync(kConsumerThreads);
  if (c.tid == 0) {
    c.barriers += 1;
    const uint32_t target = c.barriers * gridDim.x;
    __threadfence();
    red_release_add(c.P->barrier, 1);
    const uint64_t deadline = global_timer_ns() + c.P->timeout_ns;
    uint32_t spins = 0;
    while (ld_acquire(c.P->barrier) < target) {
      if ((++spins & 63u) == 0) {
        if (error_set(c.P->error)) break;
        if (global_timer_ns() > deadline) {
          atomicCAS(c.P->error, 0, kErrBarrier);
          break;
        }
      }
    }
    c.s->flag = error_set(c.P->error) ? 1u : 0u;
  }
  consumer_sync(kConsumerThreads);
  if (c.s->flag) c.ok = false;
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

// x <- rmsnorm(raw) * weight over `width` values already stored raw in x
// (math.zig:120-130: value * inverse_rms * weight).
__device__ void normalize_x(Ctx& c, uint32_t width, const float* weight) {
  float ss = 0.0f;
  for (uint32_t k = c.tid; k < width; k += kConsumerThreads) {
    const float v = c.s->x[x_index(k)];
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum(c, ss);
  const float inv = 1.0f / sqrtf(total / static_cast<float>(width) + c.m->eps);
  for (uint32_t k = c.tid; k < width; k += kConsumerThreads) {
    const uint32_t i = x_index(k);
    c.s->x[i] = c.s->x[i] * inv * __ldg(weight + k);
  }
  consumer_sync(kConsumerThreads);
}

// Copies a global vector other CTAs wrote into x (L2-coherent loads).
__device__ void load_x_global(Ctx& c, const float* src, uint32_t width) {
  for (uint32_t k4 = c.tid; k4 < width / 4; k4 += kConsumerThreads) {
    const float4 v = ld_cg4(reinterpret_cast<const float4*>(src) + k4);
    *reinterpret_cast<float4*>(&c.s->x[x_index(k4 * 4)]) = v;
  }
  consumer_sync(kConsumerThreads);
}

// Layer-0 input: the token's embedding row (decoder.zig:346-376, quant.zig:348-364)
// or an audio row, written raw into x.
__device__ void load_x_input(Ctx& c, uint32_t token, int32_t audio_row) {
  const DevModel& m = *c.m;
  const uint32_t hidden = m.hidden;
  if (audio_row >= 0) {
    const float* src = c.P->audio + size_t(audio_row) * hidden;
    for (uint32_t k = c.tid; k < hidden; k += kConsumerThreads) c.s->x[x_index(k)] = __ldg(src + k);
  } else {
    const DevMat& e = m.embed;
    const uint8_t* srow = e.scales + size_t(token) * e.scale_row;
    const uint8_t* crow = e.codes + size_t(token) * e.code_row;
    for (uint32_t k = c.tid; k < hidden; k += kConsumerThreads) {
      const uint32_t g = k / kGroup;
      const float scale = f16_bits_to_f32(__ldg(reinterpret_cast<const uint16_t*>(srow) + g));
      int code;
      if (e.format == kFormatQ4) {
        const uint8_t b = __ldg(crow + k / 2);
        code = static_cast<int>((k & 1u) ? (b >> 4) : (b & 0x0F)) - 8;
      } else {
        code = static_cast<int>(__ldg(crow + k)) - 128;
      }
      c.s->x[x_index(k)] = static_cast<float>(code) * scale;
    }
  }
  consumer_sync(kConsumerThreads);
}

// ---- GEMV over the streamed tiles ----

template <uint32_t FMT>
struct Fmt;
template <>
struct Fmt<kFormatQ4> {
  static constexpr int kVals = 32;     // weights per 16-byte chunk
  static constexpr int kPairs = 16;
  static constexpr uint32_t kDB = 32;  // code bytes per group
  static constexpr uint32_t kKPerByte = 2;
};
template <>
struct Fmt<kFormatQ8> {
  static constexpr int kVals = 16;
  static constexpr int kPairs = 8;
  static constexpr uint32_t kDB = 64;
  static constexpr uint32_t kKPerByte = 1;
};

// Loads this lane's activations for chunks [seg * CHS, seg * CHS + CHS) as
// packed pairs (q4: pre-scaled per nibble position).
template <uint32_t FMT, int CHS>
__device__ __forceinline__ void load_x_regs(const Smem* s, int lane, int seg, uint64_t (&x2)[CHS * Fmt<FMT>::kPairs]) {
#pragma unroll
  for (int jj = 0; jj < CHS; ++jj) {
    const uint32_t j = static_cast<uint32_t>(seg * CHS + jj);
    const uint32_t kbase = (16u * lane + 512u * j) * Fmt<FMT>::kKPerByte;
#pragma unroll
    for (int q = 0; q < Fmt<FMT>::kVals / 4; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(&s->x[x_index(kbase + 4 * q)]);
      if constexpr (FMT == kFormatQ4) {
        const int i0 = (4 * q) % 8;
        x2[jj * 16 + 2 * q + 0] = pack2(v.x * q4_xscale(i0 + 0), v.y * q4_xscale(i0 + 1));
        x2[jj * 16 + 2 * q + 1] = pack2(v.z * q4_xscale(i0 + 2), v.w * q4_xscale(i0 + 3));
      } else {
        x2[jj * 8 + 2 * q + 0] = pack2(v.x, v.y);
        x2[jj * 8 + 2 * q + 1] = pack2(v.z, v.w);
      }
    }
  }
}

// Dot product of one row of a tile (this lane's chunks) before the warp sum.
template <uint32_t FMT, int CHS>
__device__ __forceinline__ float row_partial(const uint8_t* srow, const uint8_t* crow, int lane, int seg,
                                             const uint64_t (&x2)[CHS * Fmt<FMT>::kPairs]) {
  float acc = 0.0f;
#pragma unroll
  for (int jj = 0; jj < CHS; ++jj) {
    const uint32_t off = 16u * lane + 512u * static_cast<uint32_t>(seg * CHS + jj);
    const uint4 w = *reinterpret_cast<const uint4*>(crow + off);
    const float scale = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(srow + (off / Fmt<FMT>::kDB) * 2));
    float d;
    if constexpr (FMT == kFormatQ4) {
      d = q4_chunk_dot(w, x2 + jj * 16);
    } else {
      d = q8_chunk_dot(w, x2 + jj * 8);
    }
    acc = fmaf(d, scale, acc);
  }
  return acc;
}

struct Best {
  float v;
  uint32_t i;
};

// Consumes the stage's tiles. Non-LM stages leave per-row partial sums in
// s->part[seg][local]; the LM stage keeps a running argmax per warp and
// optionally stores the logits.
template <uint32_t FMT, int CHS>
__device__ void gemv_tiles(Ctx& c, const Piece* pieces, int np, int ks, bool lm, Best& best, float* logits_out) {
  const int seg = c.warp % ks;
  const int rstart = c.warp / ks;
  const int rstride = kConsumerWarps / ks;
  uint64_t x2[CHS * Fmt<FMT>::kPairs];
  load_x_regs<FMT, CHS>(c.s, c.lane, seg, x2);
  for (int p = 0; p < np; ++p) {
    const DevMat& mat = *pieces[p].mat;
    const uint32_t per = rows_per_tile(mat);
    for (uint32_t r = 0; r < pieces[p].rows; r += per) {
      const uint32_t nr = min(per, pieces[p].rows - r);
      const uint32_t slot = c.it % kSlots;
      const uint32_t parity = (c.it / kSlots) & 1u;
      if (c.ok && !mbar_wait_bounded(&c.s->full[slot], parity, c.P->error, global_timer_ns() + c.P->timeout_ns,
                                     kErrFull)) {
        c.ok = false;
      }
      if (c.ok) {
        const uint8_t* base = c.s->ring[slot];
        const uint8_t* codes = base + nr * mat.scale_row;
        for (uint32_t i = rstart; i < nr; i += rstride) {
          float v = row_partial<FMT, CHS>(base + i * mat.scale_row, codes + i * mat.code_row, c.lane, seg, x2);
          v = warp_sum(v);
          if (c.lane == 0) {
            const uint32_t local = pieces[p].local0 + r + i;
            if (!lm) {
              c.s->part[seg][local] = v;
            } else {
              const uint32_t row = pieces[p].out0 + r + i;
              if (logits_out) logits_out[row] = v;
              if (v > best.v || (v == best.v && row < best.i)) best = Best{v, row};
            }
          }
        }
      }
      __syncwarp();
      if (c.lane == 0) mbar_arrive(&c.s->empty[slot]);
      ++c.it;
    }
  }
}

__device__ __forceinline__ int choose_ks(const DevMat& mat, int vals_per_chunk, int& chs) {
  const int ch = static_cast<int>(mat.code_row / 512u);
  for (int ks = 1; ks <= kConsumerWarps; ks *= 2) {
    if (ch % ks == 0 && (ch / ks) * vals_per_chunk <= 96) {
      chs = ch / ks;
      return ks;
    }
  }
  chs = 0;
  return 0;
}

// Runs one GEMV stage over the CTA's pieces; returns the K-segment count.
__device__ int gemv_stage(Ctx& c, int stage, uint32_t layer, Best& best, float* logits_out) {
  Piece pieces[3];
  const int np = stage_pieces(*c.m, layer, stage, blockIdx.x, gridDim.x, pieces);
  const DevMat& ref = stage == kStLM ? c.m->lm_head
                    : stage == kStQKV ? c.m->layers[layer].q
                    : stage == kStO ? c.m->layers[layer].o
                    : stage == kStGate ? c.m->layers[layer].gate
                    : stage == kStUp ? c.m->layers[layer].up
                                     : c.m->layers[layer].down;
  const bool lm = stage == kStLM;
  int chs = 0;
  int ks;
  if (ref.format == kFormatQ4) {
    ks = choose_ks(ref, 32, chs);
    switch (chs) {
      case 1: gemv_tiles<kFormatQ4, 1>(c, pieces, np, ks, lm, best, logits_out); break;
      case 2: gemv_tiles<kFormatQ4, 2>(c, pieces, np, ks, lm, best, logits_out); break;
      case 3: gemv_tiles<kFormatQ4, 3>(c, pieces, np, ks, lm, best, logits_out); break;
      default: if (c.tid == 0) atomicCAS(c.P->error, 0, kErrShape); c.ok = false; break;
    }
  } else {
    ks = choose_ks(ref, 16, chs);
    switch (chs) {
      case 1: gemv_tiles<kFormatQ8, 1>(c, pieces, np, ks, lm, best, logits_out); break;
      case 2: gemv_tiles<kFormatQ8, 2>(c, pieces, np, ks, lm, best, logits_out); break;
      case 3: gemv_tiles<kFormatQ8, 3>(c, pieces, np, ks, lm, best, logits_out); break;
      case 4: gemv_tiles<kFormatQ8, 4>(c, pieces, np, ks, lm, best, logits_out); break;
      case 5: gemv_tiles<kFormatQ8, 5>(c, pieces, np, ks, lm, best, logits_out); break;
      case 6: gemv_tiles<kFormatQ8, 6>(c, pieces, np, ks, lm, best, logits_out); break;
      default: if (c.tid == 0) atomicCAS(c.P->error, 0, kErrShape); c.ok = false; break;
    }
  }
  consumer_sync(kConsumerThreads);
  return ks;
}

__device__ __forceinline__ float stage_row_value(const Smem* s, uint32_t local, int ks) {
  return ks == 2 ? s->part[0][local] + s->part[1][local] : s->part[0][local];
}

// ---- attention (decodeAttentionStepQ8, kernels.zig:697-767, split-K) ----

__device__ void attention_stage(Ctx& c, uint32_t layer, uint32_t position) {
  const DevModel& m = *c.m;
  AttnSmem* a = reinterpret_cast<AttnSmem*>(c.s->x);
  const uint32_t n_pos = position + 1;
  const uint32_t chunks = (n_pos + kAttnChunk - 1) / kAttnChunk;
  const uint32_t units = m.kv_heads * chunks;
  const uint32_t kvw = m.kv_heads * kHeadDim;
  const uint32_t qw = m.q_heads * kHeadDim;
  const uint32_t kv_groups = kvw / kGroup;
  const uint8_t* kl = c.P->k_cache + size_t(layer) * m.cache_layer_stride;
  const uint8_t* vl = c.P->v_cache + size_t(layer) * m.cache_layer_stride;
  const DevLayer& L = m.layers[layer];
  const float* cos_row = m.rope_cos + size_t(position) * (kHeadDim / 2);
  const float* sin_row = m.rope_sin + size_t(position) * (kHeadDim / 2);
  const int tid = c.tid;

  for (uint32_t u = blockIdx.x; u < units && c.ok; u += gridDim.x) {
    const uint32_t h = u / chunks;
    const uint32_t ch = u % chunks;
    const int j = tid / kHeadDim;        // which query head of the pair, or k (0) / v (1)
    const int d = tid % kHeadDim;
    // Query heads 2h, 2h+1: per-head RMSNorm (decoder.zig:180-186), then RoPE.
    {
      const float raw = ld_cg(c.P->qkv + (2 * h + j) * kHeadDim + d);
      const float ss = warp_sum(raw * raw);
      if (c.lane == 0) c.s->red[c.warp] = ss;
      consumer_sync(kConsumerThreads);
      const int w0 = j * 4;
      const float total = ((c.s->red[w0] + c.s->red[w0 + 1]) + c.s->red[w0 + 2]) + c.s->red[w0 + 3];
      const float inv = 1.0f / sqrtf(total / static_cast<float>(kHeadDim) + m.eps);
      a->tmp[j][d] = raw * inv * __ldg(L.q_norm + d);
      consumer_sync(kConsumerThreads);
      if (d < kHeadDim / 2) {
        const float lo = a->tmp[j][d], hi = a->tmp[j][d + kHeadDim / 2];
        const float cs = __ldg(cos_row + d), sn = __ldg(sin_row + d);
        a->q[j][d] = lo * cs - hi * sn;
        a->q[j][d + kHeadDim / 2] = hi * cs + lo * sn;
      }
      consumer_sync(kConsumerThreads);
    }
    // The unit holding the newest position appends its key and value row
    // (decoder.zig:187-216): key -> K-RMSNorm -> RoPE -> q8; value -> q8.
    if (ch == chunks - 1) {
      const float raw = ld_cg(c.P->qkv + qw + size_t(j) * kvw + h * kHeadDim + d);
      float val = raw;
      if (j == 0) {
        const float ss = warp_sum(raw * raw);
        if (c.lane == 0) c.s->red[c.warp] = ss;
      }
      consumer_sync(kConsumerThreads);
      if (j == 0) {
        const float total = ((c.s->red[0] + c.s->red[1]) + c.s->red[2]) + c.s->red[3];
        const float inv = 1.0f / sqrtf(total / static_cast<float>(kHeadDim) + m.eps);
        a->tmp[0][d] = raw * inv * __ldg(L.k_norm + d);
      }
      consumer_sync(kConsumerThreads);
      if (j == 0) {
        const int pair = d < kHeadDim / 2 ? d : d - kHeadDim / 2;
        const float lo = a->tmp[0][pair], hi = a->tmp[0][pair + kHeadDim / 2];
        const float cs = __ldg(cos_row + pair), sn = __ldg(sin_row + pair);
        val = d < kHeadDim / 2 ? lo * cs - hi * sn : hi * cs + lo * sn;
      }
      // q8 quantization of each 64-value group (quant.zig:197-227): two warps per group.
      const float amax = warp_max(fabsf(val));
      if (c.lane == 0) c.s->red[c.warp] = amax;
      consumer_sync(kConsumerThreads);
      const int gw = (c.warp / 2) * 2;
      const float gmax = fmaxf(c.s->red[gw], c.s->red[gw + 1]);
      const __half sh = __float2half_rn(gmax / 128.0f);
      const float stored = __half2float(sh);
      const uint8_t code = q8_code(val, stored);
      uint8_t* plane = const_cast<uint8_t*>(j == 0 ? kl : vl);
      plane[m.cache_scales_bytes + size_t(position) * kvw + h * kHeadDim + d] = code;
      if ((d % kGroup) == 0) {
        reinterpret_cast<uint16_t*>(plane + size_t(position) * kv_groups * 2)[h * 2 + d / kGroup] =
            __half_as_ushort(sh);
      }
      __threadfence_block();
      consumer_sync(kConsumerThreads);
    }
    // Scores: 16 positions per warp, a lane pair per position, one 64-value
    // group per lane (q8GroupDot, kernels.zig:636-661).
    const float scaling = m.attn_scaling;
    float m_run[2];
    {
      const uint32_t pl = c.warp * 16 + c.lane / 2;
      const uint32_t p = ch * kAttnChunk + pl;
      const int g = c.lane & 1;
      float s0 = 0.0f, s1 = 0.0f;
      if (p < n_pos) {
        const uint8_t* codes = kl + m.cache_scales_bytes + size_t(p) * kvw + h * kHeadDim + g * kGroup;
        const float scale = f16_bits_to_f32(
            __ldcg(reinterpret_cast<const unsigned short*>(kl + size_t(p) * kv_groups * 2) + h * 2 + g));
        uint64_t acc0 = 0, acc1 = 0;
        const uint64_t bias = pack2(kNegQ8, kNegQ8);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 w = __ldcg(reinterpret_cast<const uint4*>(codes) + q);
          const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int base = g * kGroup + q * 16 + t * 4;
            const uint64_t c01 = add2(pack2(bits_f32(__byte_perm(words[t], kMagic, 0x7440)),
                                            bits_f32(__byte_perm(words[t], kMagic, 0x7441))), bias);
            const uint64_t c23 = add2(pack2(bits_f32(__byte_perm(words[t], kMagic, 0x7442)),
                                            bits_f32(__byte_perm(words[t], kMagic, 0x7443))), bias);
            acc0 = fma2(c01, pack2(a->q[0][base], a->q[0][base + 1]), acc0);
            acc0 = fma2(c23, pack2(a->q[0][base + 2], a->q[0][base + 3]), acc0);
            acc1 = fma2(c01, pack2(a->q[1][base], a->q[1][base + 1]), acc1);
            acc1 = fma2(c23, pack2(a->q[1][base + 2], a->q[1][base + 3]), acc1);
          }
        }
        const float2 f0 = unpack2(acc0), f1 = unpack2(acc1);
        s0 = (f0.x + f0.y) * scale;
        s1 = (f1.x + f1.y) * scale;
      }
      s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
      s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
      const bool valid = p < n_pos;
      const float sc0 = valid ? scaling * s0 : -INFINITY;
      const float sc1 = valid ? scaling * s1 : -INFINITY;
      // Chunk maxima (math.zig:77-93 subtracts the row max before exp).
      const float w0 = warp_max(sc0), w1 = warp_max(sc1);
      consumer_sync(kConsumerThreads);
      if (c.lane == 0) {
        c.s->red[c.warp] = w0;
        c.s->red[kConsumerWarps + c.warp] = w1;
      }
      consumer_sync(kConsumerThreads);
      m_run[0] = -INFINITY;
      m_run[1] = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        m_run[0] = fmaxf(m_run[0], c.s->red[w]);
        m_run[1] = fmaxf(m_run[1], c.s->red[kConsumerWarps + w]);
      }
      if ((c.lane & 1) == 0) {
        a->prob[0][pl] = valid ? expf(sc0 - m_run[0]) : 0.0f;
        a->prob[1][pl] = valid ? expf(sc1 - m_run[1]) : 0.0f;
      }
      consumer_sync(kConsumerThreads);
    }
    // Values (q8GroupAccumulate, kernels.zig:665-688): lane = 4 dims, warp = 16 positions.
    {
      float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      const int g = (4 * c.lane) / kGroup;
      for (int q = 0; q < 16; ++q) {
        const uint32_t pl = c.warp * 16 + q;
        const uint32_t p = ch * kAttnChunk + pl;
        if (p >= n_pos) break;
        const uint32_t word =
            __ldcg(reinterpret_cast<const unsigned int*>(vl + m.cache_scales_bytes + size_t(p) * kvw + h * kHeadDim) +
                   c.lane);
        const float scale = f16_bits_to_f32(
            __ldcg(reinterpret_cast<const unsigned short*>(vl + size_t(p) * kv_groups * 2) + h * 2 + g));
        const float sw0 = scale * a->prob[0][pl];
        const float sw1 = scale * a->prob[1][pl];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float cv = static_cast<float>((word >> (8 * t)) & 0xFFu) - 128.0f;
          acc[0][t] = fmaf(cv, sw0, acc[0][t]);
          acc[1][t] = fmaf(cv, sw1, acc[1][t]);
        }
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        a->vpart[c.warp][0][4 * c.lane + t] = acc[0][t];
        a->vpart[c.warp][1][4 * c.lane + t] = acc[1][t];
      }
    }
    consumer_sync(kConsumerThreads);
    // Chunk partial: o[d], max, sum -> global, then the last unit of this kv
    // head combines every chunk (flash-decode rescale).
    {
      float o = 0.0f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) o += a->vpart[w][j][d];
      float* dst = c.P->attn_part + (size_t(2 * h + j) * c.P->max_chunks + ch) * (kHeadDim + 2);
      dst[d] = o;
      if (d == 0) {
        float l = 0.0f;
        for (uint32_t q = 0; q < kAttnChunk; ++q) l += a->prob[j][q];
        dst[kHeadDim] = m_run[j];
        dst[kHeadDim + 1] = l;
      }
    }
    __threadfence();
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      const uint32_t prev = atomicAdd(c.P->attn_count + h, 1u);
      c.s->flag = (prev == chunks - 1) ? 1u : 0u;
    }
    consumer_sync(kConsumerThreads);
    if (c.s->flag) {
      __threadfence();
      float mx = -INFINITY;
      for (uint32_t q = 0; q < chunks; ++q) {
        mx = fmaxf(mx, ld_cg(c.P->attn_part + (size_t(2 * h + j) * c.P->max_chunks + q) * (kHeadDim + 2) + kHeadDim));
      }
      float o = 0.0f, l = 0.0f;
      for (uint32_t q = 0; q < chunks; ++q) {
        const float* src = c.P->attn_part + (size_t(2 * h + j) * c.P->max_chunks + q) * (kHeadDim + 2);
        const float f = expf(ld_cg(src + kHeadDim) - mx);
        o = fmaf(ld_cg(src + d), f, o);
        l = fmaf(ld_cg(src + kHeadDim + 1), f, l);
      }
      c.P->attn_out[(2 * h + j) * kHeadDim + d] = o / l;
      if (tid == 0) c.P->attn_count[h] = 0;
    }
    consumer_sync(kConsumerThreads);
  }
}

// ---- the consumer program ----

__device__ void run_consumers(const DecodeLaunch& P, Smem* s) {
  const DevModel& m = *P.model;
  Ctx c{&P, &m, s, 0, 0, 0, true, static_cast<int>(threadIdx.x / 32), static_cast<int>(threadIdx.x % 32),
        static_cast<int>(threadIdx.x)};
  const Span own = split_rows(m.hidden, blockIdx.x, gridDim.x);  // hidden rows of O and down
  const uint32_t qw = m.q_heads * kHeadDim;
  uint32_t input = P.first_input;

  for (uint32_t t = 0; t < P.n_tokens && c.ok; ++t) {
    const uint32_t position = P.first_position + t;
    int32_t row = -1;
    if (t < P.n_forced) {
      input = P.forced_token[t];
      row = P.forced_row ? P.forced_row[t] : -1;
    }
    for (uint32_t l = 0; l < m.n_layers && c.ok; ++l) {
      const DevLayer& L = m.layers[l];
      Best best{-INFINITY, 0};
      // -- QKV: x = rmsnorm(hidden) (decoder.zig:165-176)
      if (l == 0) {
        load_x_input(c, input, row);
        for (uint32_t r = own.begin + c.tid; r < own.end; r += kConsumerThreads) {
          s->resid[r - own.begin] = s->x[x_index(r)];
        }
      } else {
        load_x_global(c, P.hidden_g, m.hidden);
      }
      normalize_x(c, m.hidden, L.attn_norm);
      {
        const int ks = gemv_stage(c, kStQKV, l, best, nullptr);
        Piece pieces[3];
        const int np = stage_pieces(m, l, kStQKV, blockIdx.x, gridDim.x, pieces);
        for (int p = 0; p < np; ++p) {
          for (uint32_t i = c.tid; i < pieces[p].rows; i += kConsumerThreads) {
            P.qkv[pieces[p].out0 + i] = stage_row_value(s, pieces[p].local0 + i, ks);
          }
        }
      }
      grid_barrier(c);
      if (!c.ok) break;
      // -- attention over position + 1 cached rows (decoder.zig:216-253)
      attention_stage(c, l, position);
      grid_barrier(c);
      if (!c.ok) break;
      // -- O projection + residual (decoder.zig:256-257)
      load_x_global(c, P.attn_out, qw);
      {
        const int ks = gemv_stage(c, kStO, l, best, nullptr);
        for (uint32_t r = own.begin + c.tid; r < own.end; r += kConsumerThreads) {
          const float h = s->resid[r - own.begin] + stage_row_value(s, r - own.begin, ks);
          s->resid[r - own.begin] = h;
          P.hidden_g[r] = h;
        }
      }
      grid_barrier(c);
      if (!c.ok) break;
      // -- RMSNorm -> gate/up -> SwiGLU (decoder.zig:259-269)
      load_x_global(c, P.hidden_g, m.hidden);
      normalize_x(c, m.hidden, L.ffn_norm);
      const Span fr = split_rows(m.ffn, blockIdx.x, gridDim.x);
      {
        const int ks = gemv_stage(c, kStGate, l, best, nullptr);
        for (uint32_t i = c.tid; i < fr.end - fr.begin; i += kConsumerThreads) s->gate[i] = stage_row_value(s, i, ks);
        consumer_sync(kConsumerThreads);
      }
      {
        const int ks = gemv_stage(c, kStUp, l, best, nullptr);
        for (uint32_t i = c.tid; i < fr.end - fr.begin; i += kConsumerThreads) {
          const float g = s->gate[i];
          const float silu = g / (1.0f + expf(-g));
          P.act[fr.begin + i] = silu * stage_row_value(s, i, ks);
        }
      }
      grid_barrier(c);
      if (!c.ok) break;
      // -- down + residual (decoder.zig:270-271)
      load_x_global(c, P.act, m.ffn);
      {
        const int ks = gemv_stage(c, kStDown, l, best, nullptr);
        for (uint32_t r = own.begin + c.tid; r < own.end; r += kConsumerThreads) {
          const float h = s->resid[r - own.begin] + stage_row_value(s, r - own.begin, ks);
          s->resid[r - own.begin] = h;
          P.hidden_g[r] = h;
        }
      }
      grid_barrier(c);
      if (!c.ok) break;
    }
    if (!c.ok) break;
    if (t >= P.logits_from) {
      // -- final RMSNorm -> lm_head -> argmax (decoder.zig:277-301)
      load_x_global(c, P.hidden_g, m.hidden);
      normalize_x(c, m.hidden, m.final_norm);
      Best best{-INFINITY, 0xFFFFFFFFu};
      float* logits = (P.logits_out && t + 1 == P.n_tokens) ? P.logits_out : nullptr;
      gemv_stage(c, kStLM, 0, best, logits);
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
      grid_barrier(c);
      if (!c.ok) break;
      if (c.tid == 0) {
        // Combine in CTA order: CTA row ranges ascend, so strict `>` keeps
        // the lowest index among equal maxima.
        Best b{ld_cg(P.amax_val), __ldcg(P.amax_idx)};
        for (uint32_t q = 1; q < gridDim.x; ++q) {
          const float v = ld_cg(P.amax_val + q);
          if (v > b.v) b = Best{v, __ldcg(P.amax_idx + q)};
        }
        s->flag = b.i;
        if (blockIdx.x == 0) P.tokens_out[t] = b.i;
      }
      consumer_sync(kConsumerThreads);
      input = s->flag;
      consumer_sync(kConsumerThreads);
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeLaunch P) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem* s = reinterpret_cast<Smem*>(smem_raw);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x >= kConsumerThreads) {
    run_producer(P, s);
  } else {
    run_consumers(P, s);
  }
}

}  // namespace

int decode_kernel_smem_bytes() { return static_cast<int>(sizeof(Smem)); }

int decode_grid_size(int device) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  return sms;
}

int launch_decode(const DecodeLaunch& launch, int grid, void* stream) {
  static bool configured = false;
  const int smem = decode_kernel_smem_bytes();
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = true;
  }
  DecodeLaunch copy = launch;
  void* args[] = {&copy};
  return static_cast<int>(cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(decode_kernel), dim3(grid),
                                                      dim3(kThreads), args, static_cast<size_t>(smem),
                                                      static_cast<cudaStream_t>(stream)));
}

}  // namespace qwc

// qwc_streams.cu -- the non-GEMM kernels of the batched multi-stream step.
//
// One step advances every active slot by one position through
// Decoder.forwardToken (src/core/qwen3_asr/decoder.zig:133-287) and, for all
// slots, the lm_head and argmax (decoder.zig:277-301). The projections run on
// the tensor cores (qwc_gemm.cu) with all slots as GEMM columns; the kernels
// here sit between them:
//
//   streams_norm       residual add of the previous projection (sum of its
//                      split-K partials) or the layer-0 input row, RMSNorm,
//                      f16 activations for the next GEMM;
//   streams_qkv        per (slot, kv head): QK-RMSNorm, RoPE, q8 append of
//                      the new key/value row, rotated queries for attention;
//   streams_attention  split-K decode attention over every slot's q8 cache
//                      (TMA boxes of 64 positions), last-arriver combine,
//                      f16 activations for the O projection;
//   streams_swiglu     silu(gate) * up into f16 activations for down;
//   streams_argmax     first index of each slot's maximum logit.
//
// Activations for a GEMM are stored as f16 pairs, hi = f16(x) in row `slot`
// and lo = f16(x - hi) in row 64 + slot, with each 8-value chunk in the order
// [0 4 1 5 2 6 3 7] (the weight dequantizer's order, qwc_gemm.cu).

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>

#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

constexpr int kNormThreads = 512;
constexpr int kNormPer4 = kHiddenMax / 4 / kNormThreads;  // float4 groups per thread

// Position of element e (0..7) of a chunk in the activation layout.
__device__ __forceinline__ uint32_t chunk_slot(uint32_t e) { return ((e & 3u) << 1) | (e >> 2); }

__device__ __forceinline__ float4 add4(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float add4(float a, float b) { return a + b; }

// Sum of a projection's split-K partials p[0], p[stride], ... in split
// order. The loads of B partials are issued before their adds, so a sum
// costs one L2 round trip per B splits rather than one per split.
template <int B, typename T>
__device__ __forceinline__ T sum_splits(const T* p, size_t stride, uint32_t splits) {
  T y = p[0];
  for (uint32_t s0 = 1; s0 < splits; s0 += B) {
    T t[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (s0 + b < splits) t[b] = p[size_t(s0 + b) * stride];
    }
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (s0 + b < splits) y = add4(y, t[b]);
    }
  }
  return y;
}

// Writes 8 f32 values (K order k0..k0+7) as one 16-byte chunk of the
// activation layout: f16 hi values at `dst`, the f16 remainders x - hi at
// `dst + lo_offset` (the slot's lo row).
__device__ __forceinline__ void store_chunk(__half* dst, size_t lo_offset, const float (&v)[8]) {
  __align__(16) __half h[8];
  __align__(16) __half l[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const __half hv = __float2half_rn(v[e]);
    h[chunk_slot(e)] = hv;
    l[chunk_slot(e)] = __float2half_rn(v[e] - __half2float(hv));
  }
  *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
  *reinterpret_cast<uint4*>(dst + lo_offset) = *reinterpret_cast<const uint4*>(l);
}

__device__ __forceinline__ void store_one(__half* dst, size_t lo_offset, float v) {
  const __half hv = __float2half_rn(v);
  dst[0] = hv;
  dst[lo_offset] = __float2half_rn(v - __half2float(hv));
}

// ---- residual + RMSNorm -> f16 activations (decoder.zig:165-176, 256-262, 277-283) ----
//
// One CTA per slot; a thread owns float4 groups of the hidden vector, so the
// loads of every split's partial are independent 16-byte loads.

template <int kInput>
__global__ void __launch_bounds__(kNormThreads) streams_norm_kernel(const StreamsStep P, const float* weight,
                                                                    const float* parts, uint32_t splits) {
  pdl_wait_and_trigger();
  __shared__ float xs[kHiddenMax];
  __shared__ float red[kNormThreads / 32];
  const DevModel& m = *P.model;
  const uint32_t s = blockIdx.x;
  const uint32_t hidden = m.hidden, h4 = hidden / 4;
  __half* xb = static_cast<__half*>(P.xb_h) + size_t(s) * hidden;
  const SlotStep d = P.desc[s];
  const size_t lo = size_t(kMaxStreams) * hidden;
  if (!d.active) {
    for (uint32_t c = threadIdx.x; c < hidden / 8; c += kNormThreads) {
      *reinterpret_cast<uint4*>(xb + c * 8) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(xb + lo + c * 8) = make_uint4(0, 0, 0, 0);
    }
    return;
  }
  float4* h = reinterpret_cast<float4*>(P.hidden + size_t(s) * hidden);
  // The norm weights do not depend on the reduction: load them first.
  float4 wv[kNormPer4];
#pragma unroll
  for (int i = 0; i < kNormPer4; ++i) {
    const uint32_t k4 = threadIdx.x + i * kNormThreads;
    wv[i] = k4 < h4 ? reinterpret_cast<const float4*>(weight)[k4] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float4 v[kNormPer4];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormPer4; ++i) {
    const uint32_t k4 = threadIdx.x + i * kNormThreads;
    float4 x = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (k4 < h4) {
      if (kInput) {
        if (d.audio_row >= 0) {
          x = reinterpret_cast<const float4*>(P.audio[d.cache] + size_t(d.audio_row) * hidden)[k4];
        } else {
          // embeddingRow, quantized branch (decoder.zig:346-376, quant.zig:348-364).
          const DevMat& e = m.embed;
          const uint32_t k = k4 * 4;
          const float scale = f16_bits_to_f32(
              reinterpret_cast<const uint16_t*>(e.scales + size_t(d.token) * e.scale_row)[k / kGroup]);
          const uint8_t* crow = e.codes + size_t(d.token) * e.code_row;
          float c[4];
          if (e.format == kFormatQ4) {
            const uint16_t b = *reinterpret_cast<const uint16_t*>(crow + k / 2);
            c[0] = static_cast<float>(static_cast<int>(b & 0xF) - 8);
            c[1] = static_cast<float>(static_cast<int>((b >> 4) & 0xF) - 8);
            c[2] = static_cast<float>(static_cast<int>((b >> 8) & 0xF) - 8);
            c[3] = static_cast<float>(static_cast<int>((b >> 12) & 0xF) - 8);
          } else {
            const uint32_t b = *reinterpret_cast<const uint32_t*>(crow + k);
#pragma unroll
            for (int t = 0; t < 4; ++t) c[t] = static_cast<float>(static_cast<int>((b >> (8 * t)) & 0xFF) - 128);
          }
          x = make_float4(c[0] * scale, c[1] * scale, c[2] * scale, c[3] * scale);
        }
      } else {
        // The projection is the sum of its split-K partials, then the
        // residual add (kernels.zig:221-230).
        const float4* pp = reinterpret_cast<const float4*>(parts) + size_t(s) * h4 + k4;
        const float4 r = h[k4];
        const float4 y = sum_splits<8>(pp, size_t(kMaxStreams) * h4, splits);
        x = make_float4(r.x + y.x, r.y + y.y, r.z + y.z, r.w + y.w);
      }
      h[k4] = x;
      ss = fmaf(x.x, x.x, ss);
      ss = fmaf(x.y, x.y, ss);
      ss = fmaf(x.z, x.z, ss);
      ss = fmaf(x.w, x.w, ss);
    }
    v[i] = x;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int w = 0; w < kNormThreads / 32; ++w) total += red[w];
  const float inv = 1.0f / sqrtf(total / static_cast<float>(hidden) + m.eps);
#pragma unroll
  for (int i = 0; i < kNormPer4; ++i) {
    const uint32_t k4 = threadIdx.x + i * kNormThreads;
    if (k4 < h4) {
      const float4 w = wv[i];
      xs[k4 * 4 + 0] = v[i].x * inv * w.x;
      xs[k4 * 4 + 1] = v[i].y * inv * w.y;
      xs[k4 * 4 + 2] = v[i].z * inv * w.z;
      xs[k4 * 4 + 3] = v[i].w * inv * w.w;
    }
  }
  __syncthreads();
  for (uint32_t c = threadIdx.x; c < hidden / 8; c += kNormThreads) {
    float w8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) w8[e] = xs[c * 8 + e];
    store_chunk(xb + c * 8, lo, w8);
  }
}

// ---- QK-norm, RoPE, q8 append (decoder.zig:177-216) ----

__global__ void __launch_bounds__(256) streams_qkv_kernel(const StreamsStep P, uint32_t layer, uint32_t splits) {
  pdl_wait_and_trigger();
  __shared__ float red[16];
  __shared__ float tq[2][kHeadDim];
  __shared__ float tk[kHeadDim];
  const DevModel& m = *P.model;
  const uint32_t h = blockIdx.x, s = blockIdx.y;
  const SlotStep d = P.desc[s];
  if (!d.active) return;
  const uint32_t qw = m.q_heads * kHeadDim, kvw = m.kv_heads * kHeadDim;
  const uint32_t rows = qw + 2 * kvw;
  const int tid = threadIdx.x, j = tid / kHeadDim, dd = tid % kHeadDim, warp = tid / 32, lane = tid % 32;
  const float* row = P.part0 + size_t(s) * rows;
  const size_t stride = size_t(kMaxStreams) * rows;
  const float qraw = sum_splits<8>(row + (2 * h + j) * kHeadDim + dd, stride, splits);
  const float kvraw = sum_splits<8>(row + qw + j * kvw + h * kHeadDim + dd, stride, splits);
  if (layer + 1 == m.n_layers) {
    // Kept for qwc_debug_scratch: the inputs of this step's last append.
    P.qkv_rows[size_t(s) * rows + (2 * h + j) * kHeadDim + dd] = qraw;
    P.qkv_rows[size_t(s) * rows + qw + j * kvw + h * kHeadDim + dd] = kvraw;
  }
  const DevLayer& L = m.layers[layer];
  // QK-RMSNorm (math.zig:120-130): sums of squares in dimension order on one
  // thread per head (different warps), each product rounded, so the appended
  // key row equals the reference's on the same pre-norm values.
  tq[j][dd] = qraw;
  if (j == 0) tk[dd] = kvraw;
  __syncthreads();
  if (tid == 0 || tid == 32 || tid == 64) {
    const float* v = tid == 64 ? tk : tq[tid / 32];
    red[tid / 32] = rms_inverse(sum_squares_seq(v, kHeadDim), kHeadDim, m.eps);
  }
  __syncthreads();
  const float qn = __fmul_rn(__fmul_rn(qraw, red[j]), L.q_norm[dd]);
  const float kn = j == 0 ? __fmul_rn(__fmul_rn(kvraw, red[2]), L.k_norm[dd]) : 0.0f;
  __syncthreads();
  tq[j][dd] = qn;
  if (j == 0) tk[dd] = kn;
  __syncthreads();
  const int pair = dd % (kHeadDim / 2);
  const float* cos_row = m.rope_cos + size_t(d.position) * (kHeadDim / 2);
  const float* sin_row = m.rope_sin + size_t(d.position) * (kHeadDim / 2);
  const float cs = cos_row[pair], sn = sin_row[pair];
  P.qrot[size_t(s) * qw + (2 * h + j) * kHeadDim + dd] =
      rope_rn(dd < kHeadDim / 2, tq[j][pair], tq[j][pair + kHeadDim / 2], cs, sn);
  float val = kvraw;
  if (j == 0) val = rope_rn(dd < kHeadDim / 2, tk[pair], tk[pair + kHeadDim / 2], cs, sn);
  // q8 row (quant.zig:197-227): groups of 64 values, two warps each.
  const float amax = warp_max(fabsf(val));
  __syncthreads();
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  const int gw = (warp / 2) * 2;
  const float gmax = fmaxf(red[gw], red[gw + 1]);
  const __half sh = __float2half_rn(gmax / 128.0f);
  const uint8_t code = q8_code(val, __half2float(sh));
  uint8_t* plane =
      (j == 0 ? P.k_cache : P.v_cache) + size_t(d.cache) * m.cache_stream_stride + size_t(layer) * m.cache_layer_stride;
  plane[m.cache_scales_bytes + size_t(d.position) * kvw + h * kHeadDim + dd] = code;
  if ((dd % kGroup) == 0) {
    reinterpret_cast<uint16_t*>(plane + size_t(d.position) * (kvw / kGroup) * 2)[h * 2 + dd / kGroup] =
        __half_as_ushort(sh);
  }
}

// ---- split-K decode attention over every slot (kernels.zig:697-767) ----
//
// Units (slot, kv head, 64-position chunk) in that order are dealt to CTAs in
// contiguous ranges, so a CTA walks consecutive chunks of the same (slot,
// head) and carries an online softmax across them (running max, sum and
// output). A producer warp keeps a ring of TMA boxes of upcoming chunks in
// flight. Each (slot, head) segment a CTA finishes becomes one partial
// (o[128], max, sum) per query head; the CTA whose segment completes the
// head's chunk count combines the partials (flash-decode rescale).

constexpr uint32_t kTK = 0;                                    // [64][128] key codes
constexpr uint32_t kTV = kTK + kAttnChunk * kHeadDim;          // [64][128] value codes
constexpr uint32_t kTKS = kTV + kAttnChunk * kHeadDim;         // [64][16 B] key scales (4 kv heads)
constexpr uint32_t kTVS = kTKS + kAttnChunk * 16;              // [64][16 B] value scales
constexpr uint32_t kTileBytes = kTVS + kAttnChunk * 16;
constexpr int kAttnSlots = 4;
constexpr int kAttnConsumers = 256;
static_assert(kTV % 128 == 0 && kTKS % 128 == 0 && kTVS % 128 == 0 && kTileBytes % 128 == 0,
              "TMA boxes land on 128-byte boundaries");

struct __align__(128) AttnSmem {
  uint8_t ring[kAttnSlots][kTileBytes];
  alignas(16) float q[2][4][36];   // rotated queries, 32-dim quarters padded against bank conflicts
  alignas(16) float vpart[8][2][kHeadDim];  // per-warp outputs at a segment's end
  alignas(16) float red[2][8];              // per-warp running maxima
  alignas(16) float lsum[2][8];             // per-warp running sums
  uint32_t prefix[kMaxStreams + 1];
  uint32_t pos[kMaxStreams];    // each column's newest position
  uint32_t cache[kMaxStreams];  // each column's cache slot
  uint32_t flag;
  alignas(8) uint64_t full[kAttnSlots];
  alignas(8) uint64_t empty[kAttnSlots];
};
static_assert(offsetof(AttnSmem, vpart) % 16 == 0 && offsetof(AttnSmem, q) % 16 == 0, "vector access alignment");

__device__ __forceinline__ void tma_load_4d(void* dst, const void* map, int32_t x, int32_t y, int32_t z, int32_t w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// Unit of column s (its stream's cache slot `cache`), kv head h, chunk ch.
struct UnitPos {
  uint32_t s, h, ch, chunks, cache;
};

__device__ __forceinline__ UnitPos unit_pos(const AttnSmem* a, const StreamsStep& P, uint32_t kv_heads, uint32_t u) {
  uint32_t lo = 0, hi = kMaxStreams;
  while (hi - lo > 1) {
    const uint32_t mid = (lo + hi) / 2;
    if (a->prefix[mid] <= u) lo = mid; else hi = mid;
  }
  const uint32_t chunks = a->pos[lo] / kAttnChunk + 1;
  const uint32_t r = u - a->prefix[lo];
  return UnitPos{lo, r / chunks, r % chunks, chunks, a->cache[lo]};
}

// The unit after `up` in (column, kv head, chunk) order, skipping columns
// without units; the walk from one unit to the next costs a few compares
// instead of unit_pos's search and division.
__device__ __forceinline__ UnitPos next_unit(const AttnSmem* a, uint32_t kv_heads, UnitPos up) {
  if (++up.ch < up.chunks) return up;
  up.ch = 0;
  if (++up.h < kv_heads) return up;
  up.h = 0;
  uint32_t s = up.s + 1;
  while (s < kMaxStreams - 1 && a->prefix[s + 1] == a->prefix[s]) ++s;
  up.s = s;
  up.chunks = a->pos[s] / kAttnChunk + 1;
  up.cache = a->cache[s];
  return up;
}

__global__ void __launch_bounds__(kAttnConsumers + 32, 2) streams_attention_kernel(const StreamsStep P,
                                                                               const __grid_constant__ KvMaps4 maps,
                                                                               uint32_t layer) {
  pdl_wait_and_trigger();
  extern __shared__ __align__(128) uint8_t attn_smem_raw[];
  AttnSmem* a = reinterpret_cast<AttnSmem*>(attn_smem_raw);
  const DevModel& m = *P.model;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const uint32_t qw = m.q_heads * kHeadDim;
  const uint32_t kv_heads = m.kv_heads;
  if (tid == 0) {
    for (int i = 0; i < kAttnSlots; ++i) {
      mbar_init(&a->full[i], 1);
      mbar_init(&a->empty[i], 8);
    }
    fence_mbar_init();
    uint32_t acc = 0;
    for (uint32_t s = 0; s < kMaxStreams; ++s) {
      a->prefix[s] = acc;
      const SlotStep d = P.desc[s];
      a->pos[s] = static_cast<uint32_t>(d.position);
      a->cache[s] = static_cast<uint32_t>(d.cache);
      if (d.active) acc += kv_heads * (d.position / kAttnChunk + 1);
    }
    a->prefix[kMaxStreams] = acc;
  }
  __syncthreads();
  const uint32_t total = a->prefix[kMaxStreams];
  const uint32_t u0 = static_cast<uint32_t>((uint64_t(total) * blockIdx.x) / gridDim.x);
  const uint32_t u1 = static_cast<uint32_t>((uint64_t(total) * (blockIdx.x + 1)) / gridDim.x);

  if (warp == 8) {
    // ---- producer: TMA boxes of units u0..u1 into the ring ----
    if (lane == 0) {
      uint32_t it = 0;
      UnitPos up = unit_pos(a, P, kv_heads, u0);
      for (uint32_t u = u0; u < u1; ++u, ++it, up = next_unit(a, kv_heads, up)) {
        const uint32_t slot = it % kAttnSlots;
        if (it >= kAttnSlots &&
            !mbar_wait_bounded(&a->empty[slot], ((it / kAttnSlots) - 1) & 1u, P.error, P.timeout_ns, 102)) {
          break;
        }
        uint8_t* dst = a->ring[slot];
        mbar_arrive_expect_tx(&a->full[slot], kTileBytes);
        const int32_t y = static_cast<int32_t>(up.ch * kAttnChunk), z = static_cast<int32_t>(layer),
                      w = static_cast<int32_t>(up.cache);
        const int32_t xs = static_cast<int32_t>((up.h * 4u) & ~15u);
        tma_load_4d(dst + kTK, maps.k_codes, static_cast<int32_t>(up.h * kHeadDim), y, z, w, &a->full[slot]);
        tma_load_4d(dst + kTV, maps.v_codes, static_cast<int32_t>(up.h * kHeadDim), y, z, w, &a->full[slot]);
        tma_load_4d(dst + kTKS, maps.k_scales, xs, y, z, w, &a->full[slot]);
        tma_load_4d(dst + kTVS, maps.v_scales, xs, y, z, w, &a->full[slot]);
      }
      // Every armed box must land before the CTA exits.
      const uint32_t n = u1 > u0 ? u1 - u0 : 0;
      for (uint32_t i = (n > kAttnSlots ? n - kAttnSlots : 0); i < n; ++i) {
        const uint64_t deadline = global_timer_ns() + 1000000000ull;
        while (!mbar_try_wait(&a->full[i % kAttnSlots], (i / kAttnSlots) & 1u) && global_timer_ns() < deadline) {
        }
      }
    }
    return;
  }

  // ---- consumers: 8 warps; warp w takes positions 8w..8w+7 of every tile ----
  //
  // Each warp carries its own online softmax (running max, sum and output
  // per query head) across the units of a (slot, head) segment, so a unit
  // needs no block-wide synchronisation: the warps meet only when a segment
  // ends, where their states are merged (flash-decode rescale).
  // Scores: lane (i, qd) = (lane / 4, lane % 4) holds position 8w + i, dims
  // 32 qd .. 32 qd + 31; the two lanes of a 64-value group add their sums
  // before the group scale (q8GroupDot, kernels.zig:636-661).
  // Values: lane l holds output dims 4 l .. 4 l + 3 of both query heads.
  const int j = tid / kHeadDim, dd = tid % kHeadDim;
  const uint32_t pi = static_cast<uint32_t>(lane) / 4, qd = static_cast<uint32_t>(lane) % 4;
  const uint32_t prow = static_cast<uint32_t>(warp) * 8 + pi;  // this lane's score row in the tile
  const uint32_t grp = static_cast<uint32_t>(lane) / 16;
  bool ok = true;
  float wm[2] = {-INFINITY, -INFINITY}, wl[2] = {0.0f, 0.0f};
  float wo[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
  UnitPos cur{0xFFFFFFFFu, 0xFFFFFFFFu, 0, 0, 0};
  uint32_t seg_first = 0, seg_count = 0;

  // Merges the warps' states of the current (slot, head) segment and emits
  // it: the final output when the segment covers every chunk of the head,
  // else a partial for the last-arriving CTA to combine.
  auto flush = [&]() {
    if (lane == 0) {
      a->red[0][warp] = wm[0];
      a->red[1][warp] = wm[1];
      a->lsum[0][warp] = wl[0];
      a->lsum[1][warp] = wl[1];
    }
    *reinterpret_cast<float4*>(&a->vpart[warp][0][4 * lane]) = make_float4(wo[0][0], wo[0][1], wo[0][2], wo[0][3]);
    *reinterpret_cast<float4*>(&a->vpart[warp][1][4 * lane]) = make_float4(wo[1][0], wo[1][1], wo[1][2], wo[1][3]);
    consumer_sync(kAttnConsumers);
    float m_run = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) m_run = fmaxf(m_run, a->red[j][w]);
    float o_run = 0.0f, l_run = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float mw = a->red[j][w];
      if (mw != -INFINITY) {
        const float f = expf(mw - m_run);
        o_run = fmaf(a->vpart[w][j][dd], f, o_run);
        l_run = fmaf(a->lsum[j][w], f, l_run);
      }
    }
    __half* xq = static_cast<__half*>(P.xb_q) + size_t(cur.s) * qw;
    const size_t xq_lo = size_t(kMaxStreams) * qw;
    const uint32_t col = (2 * cur.h + j) * kHeadDim + dd;
    const uint32_t out_index = (col & ~7u) | chunk_slot(col & 7u);
    if (seg_count == cur.chunks) {
      store_one(xq + out_index, xq_lo, o_run / l_run);
      consumer_sync(kAttnConsumers);  // red / vpart reused by the next segment
      return;
    }
    float* part = P.attn_part + ((size_t(cur.s) * m.q_heads + 2 * cur.h + j) * P.max_chunks + seg_first) * (kHeadDim + 2);
    part[dd] = o_run;
    if (dd == 0) {
      part[kHeadDim] = m_run;  // a non-NaN max marks the chunk as a segment start
      part[kHeadDim + 1] = l_run;
    }
    // The counter update is acquire-release at gpu scope: its release (after
    // the bar.sync) publishes this CTA's partial, and the last arriver's
    // acquire makes every other CTA's partial visible to its loads.
    consumer_sync(kAttnConsumers);
    uint32_t* counter = P.attn_count + size_t(cur.s) * kv_heads + cur.h;
    if (tid == 0) {
      const uint32_t prev = atom_add_acq_rel(counter, seg_count);
      a->flag = (prev + seg_count == cur.chunks) ? 1u : 0u;
    }
    consumer_sync(kAttnConsumers);
    if (a->flag) {
      // Segment starts are read sixteen chunks at a time with every load of a
      // batch in flight together; NaN maxima mark chunks no segment starts at.
      float mx = -INFINITY, o = 0.0f, l = 0.0f;
      const float* base = P.attn_part + (size_t(cur.s) * m.q_heads + 2 * cur.h + j) * P.max_chunks * (kHeadDim + 2);
      for (uint32_t c0 = 0; c0 < cur.chunks; c0 += 16) {
        float pm[16], po[16], pl[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          pm[q] = -INFINITY;
          po[q] = 0.0f;
          pl[q] = 0.0f;
          if (c0 + q < cur.chunks) {
            const float* src = base + size_t(c0 + q) * (kHeadDim + 2);
            pm[q] = ld_cg(src + kHeadDim);
            po[q] = ld_cg(src + dd);
            pl[q] = ld_cg(src + kHeadDim + 1);
          }
        }
        float bm = mx;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (pm[q] == pm[q]) bm = fmaxf(bm, pm[q]);
        }
        const float rescale = (mx == -INFINITY) ? 0.0f : expf(mx - bm);
        o *= rescale;
        l *= rescale;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          if (pm[q] == pm[q] && pm[q] != -INFINITY) {
            const float f = expf(pm[q] - bm);
            o = fmaf(po[q], f, o);
            l = fmaf(pl[q], f, l);
          }
        }
        mx = bm;
      }
      store_one(xq + out_index, xq_lo, o / l);
      consumer_sync(kAttnConsumers);
      // Reset for the next step: partial maxima back to NaN, counter to 0.
      for (uint32_t c = tid; c < cur.chunks * 2; c += kAttnConsumers) {
        float* base2 = P.attn_part + (size_t(cur.s) * m.q_heads + 2 * cur.h + (c & 1u)) * P.max_chunks * (kHeadDim + 2);
        base2[size_t(c >> 1) * (kHeadDim + 2) + kHeadDim] = __int_as_float(-1);
      }
      if (tid == 0) *counter = 0;
    }
    consumer_sync(kAttnConsumers);
  };

  const float scaling = m.attn_scaling;
  const uint64_t bias = pack2(kNegQ8, kNegQ8);
  uint32_t it = 0;
  UnitPos up = unit_pos(a, P, kv_heads, u0);
  for (uint32_t u = u0; u < u1; ++u, ++it, up = next_unit(a, kv_heads, up)) {
    if (up.s != cur.s || up.h != cur.h) {
      if (cur.s != 0xFFFFFFFFu) flush();  // ends with every warp past the previous segment
      cur = up;
      seg_first = up.ch;
      seg_count = 0;
      wm[0] = wm[1] = -INFINITY;
      wl[0] = wl[1] = 0.0f;
#pragma unroll
      for (int t = 0; t < 4; ++t) wo[0][t] = wo[1][t] = 0.0f;
      a->q[j][dd / 32][dd % 32] = P.qrot[size_t(up.s) * qw + (2 * up.h + j) * kHeadDim + dd];
      consumer_sync(kAttnConsumers);
    }
    const uint32_t slot = it % kAttnSlots;
    if (ok && !mbar_wait_bounded(&a->full[slot], (it / kAttnSlots) & 1u, P.error, P.timeout_ns, 101)) {
      ok = false;
    }
    const uint8_t* tile = a->ring[slot];
    const uint32_t newest = a->pos[up.s];
    const uint32_t base_pos = up.ch * kAttnChunk + static_cast<uint32_t>(warp) * 8;
    const bool valid = ok && base_pos + pi <= newest;
    float s0, s1;
    {
      const uint4* src = reinterpret_cast<const uint4*>(tile + kTK + prow * kHeadDim + qd * 32);
      const uint4 kw0 = src[0], kw1 = src[1];
      const uint32_t kbits = *reinterpret_cast<const uint16_t*>(tile + kTKS + prow * 16 + (up.h % 4) * 4 + (qd / 2) * 2);
      const uint32_t words[8] = {kw0.x, kw0.y, kw0.z, kw0.w, kw1.x, kw1.y, kw1.z, kw1.w};
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
      s0 = valid ? scaling * g0 : -INFINITY;
      s1 = valid ? scaling * g1 : -INFINITY;
    }
    // Online softmax over this warp's 8 positions (math.zig:77-93 subtracts
    // the row max before exp); the 4 lanes of a position hold equal scores.
    float mx0 = s0, mx1 = s1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(wm[0], mx0), mn1 = fmaxf(wm[1], mx1);
    const float p0 = valid ? __expf(s0 - mn0) : 0.0f;
    const float p1 = valid ? __expf(s1 - mn1) : 0.0f;
    const float r0 = (wm[0] == -INFINITY) ? 0.0f : __expf(wm[0] - mn0);
    const float r1 = (wm[1] == -INFINITY) ? 0.0f : __expf(wm[1] - mn1);
    // Lane (i, qd) also weighs position i's values: scale of value group
    // qd & 1 times the probability of query head qd >> 1.
    const float sw_lane = f16_bits_to_f32_fast(*reinterpret_cast<const uint16_t*>(
                              tile + kTVS + prow * 16 + (up.h % 4) * 4 + (qd & 1u) * 2)) *
                          ((qd >> 1) ? p1 : p0);
    float ls0 = p0, ls1 = p1;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      ls0 += __shfl_xor_sync(0xffffffffu, ls0, o);
      ls1 += __shfl_xor_sync(0xffffffffu, ls1, o);
    }
    wl[0] = fmaf(wl[0], r0, ls0);
    wl[1] = fmaf(wl[1], r1, ls1);
    wm[0] = mn0;
    wm[1] = mn1;
    // Values (q8GroupAccumulate, kernels.zig:665-688).
    // Packed pairs: (dims 4l, 4l+1) and (4l+2, 4l+3) of each head.
    uint64_t acc01[2] = {0, 0}, acc23[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t row = static_cast<uint32_t>(warp) * 8 + i;
      const uint32_t word = *reinterpret_cast<const uint32_t*>(tile + kTV + row * kHeadDim + 4 * lane);
      const float sw0 = __shfl_sync(0xffffffffu, sw_lane, 4 * i + grp);
      const float sw1 = __shfl_sync(0xffffffffu, sw_lane, 4 * i + grp + 2);
      const uint64_t c01 = add2(pack2(bits_f32(__byte_perm(word, kMagic, 0x7440)),
                                      bits_f32(__byte_perm(word, kMagic, 0x7441))), bias);  // code - 128, exact
      const uint64_t c23 = add2(pack2(bits_f32(__byte_perm(word, kMagic, 0x7442)),
                                      bits_f32(__byte_perm(word, kMagic, 0x7443))), bias);
      acc01[0] = fma2(c01, pack2(sw0, sw0), acc01[0]);
      acc23[0] = fma2(c23, pack2(sw0, sw0), acc23[0]);
      acc01[1] = fma2(c01, pack2(sw1, sw1), acc01[1]);
      acc23[1] = fma2(c23, pack2(sw1, sw1), acc23[1]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&a->empty[slot]);  // this warp is done with the tile
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const float2 v01 = unpack2(acc01[hh]), v23 = unpack2(acc23[hh]);
      const float rr = hh == 0 ? r0 : r1;
      wo[hh][0] = fmaf(wo[hh][0], rr, v01.x);
      wo[hh][1] = fmaf(wo[hh][1], rr, v01.y);
      wo[hh][2] = fmaf(wo[hh][2], rr, v23.x);
      wo[hh][3] = fmaf(wo[hh][3], rr, v23.y);
    }
    ++seg_count;
  }
  if (cur.s != 0xFFFFFFFFu) flush();
}

// ---- SwiGLU (kernels.zig:233-239) into f16 activations ----

__global__ void streams_swiglu_kernel(const StreamsStep P, uint32_t splits) {
  pdl_wait_and_trigger();
  const DevModel& m = *P.model;
  const uint32_t ffn = m.ffn, chunks = ffn / 8;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < kMaxStreams * chunks; i += gridDim.x * blockDim.x) {
    const uint32_t s = i / chunks, c = i % chunks;
    __half* dst = static_cast<__half*>(P.xb_f) + size_t(s) * ffn + c * 8;
    const size_t lo = size_t(kMaxStreams) * ffn;
    if (!P.desc[s].active) {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(dst + lo) = make_uint4(0, 0, 0, 0);
      continue;
    }
    // Gate rows at [0, ffn), up rows at [ffn, 2 ffn) of each partial row.
    const float4* g4 = reinterpret_cast<const float4*>(P.part0 + size_t(s) * 2 * ffn + c * 8);
    const float4* u4 = reinterpret_cast<const float4*>(P.part0 + size_t(s) * 2 * ffn + ffn + c * 8);
    const size_t stride = size_t(kMaxStreams) * 2 * ffn / 4;
    const float4 ga = sum_splits<4>(g4, stride, splits), gb = sum_splits<4>(g4 + 1, stride, splits);
    const float4 ua = sum_splits<4>(u4, stride, splits), ub = sum_splits<4>(u4 + 1, stride, splits);
    const float g[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
    const float u[8] = {ua.x, ua.y, ua.z, ua.w, ub.x, ub.y, ub.z, ub.w};
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = g[e] / (1.0f + expf(-g[e])) * u[e];
    store_chunk(dst, lo, v);
  }
}

// ---- argmax per slot (decoder.zig:290-301: strict >, first index wins) ----

__global__ void __launch_bounds__(1024) streams_argmax_kernel(const StreamsStep P) {
  pdl_wait_and_trigger();
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const uint32_t s = blockIdx.x;
  if (!P.desc[s].active) return;
  const uint32_t vocab = P.model->vocab;
  const float* row = P.logits + size_t(s) * vocab;
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  // Eight independent loads per thread per round; a thread's indices ascend
  // within and across rounds, so strict > keeps its first maximum.
  constexpr uint32_t kUnroll = 8;
  for (uint32_t i0 = threadIdx.x; i0 < vocab; i0 += kUnroll * blockDim.x) {
    float v[kUnroll];
#pragma unroll
    for (uint32_t r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * blockDim.x;
      // decoder.zig:290-301: a NaN logit 0 wins (ranked +inf), other NaNs lose every comparison.
      const float x = i < vocab ? row[i] : -INFINITY;
      v[r] = (i == 0 && x != x) ? __int_as_float(0x7F800000) : x;
    }
#pragma unroll
    for (uint32_t r = 0; r < kUnroll; ++r) {
      const uint32_t i = i0 + r * blockDim.x;
      if (i < vocab && (v[r] > bv || (v[r] == bv && i < bi))) {
        bv = v[r];
        bi = i;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x / 32] = bv;
    si[threadIdx.x / 32] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (uint32_t w = 1; w < blockDim.x / 32; ++w) {
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) {
        bv = sv[w];
        bi = si[w];
      }
    }
    P.tokens[s] = bi == 0xFFFFFFFFu ? 0u : bi;
  }
}

// After a step: every active slot's next input is its argmax at the next
// position; the tokens also go to row `*counter` of `history`.
__global__ void streams_advance_kernel(const StreamsStep P, uint32_t* history, uint32_t* counter, uint32_t rows) {
  pdl_wait_and_trigger();
  const uint32_t s = threadIdx.x;
  const uint32_t step = *counter;
  __syncthreads();
  if (s < kMaxStreams) {
    SlotStep* d = const_cast<SlotStep*>(P.desc) + s;
    const uint32_t t = P.tokens[s];
    if (d->active) {
      d->position += 1;
      d->token = static_cast<int32_t>(t);
      d->audio_row = -1;
    }
    if (history && step < rows) history[size_t(step) * kMaxStreams + s] = t;
  }
  if (s == 0) *counter = step + 1;
}

}  // namespace

int launch_streams_advance(const StreamsStep& P, uint32_t* history, uint32_t* counter, uint32_t rows, void* stream) {
  return static_cast<int>(
      launch_pdl(streams_advance_kernel, dim3(1), dim3(kMaxStreams), 0, static_cast<cudaStream_t>(stream), P, history,
                 counter, rows));
}

int prepare_stream_kernels() {
  return static_cast<int>(cudaFuncSetAttribute(streams_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sizeof(AttnSmem))));
}

int launch_streams_norm(const StreamsStep& P, int input_mode, const float* weight, const float* parts, uint32_t splits,
                        void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return static_cast<int>(launch_pdl(input_mode ? streams_norm_kernel<1> : streams_norm_kernel<0>, dim3(kMaxStreams),
                                     dim3(kNormThreads), 0, st, P, weight, parts, splits));
}

int launch_streams_qkv(const StreamsStep& P, uint32_t layer, uint32_t splits, uint32_t kv_heads, void* stream) {
  return static_cast<int>(launch_pdl(streams_qkv_kernel, dim3(kv_heads, kMaxStreams), dim3(256), 0,
                                     static_cast<cudaStream_t>(stream), P, layer, splits));
}

int launch_streams_attention(const StreamsStep& P, const KvMaps4& maps, uint32_t layer, int grid, void* stream) {
  const int smem = static_cast<int>(sizeof(AttnSmem));
  return static_cast<int>(launch_pdl(streams_attention_kernel, dim3(grid), dim3(kAttnConsumers + 32), smem,
                                     static_cast<cudaStream_t>(stream), P, maps, layer));
}

int launch_streams_swiglu(const StreamsStep& P, uint32_t splits, void* stream) {
  return static_cast<int>(
      launch_pdl(streams_swiglu_kernel, dim3(592), dim3(256), 0, static_cast<cudaStream_t>(stream), P, splits));
}

int launch_streams_argmax(const StreamsStep& P, void* stream) {
  return static_cast<int>(
      launch_pdl(streams_argmax_kernel, dim3(kMaxStreams), dim3(1024), 0, static_cast<cudaStream_t>(stream), P));
}

}  // namespace qwc

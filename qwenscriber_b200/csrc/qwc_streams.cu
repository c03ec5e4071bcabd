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
          } else if (e.format == kFormatQ5) {
            const uint8_t* grp = crow + (k / kGroup) * 40u;
#pragma unroll
            for (int t = 0; t < 4; ++t) c[t] = static_cast<float>(q5_code(grp, (k + t) % kGroup));
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
// flight. At the end of a (slot, head) segment each consumer warp leaves its
// state (o[2][128], max and sum of both query heads) in one of two
// shared-memory buffers and goes on with the next segment; a merge warp
// combines the eight states (flash-decode rescale) and writes either the
// attention output (the segment is the whole head) or one partial per query
// head, and the CTA whose partial completes the head's chunk count combines
// the partials. Consumer warps never wait for one another.
//
// The products run on the tensor cores (mma.sync m16n8k16, f16 operands, f32
// accumulation). Codes enter as exact f16 values code - 128 (a byte permute
// against 0x64 and one f16 subtraction). Queries and the value weights
// (probability times the value group's scale) enter as f16 pairs hi + lo,
// which carry 22 bits of each f32. Warps 0-3 take the even chunks of the CTA's
// range and warps 4-7 the odd ones; within a chunk warp w takes positions
// 16 (w % 4) .. 16 (w % 4) + 15. Code boxes land with the 128-byte swizzle.

constexpr uint32_t kTK = 0;                                    // [64][128] key codes (128-byte swizzle)
constexpr uint32_t kTV = kTK + kAttnChunk * kHeadDim;          // [64][128] value codes (128-byte swizzle)
constexpr uint32_t kTKS = kTV + kAttnChunk * kHeadDim;         // [64][16 B] key scales (4 kv heads)
constexpr uint32_t kTVS = kTKS + kAttnChunk * 16;              // [64][16 B] value scales
constexpr uint32_t kTileBytes = kTVS + kAttnChunk * 16;
constexpr int kAttnSlots = 8;
constexpr int kAttnConsumers = 256;
constexpr float kWeightScale = 4096.0f;
constexpr uint32_t kPartFloats = kStreamsPartFloats;  // a warp's state: max[2], sum[2], o[2][128]
constexpr uint32_t kPartStride = kHeadDim + 4;          // a CTA partial row: o[128], max, sum, pad
constexpr int kAttnThreads = kAttnConsumers + 64;       // + the producer warp (8) and the merge warp (9)
constexpr uint32_t kSegBufs = 4;                        // segment-state buffers between consumers and the merge warp  // value weights are f16 pairs of 2^12 p s (kept off the f16 subnormals)
static_assert(kTV % 1024 == 0 && kTKS % 128 == 0 && kTVS % 128 == 0 && kTileBytes % 1024 == 0,
              "swizzled code boxes start on 1024-byte boundaries");

struct SegState {
  uint32_t s, h, first, count, chunks;
};

struct __align__(1024) AttnSmem {
  uint8_t ring[kAttnSlots][kTileBytes];
  alignas(16) float wstate[kSegBufs][8][kPartFloats];  // consumer warps' segment states, a ring of buffers
  SegState seg[kSegBufs];
  alignas(8) uint64_t wfull[kSegBufs];   // eight consumer warps left their states
  alignas(8) uint64_t wempty[kSegBufs];  // the merge warp is done with the buffer
  uint32_t prefix[kMaxStreams + 1];
  uint32_t pos[kMaxStreams];    // each column's newest position
  uint32_t cache[kMaxStreams];  // each column's cache slot
  uint32_t flag;
  alignas(8) uint64_t full[kAttnSlots];
  alignas(8) uint64_t empty[kAttnSlots];
};
constexpr size_t kAttnSmemBytes = sizeof(AttnSmem) + 1024;  // + alignment of the dynamic window

__device__ __forceinline__ void tma_load_4d(void* dst, const void* map, int32_t x, int32_t y, int32_t z, int32_t w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled box.
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) { return row * 128u + ((chunk ^ (row & 7u)) << 4); }

// Bytes b0, b1 of `w` as the f16 pair (b0 - 128, b1 - 128) (sel 0x4140), or
// bytes b2, b3 (sel 0x4342): 0x64 above a byte is the f16 1024 + byte.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t codes_f16x2(uint32_t w) {
  const uint32_t h = __byte_perm(w, 0x64646464u, SEL);
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));  // - (1024 + 128)
  return r;
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// d += a * b, m16n8k16, A row-major f16, B column-major f16, f32 accumulators.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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

__global__ void __launch_bounds__(kAttnThreads, 1) streams_attention_kernel(const StreamsStep P,
                                                                               const __grid_constant__ KvMaps4 maps,
                                                                               uint32_t layer) {
  // Programmatic dependent launch, split: the next kernel may start its
  // prologue at once, but this one waits for its predecessor (streams_qkv,
  // which appends this step's rows and rotates the queries) only where it
  // reads what that kernel writes. The slot descriptors and every cache row
  // before a column's last chunk are older than the predecessor.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(1024) uint8_t attn_smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(attn_smem_raw) & 1023u)) & 1023u;
  AttnSmem* a = reinterpret_cast<AttnSmem*>(attn_smem_raw + pad);
  const DevModel& m = *P.model;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const uint32_t qw = m.q_heads * kHeadDim;
  const uint32_t kv_heads = m.kv_heads;
  if (tid == 0) {
    for (int i = 0; i < kAttnSlots; ++i) {
      mbar_init(&a->full[i], 1);
      mbar_init(&a->empty[i], 4);  // the four warps that take the chunk
    }
    for (uint32_t i = 0; i < kSegBufs; ++i) {
      mbar_init(&a->wfull[i], 8);
      mbar_init(&a->wempty[i], 1);
    }
    fence_mbar_init();
  }
  // Unit prefix over the 64 columns: one column per thread of warps 0-1,
  // an inclusive scan within each warp, then warp 1 adds warp 0's total.
  static_assert(kMaxStreams == 64, "the prologue scans 64 columns with two warps");
  if (tid < 64) {
    const SlotStep d = P.desc[tid];
    const uint32_t units = d.active ? kv_heads * (static_cast<uint32_t>(d.position) / kAttnChunk + 1) : 0u;
    a->pos[tid] = static_cast<uint32_t>(d.position);
    a->cache[tid] = static_cast<uint32_t>(d.cache);
    uint32_t inc = units;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += v;
    }
    a->prefix[tid + 1] = inc;  // warp 1's values get warp 0's total below
    if (tid == 0) a->prefix[0] = 0;
  }
  __syncthreads();
  if (tid >= 32 && tid < 64) a->prefix[tid + 1] += a->prefix[32];
  __syncthreads();
  const uint32_t total = a->prefix[kMaxStreams];
  const uint32_t u0 = static_cast<uint32_t>((uint64_t(total) * blockIdx.x) / gridDim.x);
  const uint32_t u1 = static_cast<uint32_t>((uint64_t(total) * (blockIdx.x + 1)) / gridDim.x);

  if (warp == 8) {
    // ---- producer: TMA boxes of units u0..u1 into the ring ----
    if (lane == 0) {
      uint32_t it = 0;
      bool waited = false;
      UnitPos up = unit_pos(a, P, kv_heads, u0);
      for (uint32_t u = u0; u < u1; ++u, ++it, up = next_unit(a, kv_heads, up)) {
        if (!waited && up.ch + 1 == up.chunks) {  // a last chunk holds rows the predecessor wrote
          asm volatile("griddepcontrol.wait;" ::: "memory");
          waited = true;
        }
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

  if (warp == 9) {
    // ---- merge warp: the segments of u0..u1 in order ----
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t qw4 = qw;
    uint32_t nseg = 0;
    auto merge = [&]() {
      const uint32_t b = nseg % kSegBufs;
      const bool ready = mbar_wait_bounded(&a->wfull[b], (nseg / kSegBufs) & 1u, P.error, P.timeout_ns, 103);
      SegState sg = a->seg[b];
      if (!ready || sg.s >= kMaxStreams || sg.h >= kv_heads || sg.first >= P.max_chunks || sg.chunks > P.max_chunks ||
          sg.count > sg.chunks) {
        // Only a wait that gave up leaves a descriptor this kernel did not
        // write: record it and emit nothing for the segment.
        atomicCAS(P.error, 0, 105);
        __syncwarp();
        if (lane == 0) mbar_arrive(&a->wempty[b]);
        ++nseg;
        return;
      }
      // Lane l: dims 4 l .. 4 l + 3 of query heads 2 h and 2 h + 1.
      float mh[2], lh[2];
      float4 oh[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float mall = -INFINITY;
#pragma unroll
        for (int w = 0; w < 8; ++w) mall = fmaxf(mall, a->wstate[b][w][hh]);
        float l = 0.0f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < 8; ++w) {
          const float mw = a->wstate[b][w][hh];
          if (mw == -INFINITY) continue;
          const float f = __expf(mw - mall);
          const float4 v = *reinterpret_cast<const float4*>(&a->wstate[b][w][4 + hh * kHeadDim + 4 * lane]);
          o = make_float4(fmaf(v.x, f, o.x), fmaf(v.y, f, o.y), fmaf(v.z, f, o.z), fmaf(v.w, f, o.w));
          l = fmaf(a->wstate[b][w][2 + hh], f, l);
        }
        mh[hh] = mall;
        lh[hh] = l;
        oh[hh] = o;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&a->wempty[b]);  // the states are read
      __half* xq = static_cast<__half*>(P.xb_q) + size_t(sg.s) * qw4;
      const size_t xq_lo = size_t(kMaxStreams) * qw4;
      auto emit = [&](int hh, float4 o, float l) {
        const float inv = 1.0f / l;
        const float ov[4] = {o.x * inv, o.y * inv, o.z * inv, o.w * inv};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t col = (2 * sg.h + hh) * kHeadDim + 4u * lane + e;
          store_one(xq + ((col & ~7u) | chunk_slot(col & 7u)), xq_lo, ov[e]);
        }
      };
      if (sg.count == sg.chunks) {
        emit(0, oh[0], lh[0]);
        emit(1, oh[1], lh[1]);
      } else {
        // One partial row per query head at the segment's first chunk; a
        // non-NaN max marks the chunk as a segment start.
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float* row = P.attn_part + ((size_t(sg.s) * m.q_heads + 2 * sg.h + hh) * P.max_chunks + sg.first) * kPartStride;
          *reinterpret_cast<float4*>(row + 4 * lane) = oh[hh];
          if (lane == 0) {
            row[kHeadDim] = mh[hh];
            row[kHeadDim + 1] = lh[hh];
          }
        }
        // Acquire-release counter: __syncwarp orders the lanes' partial
        // stores before lane 0's release; the last arriver's acquire comes
        // before its lanes' loads of the other CTAs' partials.
        __syncwarp();
        uint32_t* counter = P.attn_count + size_t(sg.s) * kv_heads + sg.h;
        uint32_t last = 0;
        if (lane == 0) last = (atom_add_acq_rel(counter, sg.count) + sg.count == sg.chunks) ? 1u : 0u;
        last = __shfl_sync(0xffffffffu, last, 0);
        __syncwarp();
        if (last) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float* base = P.attn_part + (size_t(sg.s) * m.q_heads + 2 * sg.h + hh) * P.max_chunks * kPartStride;
            float mx = -INFINITY, l = 0.0f;
            float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
            for (uint32_t c0 = 0; c0 < sg.chunks; c0 += 8) {
              float pm[8], pl[8];
              float4 po[8];
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                pm[q] = __int_as_float(-1);
                pl[q] = 0.0f;
                po[q] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (c0 + q < sg.chunks) {
                  const float* src = base + size_t(c0 + q) * kPartStride;
                  pm[q] = ld_cg(src + kHeadDim);
                  pl[q] = ld_cg(src + kHeadDim + 1);
                  po[q] = __ldcg(reinterpret_cast<const float4*>(src) + lane);
                }
              }
              float bm = mx;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                if (pm[q] == pm[q]) bm = fmaxf(bm, pm[q]);
              }
              const float rs = (mx == -INFINITY) ? 0.0f : __expf(mx - bm);
              o = make_float4(o.x * rs, o.y * rs, o.z * rs, o.w * rs);
              l *= rs;
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                if (pm[q] == pm[q] && pm[q] != -INFINITY) {
                  const float f = __expf(pm[q] - bm);
                  o = make_float4(fmaf(po[q].x, f, o.x), fmaf(po[q].y, f, o.y), fmaf(po[q].z, f, o.z),
                                  fmaf(po[q].w, f, o.w));
                  l = fmaf(pl[q], f, l);
                }
              }
              mx = bm;
            }
            emit(hh, o, l);
            // Reset for the next step: partial maxima back to NaN.
            for (uint32_t c = lane; c < sg.chunks; c += 32) base[size_t(c) * kPartStride + kHeadDim] = __int_as_float(-1);
          }
          if (lane == 0) *counter = 0;
        }
      }
      ++nseg;
    };
    UnitPos cur{0xFFFFFFFFu, 0xFFFFFFFFu, 0, 0, 0};
    UnitPos up = unit_pos(a, P, kv_heads, u0);
    for (uint32_t u = u0; u < u1; ++u, up = next_unit(a, kv_heads, up)) {
      if (up.s != cur.s || up.h != cur.h) {
        if (cur.s != 0xFFFFFFFFu) merge();
        cur = up;
      }
    }
    if (cur.s != 0xFFFFFFFFu) merge();
    return;
  }

  // ---- consumers ----
  asm volatile("griddepcontrol.wait;" ::: "memory");  // queries, and the partial buffers other kernels use
  //
  // Lane L = 4 r + i. Scores: the m16n8k16 tile of warp w's 16 positions by
  // 16 dims; B columns are (head 0 hi, head 0 lo, head 1 hi, head 1 lo)
  // twice, so lane L ends up with head i & 1's scores of positions r and
  // r + 8. Within a 64-dim group g, lane i's 16 contiguous code bytes of a row
  // feed the four k-steps t (dims 64 g + 16 i + 4 t + 0..3); the query's B
  // fragments follow the same dim order. Values: A rows rho = 4 hl + 2 g + h
  // are the f16 hi (hl 0) / lo (hl 1) parts of head h's weights for value
  // group g at the warp's 16 positions; n-tile (c, j) has column n <-> dim
  // 32 c + 4 n + j, so the B fragment of lane L comes from one 4-byte word of
  // each of four rows.
  const uint32_t grp = static_cast<uint32_t>(warp) >> 2, wq = static_cast<uint32_t>(warp) & 3u;
  const uint32_t r = static_cast<uint32_t>(lane) >> 2, i = static_cast<uint32_t>(lane) & 3u;
  const uint32_t hrow = r & 1u, grow = (r >> 1) & 1u, hl = r >> 2;  // value-row head, group, hi/lo
  const uint32_t prow0 = 16u * wq + r, prow1 = prow0 + 8u;           // tile rows of this lane's scores
  const uint32_t va = 16u * wq + 2u * i;                              // tile rows va, va+1, va+8, va+9 (values)
  bool ok = true;
  float m_run = -INFINITY, l_run = 0.0f;  // head hq
  float acc[16][4];
  uint32_t qb[8][2];
  UnitPos cur{0xFFFFFFFFu, 0xFFFFFFFFu, 0, 0, 0};

  // At a segment's end: this warp's state into buffer (segment index mod
  // kSegBufs) for the merge warp; that buffer's previous segment must have
  // been merged.
  uint32_t nseg = 0, seg_first = 0, seg_count = 0;
  auto flush = [&]() {
    const uint32_t b = nseg % kSegBufs;
    if (nseg >= kSegBufs) mbar_wait_bounded(&a->wempty[b], ((nseg / kSegBufs) - 1) & 1u, P.error, P.timeout_ns, 104);
    float* st = a->wstate[b][warp];
    // hi + lo value rows (lanes r and r + 4 hold the same head and group),
    // the 2^12 weight scale removed.
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const float o0 = acc[nt][0] + __shfl_xor_sync(0xffffffffu, acc[nt][0], 16);
      const float o1 = acc[nt][1] + __shfl_xor_sync(0xffffffffu, acc[nt][1], 16);
      const uint32_t c = static_cast<uint32_t>(nt) >> 2, j = static_cast<uint32_t>(nt) & 3u;
      if (hl == 0 && (c >> 1) == grow) {
        st[4 + hrow * kHeadDim + 32u * c + 8u * i + j] = o0 * (1.0f / kWeightScale);
        st[4 + hrow * kHeadDim + 32u * c + 8u * i + 4u + j] = o1 * (1.0f / kWeightScale);
      }
    }
    if (lane < 2) {
      st[lane] = m_run;
      st[2 + lane] = l_run;
    }
    if (warp == 0 && lane == 0) a->seg[b] = SegState{cur.s, cur.h, seg_first, seg_count, cur.chunks};
    __syncwarp();
    if (lane == 0) mbar_arrive(&a->wfull[b]);
    ++nseg;
  };

  const float scaling = m.attn_scaling;
  // Work items: two consecutive chunks of one segment (or a segment's last
  // odd chunk alone); the two warp groups take alternate items. A warp's
  // latency chain (score MMAs, the softmax shuffles, value MMAs) then covers
  // 32 positions instead of 16.
  uint32_t it = 0, item = 0;
  UnitPos up = unit_pos(a, P, kv_heads, u0);
  for (uint32_t u = u0; u < u1;) {
    if (up.s != cur.s || up.h != cur.h) {
      if (cur.s != 0xFFFFFFFFu) flush();  // ends with every warp past the previous segment
      cur = up;
      seg_first = up.ch;
      seg_count = 0;
      m_run = -INFINITY;
      l_run = 0.0f;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
      // The query B fragments: column n = r is head (r >> 1) & 1, hi (r even) or lo part.
      const float* qsrc = P.qrot + size_t(up.s) * qw + (2 * up.h + ((r >> 1) & 1u)) * kHeadDim;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t g = static_cast<uint32_t>(kk) >> 2, t = static_cast<uint32_t>(kk) & 3u;
        const float4 qv = __ldcg(reinterpret_cast<const float4*>(qsrc + 64u * g + 16u * i + 4u * t));
        const float q4[4] = {qv.x, qv.y, qv.z, qv.w};
        float part[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float hi = __half2float(__float2half_rn(q4[e]));
          part[e] = (r & 1u) ? q4[e] - hi : hi;
        }
        qb[kk][0] = pack_f16x2(part[0], part[1]);
        qb[kk][1] = pack_f16x2(part[2], part[3]);
      }
    }
    UnitPos nx = up;
    bool two = false;
    if (u + 1 < u1) {
      nx = next_unit(a, kv_heads, up);
      two = nx.s == up.s && nx.h == up.h;
    }
    const uint32_t nt_units = two ? 2u : 1u;
    seg_count += nt_units;
    if ((item & 1u) == grp) {
      const uint8_t* tiles[2];
      uint32_t slots[2];
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        const uint32_t itt = it + (tt == 1 && two ? 1u : 0u);
        slots[tt] = itt % kAttnSlots;
        tiles[tt] = a->ring[slots[tt]];
        if ((tt == 0 || two) && ok &&
            !mbar_wait_bounded(&a->full[slots[tt]], (itt / kAttnSlots) & 1u, P.error, P.timeout_ns, 101)) {
          ok = false;
        }
      }
      const uint32_t newest = a->pos[up.s];
      // ---- scores: q . k for positions prow0, prow1 of each tile (head hq) ----
      float sc[2][2];
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        sc[tt][0] = sc[tt][1] = -INFINITY;
        if (tt == 1 && !two) continue;
        const uint8_t* tile = tiles[tt];
        const uint32_t base_pos = (up.ch + tt) * kAttnChunk;
        float d[2][4];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          d[g][0] = d[g][1] = d[g][2] = d[g][3] = 0.0f;
          const uint4 k0 = *reinterpret_cast<const uint4*>(tile + kTK + swz(prow0, 4u * g + i));
          const uint4 k1 = *reinterpret_cast<const uint4*>(tile + kTK + swz(prow1, 4u * g + i));
          const uint32_t w0[4] = {k0.x, k0.y, k0.z, k0.w};
          const uint32_t w1[4] = {k1.x, k1.y, k1.z, k1.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            mma16816(d[g], codes_f16x2<0x4140>(w0[t]), codes_f16x2<0x4140>(w1[t]), codes_f16x2<0x4342>(w0[t]),
                     codes_f16x2<0x4342>(w1[t]), qb[4 * g + t][0], qb[4 * g + t][1]);
          }
        }
        const uint32_t so = (up.h % 4u) * 4u;
        const uint32_t ks0 = *reinterpret_cast<const uint32_t*>(tile + kTKS + prow0 * 16u + so);
        const uint32_t ks1 = *reinterpret_cast<const uint32_t*>(tile + kTKS + prow1 * 16u + so);
        const float s00 = f16_bits_to_f32_fast(ks0 & 0xFFFFu), s01 = f16_bits_to_f32_fast(ks0 >> 16);
        const float s10 = f16_bits_to_f32_fast(ks1 & 0xFFFFu), s11 = f16_bits_to_f32_fast(ks1 >> 16);
        const float t0 = fmaf(s00, d[0][0] + d[0][1], s01 * (d[1][0] + d[1][1]));
        const float t1 = fmaf(s10, d[0][2] + d[0][3], s11 * (d[1][2] + d[1][3]));
        sc[tt][0] = (ok && base_pos + prow0 <= newest) ? scaling * t0 : -INFINITY;
        sc[tt][1] = (ok && base_pos + prow1 <= newest) ? scaling * t1 : -INFINITY;
      }
      // ---- online softmax over the warp's positions of the item (math.zig:77-93) ----
      float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m_run, mx);
      const float resc = (m_run == -INFINITY) ? 0.0f : __expf(m_run - m_new);
      float pp[2][2];
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) pp[tt][e] = sc[tt][e] == -INFINITY ? 0.0f : __expf(sc[tt][e] - m_new);
      }
      float ps = (pp[0][0] + pp[0][1]) + (pp[1][0] + pp[1][1]);
      ps += __shfl_xor_sync(0xffffffffu, ps, 4);
      ps += __shfl_xor_sync(0xffffffffu, ps, 8);
      ps += __shfl_xor_sync(0xffffffffu, ps, 16);
      l_run = fmaf(l_run, resc, ps);
      m_run = m_new;
      // Accumulators of value rows of head hrow: rescale when its maximum moved.
      const float f_h0 = __shfl_sync(0xffffffffu, resc, 0), f_h1 = __shfl_sync(0xffffffffu, resc, 1);
      const float f_row = hrow ? f_h1 : f_h0;
      if (__any_sync(0xffffffffu, f_row != 1.0f)) {
#pragma unroll
        for (int n = 0; n < 16; ++n) {
          acc[n][0] *= f_row;
          acc[n][1] *= f_row;
        }
      }
#pragma unroll
      for (int tt = 0; tt < 2; ++tt) {
        if (tt == 1 && !two) continue;
        const uint8_t* tile = tiles[tt];
        // ---- value weights: A rows (head hrow, group grow, hi/lo hl) at warp positions 2i, 2i+1, 2i+8, 2i+9 ----
        uint32_t pa0, pa2;
        {
          const float a00 = __shfl_sync(0xffffffffu, pp[tt][0], 8 * i + hrow);      // position 2i
          const float a10 = __shfl_sync(0xffffffffu, pp[tt][1], 8 * i + hrow);      // position 2i + 8
          const float a01 = __shfl_sync(0xffffffffu, pp[tt][0], 8 * i + 4 + hrow);  // position 2i + 1
          const float a11 = __shfl_sync(0xffffffffu, pp[tt][1], 8 * i + 4 + hrow);  // position 2i + 9
          const uint32_t so = (up.h % 4u) * 4u + grow * 2u;
          const float pw[4] = {a00, a01, a10, a11};
          const uint32_t rows[4] = {va, va + 1u, va + 8u, va + 9u};
          float wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float sv =
                f16_bits_to_f32_fast(*reinterpret_cast<const uint16_t*>(tile + kTVS + rows[e] * 16u + so));
            const float x = pw[e] > 0.0f ? pw[e] * sv * kWeightScale : 0.0f;
            const float xh = __half2float(__float2half_rn(x));
            wv[e] = hl ? x - xh : xh;
          }
          pa0 = pack_f16x2(wv[0], wv[1]);
          pa2 = pack_f16x2(wv[2], wv[3]);
        }
        // ---- values: acc[(c, j)] += weights x (code - 128) ----
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t chunk = 2u * c + (r >> 2), off = 4u * (r & 3u);
          const uint32_t wa = *reinterpret_cast<const uint32_t*>(tile + kTV + swz(va, chunk) + off);
          const uint32_t wb = *reinterpret_cast<const uint32_t*>(tile + kTV + swz(va + 1u, chunk) + off);
          const uint32_t wc = *reinterpret_cast<const uint32_t*>(tile + kTV + swz(va + 8u, chunk) + off);
          const uint32_t wd = *reinterpret_cast<const uint32_t*>(tile + kTV + swz(va + 9u, chunk) + off);
          const uint32_t ab01 = __byte_perm(wa, wb, 0x5140), ab23 = __byte_perm(wa, wb, 0x7362);
          const uint32_t cd01 = __byte_perm(wc, wd, 0x5140), cd23 = __byte_perm(wc, wd, 0x7362);
          mma16816(acc[4 * c + 0], pa0, 0u, pa2, 0u, codes_f16x2<0x4140>(ab01), codes_f16x2<0x4140>(cd01));
          mma16816(acc[4 * c + 1], pa0, 0u, pa2, 0u, codes_f16x2<0x4342>(ab01), codes_f16x2<0x4342>(cd01));
          mma16816(acc[4 * c + 2], pa0, 0u, pa2, 0u, codes_f16x2<0x4140>(ab23), codes_f16x2<0x4140>(cd23));
          mma16816(acc[4 * c + 3], pa0, 0u, pa2, 0u, codes_f16x2<0x4342>(ab23), codes_f16x2<0x4342>(cd23));
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&a->empty[slots[0]]);  // this warp is done with the item's chunks
        if (two) mbar_arrive(&a->empty[slots[1]]);
      }
    }
    ++item;
    u += nt_units;
    it += nt_units;
    up = two ? next_unit(a, kv_heads, nx) : nx;
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
                                               static_cast<int>(kAttnSmemBytes)));
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
  const int smem = static_cast<int>(kAttnSmemBytes);
  return static_cast<int>(launch_pdl(streams_attention_kernel, dim3(grid), dim3(kAttnThreads), smem,
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

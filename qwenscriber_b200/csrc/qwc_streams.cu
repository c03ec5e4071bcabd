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

constexpr int kNormThreads = 256;
constexpr int kNormPer = kHiddenMax / kNormThreads;

// Position of element e (0..7) of a chunk in the activation layout.
__device__ __forceinline__ uint32_t chunk_slot(uint32_t e) { return ((e & 3u) << 1) | (e >> 2); }

__device__ __forceinline__ float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = v;
  __syncthreads();
  float t = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  __syncthreads();
  return t;
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

template <int kInput>
__global__ void __launch_bounds__(kNormThreads) streams_norm_kernel(const StreamsStep P, const float* weight,
                                                                    const float* parts, uint32_t splits) {
  __shared__ float xs[kHiddenMax];
  __shared__ float red[8];
  const DevModel& m = *P.model;
  const uint32_t s = blockIdx.x;
  const uint32_t hidden = m.hidden;
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
  float* h = P.hidden + size_t(s) * hidden;
  float v[kNormPer];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const uint32_t k = threadIdx.x + i * kNormThreads;
    float x = 0.0f;
    if (k < hidden) {
      if (kInput) {
        if (d.audio_row >= 0) {
          x = P.audio[s][size_t(d.audio_row) * hidden + k];
        } else {
          // embeddingRow, quantized branch (decoder.zig:346-376, quant.zig:348-364).
          const DevMat& e = m.embed;
          const float scale = f16_bits_to_f32(
              reinterpret_cast<const uint16_t*>(e.scales + size_t(d.token) * e.scale_row)[k / kGroup]);
          const uint8_t* crow = e.codes + size_t(d.token) * e.code_row;
          int code;
          if (e.format == kFormatQ4) {
            const uint8_t b = crow[k / 2];
            code = static_cast<int>((k & 1u) ? (b >> 4) : (b & 0x0F)) - 8;
          } else {
            code = static_cast<int>(crow[k]) - 128;
          }
          x = static_cast<float>(code) * scale;
        }
      } else {
        // The projection is the sum of its split-K partials, then the
        // residual add (kernels.zig:221-230).
        float y = parts[size_t(s) * hidden + k];
        for (uint32_t sp = 1; sp < splits; ++sp) y += parts[(size_t(sp) * kMaxStreams + s) * hidden + k];
        x = h[k] + y;
      }
      h[k] = x;
      ss = fmaf(x, x, ss);
    }
    v[i] = x;
  }
  const float total = block_sum_256(ss, red);
  const float inv = 1.0f / sqrtf(total / static_cast<float>(hidden) + m.eps);
#pragma unroll
  for (int i = 0; i < kNormPer; ++i) {
    const uint32_t k = threadIdx.x + i * kNormThreads;
    if (k < hidden) xs[k] = v[i] * inv * weight[k];
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
  float qraw = 0.0f, kvraw = 0.0f;
  for (uint32_t sp = 0; sp < splits; ++sp) {
    const float* row = P.part0 + (size_t(sp) * kMaxStreams + s) * rows;
    qraw += row[(2 * h + j) * kHeadDim + dd];
    kvraw += row[qw + j * kvw + h * kHeadDim + dd];
  }
  const DevLayer& L = m.layers[layer];
  const float ss = warp_sum(qraw * qraw), kss = warp_sum(kvraw * kvraw);
  if (lane == 0) {
    red[warp] = ss;
    red[8 + warp] = kss;
  }
  __syncthreads();
  const int w0 = j * 4;
  const float total = ((red[w0] + red[w0 + 1]) + red[w0 + 2]) + red[w0 + 3];
  const float inv = 1.0f / sqrtf(total / static_cast<float>(kHeadDim) + m.eps);
  tq[j][dd] = qraw * inv * L.q_norm[dd];
  if (j == 0) {
    const float kt = ((red[8] + red[9]) + red[10]) + red[11];
    const float kinv = 1.0f / sqrtf(kt / static_cast<float>(kHeadDim) + m.eps);
    tk[dd] = kvraw * kinv * L.k_norm[dd];
  }
  __syncthreads();
  const int pair = dd % (kHeadDim / 2);
  const float* cos_row = m.rope_cos + size_t(d.position) * (kHeadDim / 2);
  const float* sin_row = m.rope_sin + size_t(d.position) * (kHeadDim / 2);
  const float cs = cos_row[pair], sn = sin_row[pair];
  {
    const float lo = tq[j][pair], hi = tq[j][pair + kHeadDim / 2];
    P.qrot[size_t(s) * qw + (2 * h + j) * kHeadDim + dd] = dd < kHeadDim / 2 ? lo * cs - hi * sn : hi * cs + lo * sn;
  }
  float val = kvraw;
  if (j == 0) {
    const float lo = tk[pair], hi = tk[pair + kHeadDim / 2];
    val = dd < kHeadDim / 2 ? lo * cs - hi * sn : hi * cs + lo * sn;
  }
  // q8 row (quant.zig:197-227): groups of 64 values, two warps each.
  const float amax = warp_max(fabsf(val));
  __syncthreads();
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  const int gw = (warp / 2) * 2;
  const float gmax = fmaxf(red[gw], red[gw + 1]);
  const __half sh = __float2half_rn(gmax / 128.0f);
  const uint8_t code = q8_code(val, __half2float(sh));
  uint8_t* plane = (j == 0 ? P.k_cache : P.v_cache) + size_t(s) * m.cache_stream_stride + size_t(layer) * m.cache_layer_stride;
  plane[m.cache_scales_bytes + size_t(d.position) * kvw + h * kHeadDim + dd] = code;
  if ((dd % kGroup) == 0) {
    reinterpret_cast<uint16_t*>(plane + size_t(d.position) * (kvw / kGroup) * 2)[h * 2 + dd / kGroup] =
        __half_as_ushort(sh);
  }
}

// ---- split-K decode attention over every slot (kernels.zig:697-767) ----

constexpr uint32_t kTK = 0;                                    // [64][128] key codes
constexpr uint32_t kTV = kTK + kAttnChunk * kHeadDim;          // [64][128] value codes
constexpr uint32_t kTKS = kTV + kAttnChunk * kHeadDim;         // [64][16 B] key scales (4 kv heads)
constexpr uint32_t kTVS = kTKS + kAttnChunk * 16;              // [64][16 B] value scales
constexpr uint32_t kTileBytes = kTVS + kAttnChunk * 16;
static_assert(kTV % 128 == 0 && kTKS % 128 == 0 && kTVS % 128 == 0, "TMA boxes land on 128-byte boundaries");

struct __align__(128) AttnTile {
  uint8_t tile[kTileBytes];
  alignas(16) float q[2][4][36];
  alignas(16) float prob[2][kAttnChunk];
  alignas(16) float lsum[2][8];
  alignas(16) float mx[2];
  alignas(16) float vpart[8][2][kHeadDim];
  alignas(16) float red[16];
  uint32_t prefix[kMaxStreams + 1];
  uint32_t flag;
  alignas(8) uint64_t bar;
};
static_assert(offsetof(AttnTile, vpart) % 16 == 0 && offsetof(AttnTile, q) % 16 == 0, "vector access alignment");

__device__ __forceinline__ void tma_load_4d(void* dst, const void* map, int32_t x, int32_t y, int32_t z, int32_t w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar))
      : "memory");
}

__global__ void __launch_bounds__(256) streams_attention_kernel(const StreamsStep P, const __grid_constant__ KvMaps4 maps,
                                                                uint32_t layer) {
  extern __shared__ __align__(128) uint8_t attn_smem_raw[];
  AttnTile* a = reinterpret_cast<AttnTile*>(attn_smem_raw);
  const DevModel& m = *P.model;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int j = tid / kHeadDim, dd = tid % kHeadDim;
  const uint32_t qw = m.q_heads * kHeadDim;
  if (tid == 0) {
    mbar_init(&a->bar, 1);
    fence_mbar_init();
    uint32_t acc = 0;
    for (uint32_t s = 0; s < kMaxStreams; ++s) {
      a->prefix[s] = acc;
      const SlotStep d = P.desc[s];
      if (d.active) acc += m.kv_heads * (d.position / kAttnChunk + 1);
    }
    a->prefix[kMaxStreams] = acc;
  }
  __syncthreads();
  const uint32_t total = a->prefix[kMaxStreams];
  uint32_t phase = 0;
  bool ok = true;
  for (uint32_t u = blockIdx.x; u < total; u += gridDim.x) {
    // Slot of unit u: the last s with prefix[s] <= u.
    uint32_t lo = 0, hi = kMaxStreams;
    while (hi - lo > 1) {
      const uint32_t mid = (lo + hi) / 2;
      if (a->prefix[mid] <= u) lo = mid; else hi = mid;
    }
    const uint32_t s = lo;
    const SlotStep d = P.desc[s];
    const uint32_t chunks = d.position / kAttnChunk + 1;
    const uint32_t r = u - a->prefix[s];
    const uint32_t h = r / chunks, ch = r % chunks;
    const uint32_t newest = d.position;
    if (tid == 0) {
      mbar_arrive_expect_tx(&a->bar, kTileBytes);
      const int32_t y = static_cast<int32_t>(ch * kAttnChunk), z = static_cast<int32_t>(layer),
                    w = static_cast<int32_t>(s);
      const int32_t xs = static_cast<int32_t>((h * 4u) & ~15u);
      tma_load_4d(a->tile + kTK, maps.k_codes, static_cast<int32_t>(h * kHeadDim), y, z, w, &a->bar);
      tma_load_4d(a->tile + kTV, maps.v_codes, static_cast<int32_t>(h * kHeadDim), y, z, w, &a->bar);
      tma_load_4d(a->tile + kTKS, maps.k_scales, xs, y, z, w, &a->bar);
      tma_load_4d(a->tile + kTVS, maps.v_scales, xs, y, z, w, &a->bar);
    }
    // Rotated queries 2h, 2h+1 (L2) while the tile lands.
    a->q[j][dd / 32][dd % 32] = P.qrot[size_t(s) * qw + (2 * h + j) * kHeadDim + dd];
    if (ok && !mbar_wait_bounded(&a->bar, phase, P.error, global_timer_ns() + P.timeout_ns, 101)) {
      ok = false;
      if (*reinterpret_cast<volatile int32_t*>(P.error) == 101 && tid == 0) {
        P.error[1] = static_cast<int32_t>(layer);
        P.error[2] = static_cast<int32_t>(u);
        P.error[3] = static_cast<int32_t>(s);
      }
    }
    if (__syncthreads_or(!ok)) {
      // A box never landed: wait once more (bounded) so no copy is still in
      // flight when the CTA exits, and stop.
      if (tid == 0) {
        const uint64_t deadline = global_timer_ns() + 1000000000ull;
        while (!mbar_try_wait(&a->bar, phase) && global_timer_ns() < deadline) {
        }
      }
      __syncthreads();
      return;
    }
    phase ^= 1u;
    // Scores: four lanes per position, the two lanes of a 64-value group add
    // their sums before the group scale (q8GroupDot, kernels.zig:636-661).
    const uint32_t rr = static_cast<uint32_t>(tid) / 4, qd = static_cast<uint32_t>(tid) % 4;
    const uint32_t pos = ch * kAttnChunk + rr;
    const bool valid = ok && pos <= newest;
    {
      const uint4* src = reinterpret_cast<const uint4*>(a->tile + kTK + rr * kHeadDim + qd * 32);
      const uint4 kw0 = src[0], kw1 = src[1];
      const uint32_t kbits = *reinterpret_cast<const uint16_t*>(a->tile + kTKS + rr * 16 + (h % 4) * 4 + (qd / 2) * 2);
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
      const float w0 = warp_max(sc0), w1 = warp_max(sc1);
      if (lane == 0) {
        a->red[warp] = w0;
        a->red[8 + warp] = w1;
      }
      __syncthreads();
      float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        m0 = fmaxf(m0, a->red[w]);
        m1 = fmaxf(m1, a->red[8 + w]);
      }
      const float p0 = valid ? expf(sc0 - m0) : 0.0f;
      const float p1 = valid ? expf(sc1 - m1) : 0.0f;
      if (qd == 0) {
        a->prob[0][rr] = p0;
        a->prob[1][rr] = p1;
      }
      const float l0 = warp_sum(qd == 0 ? p0 : 0.0f), l1 = warp_sum(qd == 0 ? p1 : 0.0f);
      if (lane == 0) {
        a->lsum[0][warp] = l0;
        a->lsum[1][warp] = l1;
      }
      if (tid == 0) {
        a->mx[0] = m0;
        a->mx[1] = m1;
      }
      __syncthreads();
    }
    // Values (q8GroupAccumulate, kernels.zig:665-688): lane = 4 dims, warp = 8 positions.
    {
      float acc[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
      const uint32_t grp = static_cast<uint32_t>(lane) / 16;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t q = warp * 8 + i;
        const uint32_t word = *reinterpret_cast<const uint32_t*>(a->tile + kTV + q * kHeadDim + 4 * lane);
        const uint32_t bits = *reinterpret_cast<const uint16_t*>(a->tile + kTVS + q * 16 + (h % 4) * 4 + grp * 2);
        const float scale = f16_bits_to_f32_fast(bits);
        const bool vq = ok && ch * kAttnChunk + q <= newest;
        const float sw0 = vq ? scale * a->prob[0][q] : 0.0f;
        const float sw1 = vq ? scale * a->prob[1][q] : 0.0f;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float cv = bits_f32(__byte_perm(word, kMagic, 0x7440 + t)) + kNegQ8;
          acc[0][t] = fmaf(cv, sw0, acc[0][t]);
          acc[1][t] = fmaf(cv, sw1, acc[1][t]);
        }
      }
      *reinterpret_cast<float4*>(&a->vpart[warp][0][4 * lane]) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
      *reinterpret_cast<float4*>(&a->vpart[warp][1][4 * lane]) = make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]);
    }
    __syncthreads();
    float o = 0.0f, l = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      o += a->vpart[w][j][dd];
      l += a->lsum[j][w];
    }
    const float mj = a->mx[j];
    __half* xq = static_cast<__half*>(P.xb_q) + size_t(s) * qw;
    const uint32_t col = (2 * h + j) * kHeadDim + dd;
    const uint32_t out_index = (col & ~7u) | chunk_slot(col & 7u);
    const size_t xq_lo = size_t(kMaxStreams) * qw;
    if (chunks == 1) {
      store_one(xq + out_index, xq_lo, o / l);
      __syncthreads();
      continue;
    }
    {
      float* dst = P.attn_part + ((size_t(s) * m.q_heads + 2 * h + j) * P.max_chunks + ch) * (kHeadDim + 2);
      dst[dd] = o;
      if (dd == 0) {
        dst[kHeadDim] = mj;
        dst[kHeadDim + 1] = l;
      }
    }
    __threadfence();
    __syncthreads();
    uint32_t* counter = P.attn_count + size_t(s) * m.kv_heads + h;
    if (tid == 0) {
      const uint32_t prev = atomicAdd(counter, 1u);
      a->flag = (prev == chunks - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (a->flag) {
      __threadfence();
      float mx = -INFINITY;
      o = 0.0f;
      l = 0.0f;
      const float* base = P.attn_part + (size_t(s) * m.q_heads + 2 * h + j) * P.max_chunks * (kHeadDim + 2);
      for (uint32_t q0 = 0; q0 < chunks; q0 += 8) {
        float pm[8], po[8], pl[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          pm[q] = -INFINITY;
          po[q] = 0.0f;
          pl[q] = 0.0f;
          if (q0 + q < chunks) {
            const float* src = base + size_t(q0 + q) * (kHeadDim + 2);
            pm[q] = ld_cg(src + kHeadDim);
            po[q] = ld_cg(src + dd);
            pl[q] = ld_cg(src + kHeadDim + 1);
          }
        }
        float bm = mx;
#pragma unroll
        for (int q = 0; q < 8; ++q) bm = fmaxf(bm, pm[q]);
        const float rescale = (mx == -INFINITY) ? 0.0f : expf(mx - bm);
        o *= rescale;
        l *= rescale;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float f = (pm[q] == -INFINITY) ? 0.0f : expf(pm[q] - bm);
          o = fmaf(po[q], f, o);
          l = fmaf(pl[q], f, l);
        }
        mx = bm;
      }
      store_one(xq + out_index, xq_lo, o / l);
      if (tid == 0) *counter = 0;
    }
    __syncthreads();
  }
}

// ---- SwiGLU (kernels.zig:233-239) into f16 activations ----

__global__ void streams_swiglu_kernel(const StreamsStep P, uint32_t splits) {
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
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const size_t idx = size_t(s) * 2 * ffn + c * 8 + e;
      float g = P.part0[idx], u = P.part0[idx + ffn];
      for (uint32_t sp = 1; sp < splits; ++sp) {
        g += P.part0[size_t(sp) * kMaxStreams * 2 * ffn + idx];
        u += P.part0[size_t(sp) * kMaxStreams * 2 * ffn + idx + ffn];
      }
      v[e] = g / (1.0f + expf(-g)) * u;
    }
    store_chunk(dst, lo, v);
  }
}

// ---- argmax per slot (decoder.zig:290-301: strict >, first index wins) ----

__global__ void __launch_bounds__(1024) streams_argmax_kernel(const StreamsStep P) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const uint32_t s = blockIdx.x;
  if (!P.desc[s].active) return;
  const uint32_t vocab = P.model->vocab;
  const float* row = P.logits + size_t(s) * vocab;
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = row[i];
    if (v > bv || (v == bv && i < bi)) {
      bv = v;
      bi = i;
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
  streams_advance_kernel<<<1, kMaxStreams, 0, static_cast<cudaStream_t>(stream)>>>(P, history, counter, rows);
  return static_cast<int>(cudaGetLastError());
}

int prepare_stream_kernels() {
  return static_cast<int>(cudaFuncSetAttribute(streams_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sizeof(AttnTile))));
}

int launch_streams_norm(const StreamsStep& P, int input_mode, const float* weight, const float* parts, uint32_t splits,
                        void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (input_mode) {
    streams_norm_kernel<1><<<kMaxStreams, kNormThreads, 0, st>>>(P, weight, parts, splits);
  } else {
    streams_norm_kernel<0><<<kMaxStreams, kNormThreads, 0, st>>>(P, weight, parts, splits);
  }
  return static_cast<int>(cudaGetLastError());
}

int launch_streams_qkv(const StreamsStep& P, uint32_t layer, uint32_t splits, uint32_t kv_heads, void* stream) {
  streams_qkv_kernel<<<dim3(kv_heads, kMaxStreams), 256, 0, static_cast<cudaStream_t>(stream)>>>(P, layer, splits);
  return static_cast<int>(cudaGetLastError());
}

int launch_streams_attention(const StreamsStep& P, const KvMaps4& maps, uint32_t layer, int grid, void* stream) {
  const int smem = static_cast<int>(sizeof(AttnTile));
  streams_attention_kernel<<<grid, 256, smem, static_cast<cudaStream_t>(stream)>>>(P, maps, layer);
  return static_cast<int>(cudaGetLastError());
}

int launch_streams_swiglu(const StreamsStep& P, uint32_t splits, void* stream) {
  streams_swiglu_kernel<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(P, splits);
  return static_cast<int>(cudaGetLastError());
}

int launch_streams_argmax(const StreamsStep& P, void* stream) {
  streams_argmax_kernel<<<kMaxStreams, 1024, 0, static_cast<cudaStream_t>(stream)>>>(P);
  return static_cast<int>(cudaGetLastError());
}

}  // namespace qwc

// qwc_audio.cu -- the audio tower and projector (Model.projectAudio,
// src/core/qwen3_asr/model.zig:445-744) on the device: every kernel of the
// tower except its GEMMs, which are the tensor-core GEMMs of qwc_gemm.cu
// (dense f16 weights for the convolutions, quantized weights for the rest).
//
// Data layout (one clip, `chunks` convolution chunks of chunk_frames mel
// frames, `steps` packed encoder steps):
//   conv planes   channel-last f32 [chunk][height][width][channel], so a
//                 convolution tap reads 8 consecutive input channels with
//                 two 16-byte loads;
//   GEMM inputs   f16 hi and lo rows per 64-column block (the layout of the
//                 GEMMs' activation boxes); the convolutions' K index is
//                 (tap, input channel) in natural order, the quantized GEMMs'
//                 K chunks of 8 are permuted [0 4 1 5 2 6 3 7];
//   tower rows    f32 [step][width] (the reference's encoder scratch).
//
// Parity: the first convolution, GELU (math.zig:46-66, with CUDA's expf) and
// the sinusoidal position rows follow the reference's order. The GEMM-shaped
// steps (convolutions 2 and 3, every projection) sum in another order with
// 22-bit activations, and the LayerNorm and attention reductions are trees,
// so the tower agrees with the reference to f32 rounding, not bit for bit.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "../../include/qwenscriber_cuda.h"
#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

constexpr uint32_t kCols = 64;  // GEMM columns per column block
// K order inside an 8-value chunk of the quantized GEMMs' activation rows:
// position e holds value perm8(e) = [0 4 1 5 2 6 3 7][e].
__host__ __device__ constexpr int perm8(int e) { return (e & 1) ? 4 + (e >> 1) : (e >> 1); }

// math.zig:46-60, rounded as written (no contraction), with the exponential
// from CUDA's expf (within 2 ulp of exp). The reference's own exp (the host
// libm expf, restated bit for bit as exp_ref) computes in double, and double
// arithmetic is slow enough on this part that it made the first convolution's
// 46 M GELUs of a 30-second clip its most expensive kernel.
__device__ __forceinline__ float erf_ref(float x) {
  const float sign = x < 0.0f ? -1.0f : 1.0f;
  const float m = fabsf(x);
  const float t = __frcp_rn(__fadd_rn(1.0f, __fmul_rn(0.5f, m)));  // 1 / (1 + m / 2), correctly rounded
  float poly = __fadd_rn(-0.82215223f, __fmul_rn(t, 0.17087277f));
  poly = __fadd_rn(1.48851587f, __fmul_rn(t, poly));
  poly = __fadd_rn(-1.13520398f, __fmul_rn(t, poly));
  poly = __fadd_rn(0.27886807f, __fmul_rn(t, poly));
  poly = __fadd_rn(-0.18628806f, __fmul_rn(t, poly));
  poly = __fadd_rn(0.09678418f, __fmul_rn(t, poly));
  poly = __fadd_rn(0.37409196f, __fmul_rn(t, poly));
  poly = __fadd_rn(1.00002368f, __fmul_rn(t, poly));
  const float arg = __fadd_rn(__fsub_rn(__fmul_rn(-m, m), 1.26551223f), __fmul_rn(t, poly));
  const float tau = __fmul_rn(t, expf(arg));
  return __fmul_rn(sign, __fsub_rn(1.0f, tau));
}

// math.zig:63-66
__device__ __forceinline__ float gelu_ref(float x) {
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, erf_ref(__fmul_rn(x, 0.70710678f))));
}

__device__ __forceinline__ void split_store(__half* hi_row, __half* lo_row, const float (&v)[8]) {
  __align__(16) __half hi[8];
  __align__(16) __half lo[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    hi[j] = __float2half_rn(v[j]);
    lo[j] = __float2half_rn(v[j] - __half2float(hi[j]));
  }
  *reinterpret_cast<uint4*>(hi_row) = *reinterpret_cast<const uint4*>(hi);
  *reinterpret_cast<uint4*>(lo_row) = *reinterpret_cast<const uint4*>(lo);
}

// The f16 hi row of GEMM column `col` in a packed buffer of `k` columns per
// row; its lo row is kCols rows further.
__device__ __forceinline__ __half* packed_row(__half* base, uint32_t col, uint32_t k) {
  return base + (size_t(col / kCols) * (2 * kCols) + col % kCols) * k;
}

// ---- convolution 1 (one input channel): kernels.zig:332-432 ----
// mel [mel_bins][frames] -> out [chunk][h1][w1][channels], zero frames past
// the clip (the reference pads each chunk in the mel domain, model.zig:535-545).
// A thread takes one position and kConv1Group channels c0 + k * (C / group),
// channels fastest across threads, so a warp's taps are broadcast loads, read
// once for the group, and its stores are contiguous. The weights sit in
// shared memory as [tap][channel] floats (lanes read consecutive banks).
// Each channel sums its valid taps in the reference's order.
constexpr uint32_t kConv1MaxChannels = 1024;
constexpr uint32_t kConv1Group = 4;

__global__ void __launch_bounds__(256) audio_conv1_kernel(const float* mel, uint32_t frames, uint32_t mel_bins,
                                                          uint32_t chunk_frames, uint32_t chunks, const __half* w,
                                                          const float* bias, uint32_t channels, float* out) {
  __shared__ float ws[9 * kConv1MaxChannels];
  __shared__ float bs[kConv1MaxChannels];
  for (uint32_t i = threadIdx.x; i < 9 * channels; i += blockDim.x) {
    const uint32_t oc = i / 9, t = i % 9;
    ws[t * channels + oc] = __half2float(w[i]);
  }
  for (uint32_t i = threadIdx.x; i < channels; i += blockDim.x) bs[i] = bias[i];
  __syncthreads();
  pdl_wait_and_trigger();
  const uint32_t h1 = (mel_bins - 1) / 2 + 1, w1 = (chunk_frames - 1) / 2 + 1;
  const uint32_t per = channels / kConv1Group;
  const uint32_t total = chunks * h1 * w1 * per;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t c0 = i % per, pos = i / per;
    const uint32_t ox = pos % w1, oy = (pos / w1) % h1, chunk = pos / (w1 * h1);
    float x[9];
    bool in[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) {
      const int iy = int(2 * oy) + t / 3 - 1, ix = int(2 * ox) + t % 3 - 1;
      in[t] = iy >= 0 && iy < int(mel_bins) && ix >= 0 && ix < int(chunk_frames);
      const uint32_t frame = chunk * chunk_frames + uint32_t(ix);
      x[t] = in[t] && frame < frames ? mel[size_t(iy) * frames + frame] : 0.0f;
    }
#pragma unroll
    for (uint32_t k = 0; k < kConv1Group; ++k) {
      const uint32_t oc = c0 + k * per;
      float acc = 0.0f;
#pragma unroll
      for (int t = 0; t < 9; ++t) {
        if (in[t]) acc = __fadd_rn(acc, __fmul_rn(ws[t * channels + oc], x[t]));
      }
      out[size_t(pos) * channels + oc] = gelu_ref(__fadd_rn(bs[oc], acc));
    }
  }
}

// ---- im2col for convolutions 2 and 3 ----
// in [chunk][ih][iw][channels] -> GEMM activation rows, column n =
// (chunk, oy, ox), K index (ky * 3 + kx) * channels + ic, zero past 9 channels
// and outside the input (padding 1). channels % 8 == 0.
__global__ void audio_im2col_kernel(const float* in, uint32_t chunks, uint32_t ih, uint32_t iw, uint32_t channels,
                                    uint32_t kpad, __half* out) {
  pdl_wait_and_trigger();
  const uint32_t oh = (ih - 1) / 2 + 1, ow = (iw - 1) / 2 + 1;
  const uint32_t columns = chunks * oh * ow, groups = kpad / 8, taps_k = 9 * channels;
  const uint32_t total = columns * groups;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t g = i % groups, col = i / groups;
    const uint32_t k0 = g * 8;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (k0 < taps_k) {
      const uint32_t tap = k0 / channels, ic = k0 % channels;
      const uint32_t ox = col % ow, oy = (col / ow) % oh, chunk = col / (ow * oh);
      const int iy = int(2 * oy) + int(tap / 3) - 1, ix = int(2 * ox) + int(tap % 3) - 1;
      if (iy >= 0 && iy < int(ih) && ix >= 0 && ix < int(iw)) {
        const float4* src =
            reinterpret_cast<const float4*>(in + ((size_t(chunk) * ih + iy) * iw + ix) * channels + ic);
        const float4 a = src[0], b = src[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      }
    }
    __half* hi = packed_row(out, col, kpad) + k0;
    split_store(hi, hi + size_t(kCols) * kpad, v);
  }
}

// Convolution epilogue: out[n][c] = gelu(bias[c] + sum of the split partials).
__global__ void audio_conv_epilogue_kernel(const float* parts, uint32_t splits, uint32_t columns, uint32_t channels,
                                           const float* bias, float* out) {
  pdl_wait_and_trigger();
  const uint32_t n = columns * channels;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float acc = parts[i];
    for (uint32_t sp = 1; sp < splits; ++sp) acc += parts[size_t(sp) * n + i];
    out[i] = gelu_ref(__fadd_rn(bias[i % channels], acc));
  }
}

// model.zig:580-597: the conv_out input of packed step p (chunk p / steps,
// time step p % steps) is flat[c * bins + f] = conv3[chunk][f][t][c]; packed
// for the quantized GEMM (K chunks permuted).
__global__ void audio_flatten_kernel(const float* conv3, uint32_t steps, uint32_t chunk_steps, uint32_t bins,
                                     uint32_t channels, __half* out) {
  pdl_wait_and_trigger();
  const uint32_t k = channels * bins, groups = k / 8;
  const uint32_t total = steps * groups;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t g = i % groups, p = i / groups;
    const uint32_t chunk = p / chunk_steps, t = p % chunk_steps;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t j = g * 8 + perm8(e), c = j / bins, f = j % bins;
      v[e] = conv3[((size_t(chunk) * bins + f) * chunk_steps + t) * channels + c];
    }
    __half* hi = packed_row(out, p, k) + g * 8;
    split_store(hi, hi + size_t(kCols) * k, v);
  }
}

// Epilogues of the tower's quantized GEMMs over parts[split][steps][ld]
// (columns [col0, col0 + width) of each row):
//   kPosition  x[p][i] = sum + position[p % chunk_steps][i]   (conv_out, model.zig:600-601)
//   kBias      x[p][i] = sum + bias[i]                        (q|k|v, projector out)
//   kResidual  x[p][i] = x[p][i] + (sum + bias[i])           (kernels.zig:221-230)
//   kGeluPack  gelu(sum + bias[i]) into GEMM activation rows (model.zig:863-866, 719)
enum EpilogueMode : int { kPosition = 0, kBias = 1, kResidual = 2, kGeluPack = 3 };

template <int Mode>
__global__ void audio_epilogue_kernel(const float* parts, uint32_t splits, uint32_t steps, uint32_t ld,
                                      uint32_t width, const float* add, uint32_t chunk_steps, float* x,
                                      uint32_t x_ld, __half* packed) {
  pdl_wait_and_trigger();
  const uint32_t groups = width / 8;
  const uint32_t total = steps * groups;
  const size_t plane = size_t(steps) * ld;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const uint32_t g = i % groups, p = i / groups;
    const float* src = parts + size_t(p) * ld + g * 8;
    float v[8];
    {
      const float4 a = reinterpret_cast<const float4*>(src)[0], b = reinterpret_cast<const float4*>(src)[1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
    for (uint32_t sp = 1; sp < splits; ++sp) {
      const float4 a = reinterpret_cast<const float4*>(src + sp * plane)[0];
      const float4 b = reinterpret_cast<const float4*>(src + sp * plane)[1];
      v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w;
      v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
    }
    const float* addp = Mode == kPosition ? add + size_t(p % chunk_steps) * width + g * 8 : add + g * 8;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(v[e], addp[e]);
    if (Mode == kGeluPack) {
      float w[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) w[e] = gelu_ref(v[perm8(e)]);
      __half* hi = packed_row(packed, p, width) + g * 8;
      split_store(hi, hi + size_t(kCols) * width, w);
    } else {
      float* dst = x + size_t(p) * x_ld + g * 8;
      if (Mode == kResidual) {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fadd_rn(dst[e], v[e]);
      }
      reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
}

// LayerNorm of each step row (math.zig:99-116: mean, then the mean of the
// centred squares, 1 / sqrt(var + eps), (x - mean) * inv * w + b), one
// 128-thread block per row, optionally after the residual add that precedes
// it in the block (kernels.zig:221-230): with `parts`, the row first becomes
// x + (sum of the split partials + rbias) and is written back to x. The
// normalized row goes to the GEMM activation rows (`packed`) and/or to `out`
// (f32; may be x itself, which then holds the normalized row).
// width % 8 == 0, width <= 128 * 8 * 4.
constexpr int kNormThreads = 128;
constexpr int kNormMaxChunks = 4;  // 8-value chunks per thread

__global__ void __launch_bounds__(kNormThreads) audio_layernorm_kernel(float* x, const float* parts, uint32_t splits,
                                                                       size_t plane, const float* rbias,
                                                                       const float* weight, const float* bias,
                                                                       uint32_t width, float eps, float* out,
                                                                       __half* packed) {
  pdl_wait_and_trigger();
  __shared__ float red[kNormThreads / 32];
  __shared__ float stat;
  const uint32_t p = blockIdx.x, tid = threadIdx.x, chunks = width / 8;
  float* row = x + size_t(p) * width;
  float v[kNormMaxChunks][8];
  float sum = 0.0f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const uint32_t ch = tid + c * kNormThreads;
    if (ch < chunks) {
      const float4 a = reinterpret_cast<const float4*>(row + ch * 8)[0];
      const float4 b = reinterpret_cast<const float4*>(row + ch * 8)[1];
      v[c][0] = a.x; v[c][1] = a.y; v[c][2] = a.z; v[c][3] = a.w;
      v[c][4] = b.x; v[c][5] = b.y; v[c][6] = b.z; v[c][7] = b.w;
      if (parts) {
        const float* src = parts + size_t(p) * width + ch * 8;
        float r[8];
        {
          const float4 u = reinterpret_cast<const float4*>(src)[0], w = reinterpret_cast<const float4*>(src)[1];
          r[0] = u.x; r[1] = u.y; r[2] = u.z; r[3] = u.w;
          r[4] = w.x; r[5] = w.y; r[6] = w.z; r[7] = w.w;
        }
        for (uint32_t sp = 1; sp < splits; ++sp) {
          const float4 u = reinterpret_cast<const float4*>(src + sp * plane)[0];
          const float4 w = reinterpret_cast<const float4*>(src + sp * plane)[1];
          r[0] += u.x; r[1] += u.y; r[2] += u.z; r[3] += u.w;
          r[4] += w.x; r[5] += w.y; r[6] += w.z; r[7] += w.w;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) v[c][e] = __fadd_rn(v[c][e], __fadd_rn(r[e], rbias[ch * 8 + e]));
        if (out != x) {
          reinterpret_cast<float4*>(row + ch * 8)[0] = make_float4(v[c][0], v[c][1], v[c][2], v[c][3]);
          reinterpret_cast<float4*>(row + ch * 8)[1] = make_float4(v[c][4], v[c][5], v[c][6], v[c][7]);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) sum += v[c][e];
    }
  }
  auto block_sum = [&](float s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((tid & 31) == 0) red[tid / 32] = s;
    __syncthreads();
    if (tid == 0) {
      float t = 0.0f;
      for (int w = 0; w < kNormThreads / 32; ++w) t += red[w];
      stat = t;
    }
    __syncthreads();
    const float r = stat;
    __syncthreads();
    return r;
  };
  const float mean = __fdiv_rn(block_sum(sum), static_cast<float>(width));
  float sq = 0.0f;
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    if (tid + c * kNormThreads < chunks) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float d = __fsub_rn(v[c][e], mean);
        sq = __fadd_rn(sq, __fmul_rn(d, d));
      }
    }
  }
  const float variance = __fdiv_rn(block_sum(sq), static_cast<float>(width));
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
#pragma unroll
  for (int c = 0; c < kNormMaxChunks; ++c) {
    const uint32_t ch = tid + c * kNormThreads;
    if (ch < chunks) {
      float y[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t i = ch * 8 + e;
        y[e] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v[c][e], mean), inv), weight[i]), bias[i]);
      }
      if (out) {
        float* dst = out + size_t(p) * width + ch * 8;
        reinterpret_cast<float4*>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
      }
      if (packed) {
        float z[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) z[e] = y[perm8(e)];
        __half* hi = packed_row(packed, p, width) + ch * 8;
        split_store(hi, hi + size_t(kCols) * width, z);
      }
    }
  }
}

// kernels.zig:435-487 for one (window, head): scores = q.k / sqrt(head_dim)
// over the window's keys, softmax (math.zig:77-93), weighted sum of values.
// The q|k|v rows are the Q|K|V GEMM's split partials [split][step][3 width]
// summed here, plus the biases (projectQkv, model.zig:764-782); the output
// goes straight into the O GEMM's activation rows (f16 hi and lo, K chunks
// permuted). head_dim 64,
// windows of at most 128 steps. One CTA per (window, head, 16 queries): the
// window's keys and values in shared memory (key rows padded by one float
// against bank conflicts), each of 4 warps takes 4 queries at once, so a lane
// carries 16 independent score sums (4 queries x its 4 keys) and 8 value sums
// (4 queries x its 2 dimensions) instead of one long chain.
constexpr int kAttnWarps = 4;
constexpr int kAttnQueries = 4;                        // per warp
constexpr int kAttnCtaQueries = kAttnWarps * kAttnQueries;
constexpr uint32_t kAttnHead = 64;
constexpr uint32_t kAttnMaxWindow = 128;

// Position of value v inside an 8-value chunk of the activation rows.
__device__ __forceinline__ uint32_t perm8_inverse(uint32_t v) { return v < 4 ? 2 * v : 2 * (v - 4) + 1; }

__global__ void __launch_bounds__(kAttnWarps * 32) audio_window_attention_kernel(const float* parts, uint32_t splits,
                                                                                 const float* qkv_bias, uint32_t steps,
                                                                                 uint32_t width, uint32_t window,
                                                                                 __half* packed) {
  pdl_wait_and_trigger();
  extern __shared__ float attn_smem[];
  constexpr uint32_t hd = kAttnHead, kstride = hd + 1;
  const uint32_t w0 = blockIdx.x * window, h = blockIdx.y;
  const uint32_t len = min(window, steps - w0);
  const uint32_t q0 = blockIdx.z * kAttnCtaQueries;
  if (q0 >= len) return;
  float* ks = attn_smem;                                       // [window][hd + 1]
  float* vs = ks + (size_t(window) * kstride + 3) / 4 * 4;     // [window][hd], 16-byte aligned
  float* qs = vs + size_t(window) * hd;                        // [warps][queries][hd]
  float* ps = qs + size_t(kAttnWarps) * kAttnQueries * hd;     // [warps][queries][window]
  const uint32_t ld = 3 * width;
  const size_t plane = size_t(steps) * ld;
  // Element e of q|k|v row `step`: the sum of its split partials plus its bias.
  auto qkv4 = [&](uint32_t step, uint32_t e) {
    const float* src = parts + size_t(step) * ld + e;
    float4 a = *reinterpret_cast<const float4*>(src);
    for (uint32_t sp = 1; sp < splits; ++sp) {
      const float4 b = *reinterpret_cast<const float4*>(src + sp * plane);
      a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    }
    const float4 bias = *reinterpret_cast<const float4*>(qkv_bias + e);
    return make_float4(__fadd_rn(a.x, bias.x), __fadd_rn(a.y, bias.y), __fadd_rn(a.z, bias.z),
                       __fadd_rn(a.w, bias.w));
  };
  // The window's key and value rows, 16 bytes a load.
  constexpr uint32_t kVec = hd / 4;
#pragma unroll 4
  for (uint32_t i = threadIdx.x; i < len * kVec; i += blockDim.x) {
    const uint32_t j = i / kVec, d = (i % kVec) * 4;
    const float4 kv = qkv4(w0 + j, width + h * hd + d);
    const float4 vv = qkv4(w0 + j, 2 * width + h * hd + d);
    float* kd = ks + j * kstride + d;
    kd[0] = kv.x;
    kd[1] = kv.y;
    kd[2] = kv.z;
    kd[3] = kv.w;
    *reinterpret_cast<float4*>(vs + j * hd + d) = vv;
  }
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t qw = q0 + warp * kAttnQueries;  // this warp's first query
  float* q = qs + size_t(warp) * kAttnQueries * hd;
  float* pw = ps + size_t(warp) * kAttnQueries * window;
  for (uint32_t i = lane; i < kAttnQueries * hd / 4; i += 32) {
    const uint32_t qq = i / (hd / 4), d = (i % (hd / 4)) * 4;
    const float4 v = qw + qq < len ? qkv4(w0 + qw + qq, h * hd + d) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    q[qq * hd + d] = v.x;
    q[qq * hd + d + 1] = v.y;
    q[qq * hd + d + 2] = v.z;
    q[qq * hd + d + 3] = v.w;
  }
  __syncthreads();
  if (qw >= len) return;
  const float scaling = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));
  float acc[kAttnQueries][4];
#pragma unroll
  for (int a = 0; a < kAttnQueries; ++a) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) acc[a][kk] = 0.0f;
  }
  uint32_t kidx[4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) kidx[kk] = min(lane + 32u * kk, len - 1) * kstride;
#pragma unroll 4
  for (uint32_t d = 0; d < hd; ++d) {
    float kv[4], qv[kAttnQueries];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) kv[kk] = ks[kidx[kk] + d];
#pragma unroll
    for (int a = 0; a < kAttnQueries; ++a) qv[a] = q[a * hd + d];
#pragma unroll
    for (int a = 0; a < kAttnQueries; ++a) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) acc[a][kk] = fmaf(qv[a], kv[kk], acc[a][kk]);
    }
  }
#pragma unroll
  for (int a = 0; a < kAttnQueries; ++a) {
    float mx = -INFINITY;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      acc[a][kk] = __fmul_rn(acc[a][kk], scaling);
      if (lane + 32u * kk < len) mx = fmaxf(mx, acc[a][kk]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float total = 0.0f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const float e = lane + 32u * kk < len ? expf(__fsub_rn(acc[a][kk], mx)) : 0.0f;
      acc[a][kk] = e;
      total += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    const float inv = __fdiv_rn(1.0f, total);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      if (lane + 32u * kk < len) pw[a * window + lane + 32u * kk] = __fmul_rn(acc[a][kk], inv);
    }
  }
  __syncwarp();
  float o[kAttnQueries][2];
#pragma unroll
  for (int a = 0; a < kAttnQueries; ++a) o[a][0] = o[a][1] = 0.0f;
#pragma unroll 4
  for (uint32_t j = 0; j < len; ++j) {
    const float v0 = vs[j * hd + lane], v1 = vs[j * hd + lane + 32];
#pragma unroll
    for (int a = 0; a < kAttnQueries; ++a) {
      const float p = pw[a * window + j];
      o[a][0] = fmaf(v0, p, o[a][0]);
      o[a][1] = fmaf(v1, p, o[a][1]);
    }
  }
#pragma unroll
  for (int a = 0; a < kAttnQueries; ++a) {
    if (qw + a < len) {
      __half* hi = packed_row(packed, w0 + qw + a, width);
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t k = h * hd + lane + 32 * u;
        const uint32_t at = (k & ~7u) + perm8_inverse(k & 7u);
        const __half vh = __float2half_rn(o[a][u]);
        hi[at] = vh;
        hi[size_t(kCols) * width + at] = __float2half_rn(o[a][u] - __half2float(vh));
      }
    }
  }
}

uint32_t grid_for(size_t work, uint32_t threads) {
  const size_t blocks = (work + threads - 1) / threads;
  return static_cast<uint32_t>(blocks < 148 * 16 ? (blocks ? blocks : 1) : 148 * 16);
}

}  // namespace

int launch_audio_conv1(const float* mel, uint32_t frames, uint32_t mel_bins, uint32_t chunk_frames, uint32_t chunks,
                       const void* w, const float* bias, uint32_t channels, float* out, void* stream) {
  const size_t work = size_t(chunks) * ((mel_bins - 1) / 2 + 1) * ((chunk_frames - 1) / 2 + 1) * channels / 4;
  return static_cast<int>(launch_pdl(audio_conv1_kernel, dim3(grid_for(work, 256)), dim3(256), 0,
                                     static_cast<cudaStream_t>(stream), mel, frames, mel_bins, chunk_frames, chunks,
                                     static_cast<const __half*>(w), bias, channels, out));
}

int launch_audio_im2col(const float* in, uint32_t chunks, uint32_t ih, uint32_t iw, uint32_t channels, uint32_t kpad,
                        void* out, void* stream) {
  const size_t work = size_t(chunks) * ((ih - 1) / 2 + 1) * ((iw - 1) / 2 + 1) * (kpad / 8);
  return static_cast<int>(launch_pdl(audio_im2col_kernel, dim3(grid_for(work, 256)), dim3(256), 0,
                                     static_cast<cudaStream_t>(stream), in, chunks, ih, iw, channels, kpad,
                                     static_cast<__half*>(out)));
}

int launch_audio_conv_epilogue(const float* parts, uint32_t splits, uint32_t columns, uint32_t channels,
                               const float* bias, float* out, void* stream) {
  return static_cast<int>(launch_pdl(audio_conv_epilogue_kernel, dim3(grid_for(size_t(columns) * channels, 256)),
                                     dim3(256), 0, static_cast<cudaStream_t>(stream), parts, splits, columns,
                                     channels, bias, out));
}

int launch_audio_flatten(const float* conv3, uint32_t steps, uint32_t chunk_steps, uint32_t bins, uint32_t channels,
                         void* out, void* stream) {
  return static_cast<int>(launch_pdl(audio_flatten_kernel, dim3(grid_for(size_t(steps) * channels * bins / 8, 256)),
                                     dim3(256), 0, static_cast<cudaStream_t>(stream), conv3, steps, chunk_steps, bins,
                                     channels, static_cast<__half*>(out)));
}

int launch_audio_epilogue(int mode, const float* parts, uint32_t splits, uint32_t steps, uint32_t ld, uint32_t width,
                          const float* add, uint32_t chunk_steps, float* x, uint32_t x_ld, void* packed,
                          void* stream) {
  const dim3 grid(grid_for(size_t(steps) * width / 8, 256)), block(256);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  __half* pk = static_cast<__half*>(packed);
  switch (mode) {
    case kPosition:
      return static_cast<int>(launch_pdl(audio_epilogue_kernel<kPosition>, grid, block, 0, st, parts, splits, steps,
                                         ld, width, add, chunk_steps, x, x_ld, pk));
    case kBias:
      return static_cast<int>(launch_pdl(audio_epilogue_kernel<kBias>, grid, block, 0, st, parts, splits, steps, ld,
                                         width, add, chunk_steps, x, x_ld, pk));
    case kResidual:
      return static_cast<int>(launch_pdl(audio_epilogue_kernel<kResidual>, grid, block, 0, st, parts, splits, steps,
                                         ld, width, add, chunk_steps, x, x_ld, pk));
    default:
      return static_cast<int>(launch_pdl(audio_epilogue_kernel<kGeluPack>, grid, block, 0, st, parts, splits, steps,
                                         ld, width, add, chunk_steps, x, x_ld, pk));
  }
}

int launch_audio_layernorm(float* x, const float* parts, uint32_t splits, const float* rbias, const float* weight,
                           const float* bias, uint32_t width, float eps, uint32_t steps, float* out, void* packed,
                           void* stream) {
  return static_cast<int>(launch_pdl(audio_layernorm_kernel, dim3(steps), dim3(kNormThreads), 0,
                                     static_cast<cudaStream_t>(stream), x, parts, splits,
                                     size_t(steps) * width, rbias, weight, bias, width, eps, out,
                                     static_cast<__half*>(packed)));
}

size_t audio_attention_smem(uint32_t window, uint32_t head_dim) {
  if (head_dim != kAttnHead || window > kAttnMaxWindow) return ~size_t(0);  // the kernel's limits
  return ((size_t(window) * (head_dim + 1) + 3) / 4 * 4 + size_t(window) * head_dim +
          size_t(kAttnWarps) * kAttnQueries * (head_dim + window)) * 4;
}

int launch_audio_attention(const float* parts, uint32_t splits, const float* qkv_bias, uint32_t steps,
                           uint32_t width, uint32_t heads, uint32_t head_dim, uint32_t window, void* packed,
                           void* stream) {
  const size_t smem = audio_attention_smem(window, head_dim);
  const dim3 grid((steps + window - 1) / window, heads, (window + kAttnCtaQueries - 1) / kAttnCtaQueries);
  return static_cast<int>(launch_pdl(audio_window_attention_kernel, grid, dim3(kAttnWarps * 32), smem,
                                     static_cast<cudaStream_t>(stream), parts, splits, qkv_bias, steps, width,
                                     window, static_cast<__half*>(packed)));
}

int prepare_audio_kernels(uint32_t window, uint32_t head_dim) {
  return static_cast<int>(cudaFuncSetAttribute(audio_window_attention_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(audio_attention_smem(window, head_dim))));
}

}  // namespace qwc

// qwc_ops.cu -- device-pointer operators of the C ABI (qwc_op_*).
//
// Each operator runs one building block of the token loop on caller-owned
// device buffers: dequantization and q8 quantization (bit exact with
// src/core/quant.zig), the fused dequant GEMV, decode attention over a q8
// cache, RMSNorm, RoPE, SwiGLU and the argmax. They share the dequantization
// arithmetic of the persistent decode kernel (qwc_device.cuh).

#include <cuda_runtime.h>

#include <mutex>

#include "../../include/qwenscriber_cuda.h"
#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

__global__ void dequantize_kernel(uint32_t format, const uint8_t* scales, const uint8_t* codes, uint32_t rows,
                                  uint32_t cols, float* out) {
  const uint64_t n = uint64_t(rows) * cols;
  const uint32_t groups = cols / kGroup;
  for (uint64_t idx = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; idx < n;
       idx += uint64_t(gridDim.x) * blockDim.x) {
    const uint64_t r = idx / cols;
    const uint32_t k = static_cast<uint32_t>(idx % cols);
    const uint32_t g = k / kGroup;
    const float scale = f16_bits_to_f32(reinterpret_cast<const uint16_t*>(scales)[r * groups + g]);
    int code;
    if (format == kFormatQ4) {
      const uint8_t b = codes[r * groups * 32 + k / 2];
      code = static_cast<int>((k & 1u) ? (b >> 4) : (b & 0x0F)) - 8;
    } else if (format == kFormatQ5) {
      code = q5_code(codes + (r * groups + g) * 40, k % kGroup);
    } else {
      code = static_cast<int>(codes[r * groups * 64 + k]) - 128;
    }
    // quant.zig:336-344: float(code) then times the scale.
    out[idx] = static_cast<float>(code) * scale;
  }
}

// One warp per 64-value group (quant.zig:209-226).
__global__ void quantize_q8_kernel(const float* values, uint32_t rows, uint32_t cols, uint8_t* scales, uint8_t* codes) {
  const uint32_t groups = cols / kGroup;
  const uint64_t total = uint64_t(rows) * groups;
  const uint32_t lane = threadIdx.x & 31;
  for (uint64_t gi = (blockIdx.x * uint64_t(blockDim.x) + threadIdx.x) / 32; gi < total;
       gi += uint64_t(gridDim.x) * blockDim.x / 32) {
    const float* v = values + gi * kGroup;
    const float a = v[lane], b = v[lane + 32];
    const float amax = warp_max(fmaxf(fabsf(a), fabsf(b)));
    const __half sh = __float2half_rn(amax / 128.0f);
    const float stored = __half2float(sh);
    codes[gi * kGroup + lane] = q8_code(a, stored);
    codes[gi * kGroup + lane + 32] = q8_code(b, stored);
    if (lane == 0) reinterpret_cast<uint16_t*>(scales)[gi] = __half_as_ushort(sh);
  }
}

// One warp per row; lane l takes the 16-byte chunks at l*16 + 512*j of the row
// (q5: half l & 1 of group l / 2 + 16 j).
__global__ void gemv_kernel(uint32_t format, const uint8_t* scales, const uint8_t* codes, uint32_t rows, uint32_t cols,
                            const float* x, float* out) {
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t warps = blockDim.x / 32;
  const uint32_t groups = cols / kGroup;
  const uint32_t db = data_bytes_per_group(format);
  const uint32_t code_row = groups * db;
  for (uint32_t r = blockIdx.x * warps + threadIdx.x / 32; r < rows; r += gridDim.x * warps) {
    const uint8_t* crow = codes + size_t(r) * code_row;
    const uint16_t* srow = reinterpret_cast<const uint16_t*>(scales) + size_t(r) * groups;
    float acc = 0.0f;
    if (format == kFormatQ5) {
      for (uint32_t g = lane / 2; g < groups; g += 16) {
        const uint32_t h = lane & 1u;
        const uint8_t* grp = crow + size_t(g) * 40;
        const uint2 l0 = *reinterpret_cast<const uint2*>(grp + 16u * h);
        const uint2 l1 = *reinterpret_cast<const uint2*>(grp + 16u * h + 8u);
        const uint32_t fifth = *reinterpret_cast<const uint32_t*>(grp + 32u + 4u * h);
        const float d = q5_half_dot(l0.x, l0.y, l1.x, l1.y, fifth, x + 64u * g + 32u * h);
        acc = fmaf(d, f16_bits_to_f32(srow[g]), acc);
      }
      acc = warp_sum(acc);
      if (lane == 0) out[r] = acc;
      continue;
    }
    for (uint32_t off = 16u * lane; off < code_row; off += 512u) {
      const uint4 w = ld_nc4(crow + off);
      const float scale = f16_bits_to_f32(srow[off / db]);
      float d;
      if (format == kFormatQ4) {
        uint64_t x2[16];
        const uint32_t k0 = off * 2;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(x + k0 + 4 * q);
          const int i0 = (4 * q) % 8;
          x2[2 * q] = pack2(v.x * q4_xscale(i0), v.y * q4_xscale(i0 + 1));
          x2[2 * q + 1] = pack2(v.z * q4_xscale(i0 + 2), v.w * q4_xscale(i0 + 3));
        }
        d = q4_chunk_dot(w, x2);
      } else {
        uint64_t x2[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 v = *reinterpret_cast<const float4*>(x + off + 4 * q);
          x2[2 * q] = pack2(v.x, v.y);
          x2[2 * q + 1] = pack2(v.z, v.w);
        }
        d = q8_chunk_dot(w, x2);
      }
      acc = fmaf(d, scale, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) out[r] = acc;
  }
}

// One block per query head, blockDim = 128 (one thread per dim for the value
// pass; positions striped over threads for the score pass). Shared memory:
// `cached` scores.
__global__ void attention_q8_kernel(const float* query, const uint8_t* ks, const uint8_t* kc, const uint8_t* vs,
                                    const uint8_t* vc, uint32_t cached, uint32_t heads, uint32_t kv_heads,
                                    uint32_t head_dim, float scaling, float* out) {
  extern __shared__ float sh[];
  float* scores = sh;
  float* red = sh + cached;
  const uint32_t head = blockIdx.x;
  const uint32_t kvh = head / (heads / kv_heads);
  const uint32_t kvw = kv_heads * head_dim;
  const uint32_t groups_per_row = kvw / kGroup;
  const uint32_t tid = threadIdx.x;
  const float* q = query + size_t(head) * head_dim;
  for (uint32_t p = tid; p < cached; p += blockDim.x) {
    const uint8_t* codes = kc + size_t(p) * kvw + size_t(kvh) * head_dim;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(ks) + size_t(p) * groups_per_row + size_t(kvh) * head_dim / kGroup;
    float total = 0.0f;
    for (uint32_t g = 0; g < head_dim / kGroup; ++g) {
      float inner = 0.0f;
      for (uint32_t i = 0; i < kGroup; ++i) {
        inner = fmaf(static_cast<float>(codes[g * kGroup + i]) - 128.0f, q[g * kGroup + i], inner);
      }
      total = fmaf(inner, f16_bits_to_f32(sc[g]), total);
    }
    scores[p] = scaling * total;
  }
  __syncthreads();
  // softmax (math.zig:77-93)
  float mx = -INFINITY;
  for (uint32_t p = tid; p < cached; p += blockDim.x) mx = fmaxf(mx, scores[p]);
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid / 32] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (uint32_t w = 0; w < blockDim.x / 32; ++w) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float sum = 0.0f;
  for (uint32_t p = tid; p < cached; p += blockDim.x) {
    const float e = expf(scores[p] - mx);
    scores[p] = e;
    sum += e;
  }
  sum = warp_sum(sum);
  if ((tid & 31) == 0) red[tid / 32] = sum;
  __syncthreads();
  sum = 0.0f;
  for (uint32_t w = 0; w < blockDim.x / 32; ++w) sum += red[w];
  const float inv = 1.0f / sum;
  for (uint32_t d = tid; d < head_dim; d += blockDim.x) {
    float acc = 0.0f;
    const uint32_t g = d / kGroup;
    for (uint32_t p = 0; p < cached; ++p) {
      const uint8_t code = vc[size_t(p) * kvw + size_t(kvh) * head_dim + d];
      const float scale =
          f16_bits_to_f32(reinterpret_cast<const uint16_t*>(vs)[size_t(p) * groups_per_row + size_t(kvh) * head_dim / kGroup + g]);
      acc = fmaf(static_cast<float>(code) - 128.0f, scale * (scores[p] * inv), acc);
    }
    out[size_t(head) * head_dim + d] = acc;
  }
}

struct ArgmaxPartial {
  float value;
  uint32_t index;
};

__device__ __forceinline__ bool better(float v, uint32_t i, float bv, uint32_t bi) {
  return v > bv || (v == bv && i < bi);
}

// decoder.zig:290-301 seeds the maximum with values[0] and replaces it only on
// a strict `>`: a NaN at index 0 is never replaced, a NaN elsewhere never
// wins. Ranking a NaN at index 0 as +inf (ties go to the lowest index) and
// letting every other NaN lose all comparisons gives that answer from any
// reduction order.
__device__ __forceinline__ float argmax_key(float v, uint32_t i) {
  return (i == 0 && v != v) ? __int_as_float(0x7F800000) : v;
}

// Pass 1: each block reduces a contiguous range to (max, first index).
__global__ void argmax_partial_kernel(const float* values, uint32_t count, ArgmaxPartial* partial) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  const uint32_t per = (count + gridDim.x - 1) / gridDim.x;
  const uint32_t begin = blockIdx.x * per;
  const uint32_t end = min(count, begin + per);
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const float v = argmax_key(values[i], i);
    if (better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
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
      if (better(sv[w], si[w], bv, bi)) {
        bv = sv[w];
        bi = si[w];
      }
    }
    partial[blockIdx.x] = ArgmaxPartial{bv, bi};
  }
}

// Pass 2: one warp combines the block partials.
__global__ void argmax_final_kernel(const ArgmaxPartial* partial, uint32_t n, uint32_t* out) {
  float bv = -INFINITY;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t i = threadIdx.x; i < n; i += 32) {
    if (better(partial[i].value, partial[i].index, bv, bi)) {
      bv = partial[i].value;
      bi = partial[i].index;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (threadIdx.x == 0) *out = bi == 0xFFFFFFFFu ? 0u : bi;
}

// math.zig:120-130 as written: the sum of squares in index order (one
// thread), then value * inverse_rms * weight with each product rounded.
__global__ void rmsnorm_kernel(const float* x, const float* w, uint32_t width, float eps, float* out) {
  __shared__ float inv_s;
  const float* row = x + size_t(blockIdx.x) * width;
  if (threadIdx.x == 0) inv_s = rms_inverse(sum_squares_seq(row, width), width, eps);
  __syncthreads();
  const float inv = inv_s;
  for (uint32_t i = threadIdx.x; i < width; i += blockDim.x) {
    out[size_t(blockIdx.x) * width + i] = __fmul_rn(__fmul_rn(row[i], inv), w[i]);
  }
}

__global__ void rope_kernel(float* x, uint32_t heads, uint32_t head_dim, const float* cos_t, const float* sin_t,
                            uint32_t position) {
  const uint32_t half = head_dim / 2;
  const uint32_t n = heads * half;
  for (uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += gridDim.x * blockDim.x) {
    const uint32_t h = idx / half, i = idx % half;
    float* row = x + size_t(h) * head_dim;
    const float lo = row[i], hi = row[i + half];
    const float c = cos_t[size_t(position) * half + i], s = sin_t[size_t(position) * half + i];
    row[i] = rope_rn(true, lo, hi, c, s);
    row[i + half] = rope_rn(false, lo, hi, c, s);
  }
}

__global__ void silu_mul_kernel(const float* gate, const float* up, uint32_t n, float* out) {
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float g = gate[i];
    out[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g))), up[i]);  // math.zig:69-71, kernels.zig:233-239
  }
}

int32_t status_of(cudaError_t e) {
  if (e == cudaSuccess) return QWC_OK;
  if (e == cudaErrorMemoryAllocation) return QWC_OUT_OF_MEMORY;
  return QWC_INVALID_STATE;
}

bool aligned(const void* p, uintptr_t a) { return reinterpret_cast<uintptr_t>(p) % a == 0; }

bool quant_format_ok(uint32_t format) { return format == kFormatQ4 || format == kFormatQ5 || format == kFormatQ8; }

// ---- argmax over a fixed, statically allocated device scratch ----
//
// qwc_op_argmax_noalloc runs the same two passes as qwc_op_argmax, but its
// block partials live in this file-scope array instead of a per-call
// workspace. Pass 1 writes every partial that pass 2 reads, so nothing in
// it has to start at zero. There is one array per device: two calls in
// flight on one device at the same time (different streams or host
// threads) share it and race.
constexpr uint32_t kNoallocPartials = 512;   // capacity: 512 partials, 4 KiB
constexpr uint32_t kNoallocPerBlock = 8192;  // most values one pass-1 block reduces
static_assert(uint64_t(kNoallocPartials) * kNoallocPerBlock == QWC_ARGMAX_NOALLOC_MAX_COUNT,
              "the header's count limit is the scratch capacity times the values per block");
static __device__ __align__(256) ArgmaxPartial g_argmax_scratch[kNoallocPartials];

constexpr int kNoallocDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_scratch[kNoallocDevices] = {};

// The device address of g_argmax_scratch on the current device, looked up
// once per device (the first call on that device does the lookup).
int32_t noalloc_scratch(ArgmaxPartial** out) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return status_of(e);
  if (device < 0 || device >= kNoallocDevices) return QWC_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_scratch[device]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_argmax_scratch);
    if (e != cudaSuccess) return status_of(e);
    g_noalloc_scratch[device] = p;
  }
  *out = static_cast<ArgmaxPartial*>(g_noalloc_scratch[device]);
  return QWC_OK;
}

}  // namespace
}  // namespace qwc

using namespace qwc;

extern "C" {

int32_t qwc_op_dequantize(uint32_t format, const void* scales, const void* codes, uint32_t rows, uint32_t cols,
                          float* out, void* stream) {
  if (!quant_format_ok(format)) return QWC_UNSUPPORTED;
  if (!scales || !codes || !out || cols % kGroup != 0) return QWC_INVALID_ARGUMENT;
  if (!aligned(scales, 2) || !aligned(out, 4)) return QWC_INVALID_ARGUMENT;
  if (rows == 0) return QWC_OK;
  dequantize_kernel<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      format, static_cast<const uint8_t*>(scales), static_cast<const uint8_t*>(codes), rows, cols, out);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_quantize_q8(const float* values, uint32_t rows, uint32_t cols, void* scales, void* codes, void* stream) {
  if (!values || !scales || !codes || cols % kGroup != 0) return QWC_INVALID_ARGUMENT;
  if (rows == 0) return QWC_OK;
  quantize_q8_kernel<<<592, 256, 0, static_cast<cudaStream_t>(stream)>>>(values, rows, cols,
                                                                          static_cast<uint8_t*>(scales),
                                                                          static_cast<uint8_t*>(codes));
  return status_of(cudaGetLastError());
}

int32_t qwc_op_gemv(uint32_t format, const void* scales, const void* codes, uint32_t rows, uint32_t cols,
                    const float* x, float* out, void* stream) {
  if (!quant_format_ok(format)) return QWC_UNSUPPORTED;
  if (!scales || !codes || !x || !out) return QWC_INVALID_ARGUMENT;
  // The kernel reads codes and activations with vector loads (16-byte for
  // q4/q8; 8-byte codes and scalar activations for q5): refuse pointers they
  // would fault on.
  const bool q5 = format == kFormatQ5;
  if (!aligned(codes, q5 ? 8 : 16) || !aligned(x, q5 ? 4 : 16) || !aligned(scales, 2) || !aligned(out, 4)) {
    return QWC_INVALID_ARGUMENT;
  }
  // The chunk walk needs whole 512-byte spans of codes per row (q5: whole
  // groups, 8-byte aligned rows).
  const uint32_t code_row = cols / kGroup * data_bytes_per_group(format);
  if (cols % kGroup != 0 || code_row % (format == kFormatQ5 ? 8u : 512u) != 0) return QWC_SHAPE_MISMATCH;
  if (rows == 0) return QWC_OK;
  const uint32_t blocks = (rows + 7) / 8;
  gemv_kernel<<<blocks < 4096 ? blocks : 4096, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      format, static_cast<const uint8_t*>(scales), static_cast<const uint8_t*>(codes), rows, cols, x, out);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_attention_q8(const float* query, const void* keys_scales, const void* keys_codes,
                            const void* values_scales, const void* values_codes, uint32_t cached, uint32_t heads,
                            uint32_t kv_heads, uint32_t head_dim, float* out, void* stream) {
  if (!query || !keys_scales || !keys_codes || !values_scales || !values_codes || !out) return QWC_INVALID_ARGUMENT;
  if (kv_heads == 0 || heads % kv_heads != 0 || head_dim % kGroup != 0 || cached == 0) return QWC_SHAPE_MISMATCH;
  const size_t smem = (size_t(cached) + 32) * sizeof(float);
  if (smem > 200 * 1024) return QWC_LIMIT_EXCEEDED;
  cudaFuncSetAttribute(attention_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  const float scaling = 1.0f / sqrtf(static_cast<float>(head_dim));
  attention_q8_kernel<<<heads, 128, smem, static_cast<cudaStream_t>(stream)>>>(
      query, static_cast<const uint8_t*>(keys_scales), static_cast<const uint8_t*>(keys_codes),
      static_cast<const uint8_t*>(values_scales), static_cast<const uint8_t*>(values_codes), cached, heads, kv_heads,
      head_dim, scaling, out);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_argmax(const float* values, uint32_t count, uint32_t* out_index, void* stream) {
  if (!values || !out_index || count == 0) return QWC_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t blocks = count < 148u * 256u ? (count + 255u) / 256u : 148u * 2u;
  void* workspace = nullptr;
  cudaError_t e = cudaMallocAsync(&workspace, sizeof(ArgmaxPartial) * blocks, s);
  if (e != cudaSuccess) return status_of(e);
  argmax_partial_kernel<<<blocks, 256, 0, s>>>(values, count, static_cast<ArgmaxPartial*>(workspace));
  argmax_final_kernel<<<1, 32, 0, s>>>(static_cast<ArgmaxPartial*>(workspace), blocks, out_index);
  e = cudaGetLastError();
  cudaFreeAsync(workspace, s);
  return status_of(e);
}

int32_t qwc_op_rmsnorm(const float* x, const float* weight, uint32_t width, uint32_t rows, float eps, float* out,
                       void* stream) {
  if (!x || !weight || !out || width == 0) return QWC_INVALID_ARGUMENT;
  if (rows == 0) return QWC_OK;
  rmsnorm_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, weight, width, eps, out);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_rope(float* x, uint32_t heads, uint32_t head_dim, const float* cos_table, const float* sin_table,
                    uint32_t position, void* stream) {
  if (!x || !cos_table || !sin_table || head_dim % 2 != 0) return QWC_INVALID_ARGUMENT;
  rope_kernel<<<64, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, heads, head_dim, cos_table, sin_table, position);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_silu_mul(const float* gate, const float* up, uint32_t n, float* out, void* stream) {
  if (!gate || !up || !out) return QWC_INVALID_ARGUMENT;
  if (n == 0) return QWC_OK;
  silu_mul_kernel<<<(n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      gate, up, n, out);
  return status_of(cudaGetLastError());
}

int32_t qwc_op_argmax_noalloc(const float* values, uint32_t count, uint32_t* out_index, void* stream) {
  if (!values || !out_index || count == 0) return QWC_INVALID_ARGUMENT;
  if (count > QWC_ARGMAX_NOALLOC_MAX_COUNT) return QWC_LIMIT_EXCEEDED;
  ArgmaxPartial* scratch = nullptr;
  const int32_t st = noalloc_scratch(&scratch);
  if (st != QWC_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint32_t blocks = (count + 255u) / 256u;
  if (blocks > kNoallocPartials) blocks = kNoallocPartials;
  argmax_partial_kernel<<<blocks, 256, 0, s>>>(values, count, scratch);
  argmax_final_kernel<<<1, 32, 0, s>>>(scratch, blocks, out_index);
  return status_of(cudaGetLastError());
}

}  // extern "C"

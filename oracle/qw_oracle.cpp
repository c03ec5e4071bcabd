// qw_oracle.cpp -- CPU restatement of the Qwenscriber decoder token loop.
//
// TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA backend. The
// product library never links or calls this file. Parity of this restatement
// with the reference is pinned by the reference's own known-answer tests
// (quant_hash of selftest.zig:288-298, the exact-code tests of quant.zig, the
// 56.0 row-of-ones case of kernels.zig:932-971, the LCG q8-vs-f32 attention
// case of kernels.zig:769-836, rope and inverse-frequency values of
// kernels.zig:1080-1117, the math.zig values), see tests/test_oracle_kat.py.
//
// Arithmetic follows the Zig source exactly where that decides bits:
//   * f32 products and sums are rounded separately (Zig's default float mode
//     does not contract a*b+c into an FMA); build with -ffp-contract=off.
//   * `@Vector(4, f32)` accumulators keep four lanes, and `@reduce(.Add)` sums
//     them in order (((l0 + l1) + l2) + l3), as LLVM's ordered fadd reduction.
//   * sums that the Zig code writes as sequential loops stay sequential.
// Transcendentals (expf, logf, sinf, cosf) come from the C library; Zig's
// compiler_rt versions may differ from them in the last bit, which no
// reference test observes.

#include "qw_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// abi.zig:50-84
enum Status : int32_t {
  kOk = 0,
  kInvalidArgument = -1,
  kOutOfMemory = -2,
  kUnsupported = -3,
  kShapeMismatch = -7,
  kInvalidState = -8,
  kLimitExceeded = -9,
  kNotFound = -10,
  kUnsupportedModel = -13,
};

constexpr uint32_t kGroup = 64;  // quant.zig:49

uint32_t round_shift_right(uint32_t value, uint32_t shift) {
  const uint32_t kept = value >> shift;
  const uint32_t remainder = value & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1u);
  if (remainder > halfway) return kept + 1u;
  if (remainder < halfway) return kept;
  return kept + (kept & 1u);
}

uint16_t read_f16_le(const uint8_t* bytes, size_t group_index) {
  return static_cast<uint16_t>(bytes[group_index * 2] | (bytes[group_index * 2 + 1] << 8));
}

void write_f16_le(uint8_t* bytes, size_t group_index, uint16_t bits) {
  bytes[group_index * 2] = static_cast<uint8_t>(bits & 0xFF);
  bytes[group_index * 2 + 1] = static_cast<uint8_t>(bits >> 8);
}

// quant.zig:280-288
int32_t quantize_one(float value, float stored_scale, int32_t min_code, int32_t max_code) {
  if (stored_scale == 0.0f) return 0;
  const float scaled = value / stored_scale;
  const float rounded = scaled >= 0.0f ? std::floor(scaled + 0.5f) : std::ceil(scaled - 0.5f);
  if (rounded <= static_cast<float>(min_code)) return min_code;
  if (rounded >= static_cast<float>(max_code)) return max_code;
  return static_cast<int32_t>(rounded);
}

// quant.zig:229-278
void quantize_group(int format, const float* values, float stored_scale, uint8_t* codes) {
  const int32_t shift = orc_bias(format);
  const int32_t min_code = -shift;
  const int32_t max_code = shift - 1;
  switch (format) {
    case ORC_Q4:
      std::memset(codes, 0, 32);
      for (uint32_t i = 0; i < kGroup; ++i) {
        const uint8_t u = static_cast<uint8_t>(quantize_one(values[i], stored_scale, min_code, max_code) + shift);
        codes[i / 2] |= (i % 2 == 0) ? u : static_cast<uint8_t>(u << 4);
      }
      break;
    case ORC_Q5:
      std::memset(codes, 0, 40);
      for (uint32_t i = 0; i < kGroup; ++i) {
        const uint8_t u = static_cast<uint8_t>(quantize_one(values[i], stored_scale, min_code, max_code) + shift);
        const uint8_t low = u & 0x0F;
        codes[i / 2] |= (i % 2 == 0) ? low : static_cast<uint8_t>(low << 4);
        if (u & 0x10) codes[32 + i / 8] |= static_cast<uint8_t>(1u << (i % 8));
      }
      break;
    case ORC_Q8:
      for (uint32_t i = 0; i < kGroup; ++i) {
        codes[i] = static_cast<uint8_t>(quantize_one(values[i], stored_scale, min_code, max_code) + shift);
      }
      break;
    default:
      std::abort();
  }
}

// quant.zig:315-345
void dequantize_group(int format, const uint8_t* codes, float scale, float* out) {
  const int32_t shift = orc_bias(format);
  switch (format) {
    case ORC_Q4:
      for (uint32_t i = 0; i < kGroup; ++i) {
        const uint8_t byte = codes[i / 2];
        const uint8_t nibble = (i % 2 == 0) ? (byte & 0x0F) : (byte >> 4);
        out[i] = static_cast<float>(static_cast<int32_t>(nibble) - shift);
      }
      break;
    case ORC_Q5:
      for (uint32_t i = 0; i < kGroup; ++i) {
        const uint8_t byte = codes[i / 2];
        const uint32_t low = (i % 2 == 0) ? (byte & 0x0F) : (byte >> 4);
        const uint32_t high = (codes[32 + i / 8] >> (i % 8)) & 1u;
        out[i] = static_cast<float>(static_cast<int32_t>(low | (high << 4)) - shift);
      }
      break;
    case ORC_Q8:
      for (uint32_t i = 0; i < kGroup; ++i) out[i] = static_cast<float>(static_cast<int32_t>(codes[i]) - shift);
      break;
    default:
      std::abort();
  }
  for (uint32_t i = 0; i < kGroup; ++i) out[i] *= scale;
}

// Runs fn(begin, end) over [0, n) on up to `threads` threads. Each index is
// computed identically whatever the split, so results do not depend on it.
template <typename Fn>
void parallel_rows(size_t n, int threads, size_t work_per_row, Fn fn) {
  const size_t min_work = size_t(1) << 18;
  if (threads <= 1 || n < 2 || n * work_per_row < min_work) {
    fn(size_t(0), n);
    return;
  }
  const size_t count = std::min<size_t>(static_cast<size_t>(threads), n);
  std::vector<std::thread> pool;
  pool.reserve(count);
  for (size_t t = 0; t < count; ++t) {
    const size_t begin = n * t / count;
    const size_t end = n * (t + 1) / count;
    pool.emplace_back([=] { fn(begin, end); });
  }
  for (auto& thread : pool) thread.join();
}

// kernels.zig:636-661
float q8_group_dot(const float* query_row, const uint8_t* codes, const uint8_t* scales, size_t first_group,
                   uint32_t groups) {
  float total = 0.0f;
  for (uint32_t g = 0; g < groups; ++g) {
    const size_t base = size_t(g) * kGroup;
    const float scale = orc_from_f16(read_f16_le(scales, first_group + g));
    float i0 = 0.0f, i1 = 0.0f, i2 = 0.0f, i3 = 0.0f;
    for (uint32_t index = 0; index < kGroup; index += 4) {
      const float c0 = static_cast<float>(codes[base + index + 0]) - 128.0f;
      const float c1 = static_cast<float>(codes[base + index + 1]) - 128.0f;
      const float c2 = static_cast<float>(codes[base + index + 2]) - 128.0f;
      const float c3 = static_cast<float>(codes[base + index + 3]) - 128.0f;
      i0 = i0 + c0 * query_row[base + index + 0];
      i1 = i1 + c1 * query_row[base + index + 1];
      i2 = i2 + c2 * query_row[base + index + 2];
      i3 = i3 + c3 * query_row[base + index + 3];
    }
    total = total + (((i0 + i1) + i2) + i3) * scale;
  }
  return total;
}

// kernels.zig:665-688
void q8_group_accumulate(float* out_row, const uint8_t* codes, const uint8_t* scales, size_t first_group,
                         uint32_t groups, float weight) {
  for (uint32_t g = 0; g < groups; ++g) {
    const size_t base = size_t(g) * kGroup;
    const float scale = orc_from_f16(read_f16_le(scales, first_group + g));
    const float scaled_weight = scale * weight;
    for (uint32_t index = 0; index < kGroup; ++index) {
      const float centred = static_cast<float>(codes[base + index]) - 128.0f;
      out_row[base + index] = out_row[base + index] + centred * scaled_weight;
    }
  }
}

}  // namespace

extern "C" {

// half_float.zig:14-17 (round to nearest, ties to even; overflow saturates to infinity)
uint16_t orc_to_f16(float value) {
  uint32_t bits;
  std::memcpy(&bits, &value, 4);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const uint32_t exponent = (bits >> 23) & 0xFFu;
  uint32_t mantissa = bits & 0x7FFFFFu;
  if (exponent == 0xFF) return static_cast<uint16_t>(sign | 0x7C00u | (mantissa ? 0x200u : 0u));
  const int32_t half_exponent = static_cast<int32_t>(exponent) - 127 + 15;
  if (half_exponent >= 0x1F) return static_cast<uint16_t>(sign | 0x7C00u);
  if (half_exponent <= 0) {
    if (half_exponent < -10) return static_cast<uint16_t>(sign);
    mantissa |= 0x800000u;
    return static_cast<uint16_t>(sign | round_shift_right(mantissa, static_cast<uint32_t>(14 - half_exponent)));
  }
  const uint32_t rounded = round_shift_right(mantissa, 13);
  // A carry out of the mantissa bumps the exponent, up to infinity: exactly RNE.
  return static_cast<uint16_t>(sign | ((static_cast<uint32_t>(half_exponent) << 10) + rounded));
}

// half_float.zig:20-23
float orc_from_f16(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const uint32_t exponent = (h >> 10) & 0x1Fu;
  const uint32_t mantissa = h & 0x3FFu;
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
    } else {
      float magnitude = std::ldexp(static_cast<float>(mantissa), -24);
      std::memcpy(&bits, &magnitude, 4);
      bits |= sign;
    }
  } else if (exponent == 31) {
    bits = sign | 0x7F800000u | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// quant.zig:52-63, 101-118
uint32_t orc_data_bytes_per_group(int format) {
  switch (format) {
    case ORC_Q4: return 32;
    case ORC_Q5: return 40;
    case ORC_Q8: return 64;
    default: return 0;
  }
}

int32_t orc_bias(int format) {
  switch (format) {
    case ORC_Q4: return 8;
    case ORC_Q5: return 16;
    case ORC_Q8: return 128;
    default: return 0;
  }
}

// quant.zig:197-227
void orc_quantize_row(int format, const float* values, size_t cols, uint8_t* scales_out, uint8_t* data_out) {
  const size_t groups = cols / kGroup;
  const uint32_t data_bytes = orc_data_bytes_per_group(format);
  for (size_t g = 0; g < groups; ++g) {
    const float* group_values = values + g * kGroup;
    float max_abs = 0.0f;
    for (uint32_t i = 0; i < kGroup; ++i) max_abs = std::max(max_abs, std::fabs(group_values[i]));
    const float denominator = static_cast<float>(orc_bias(format));
    const uint16_t scale_bits = orc_to_f16(max_abs / denominator);
    write_f16_le(scales_out, g, scale_bits);
    // Quantize against the *stored* f16 scale (quant.zig:221-225).
    const float stored_scale = orc_from_f16(scale_bits);
    quantize_group(format, group_values, stored_scale, data_out + g * data_bytes);
  }
}

void orc_quantize_rows(int format, const float* values, size_t rows, size_t cols, uint8_t* scales_out,
                       uint8_t* data_out, int threads) {
  const size_t groups = cols / kGroup;
  const size_t data_row = groups * orc_data_bytes_per_group(format);
  parallel_rows(rows, threads, cols, [&](size_t begin, size_t end) {
    for (size_t r = begin; r < end; ++r) {
      orc_quantize_row(format, values + r * cols, cols, scales_out + r * groups * 2, data_out + r * data_row);
    }
  });
}

// quant.zig:348-364
void orc_dequantize_row(int format, const uint8_t* scales, const uint8_t* data, size_t cols, float* out) {
  const size_t groups = cols / kGroup;
  const uint32_t data_bytes = orc_data_bytes_per_group(format);
  for (size_t g = 0; g < groups; ++g) {
    const float scale = orc_from_f16(read_f16_le(scales, g));
    dequantize_group(format, data + g * data_bytes, scale, out + g * kGroup);
  }
}

// quant.zig:370-391
float orc_dot_row(int format, const uint8_t* scales, const uint8_t* data, const float* x, size_t cols) {
  const size_t groups = cols / kGroup;
  const uint32_t data_bytes = orc_data_bytes_per_group(format);
  float accumulator = 0.0f;
  float codes[kGroup];
  for (size_t g = 0; g < groups; ++g) {
    const float scale = orc_from_f16(read_f16_le(scales, g));
    dequantize_group(format, data + g * data_bytes, scale, codes);
    for (uint32_t i = 0; i < kGroup; ++i) accumulator = accumulator + codes[i] * x[g * kGroup + i];
  }
  return accumulator;
}

// kernels.zig:39-51
float orc_dot_f32(const float* a, const float* b, size_t n) {
  float l0 = 0.0f, l1 = 0.0f, l2 = 0.0f, l3 = 0.0f;
  size_t i = 0;
  for (; i + 4 <= n; i += 4) {
    l0 = l0 + a[i + 0] * b[i + 0];
    l1 = l1 + a[i + 1] * b[i + 1];
    l2 = l2 + a[i + 2] * b[i + 2];
    l3 = l3 + a[i + 3] * b[i + 3];
  }
  float total = ((l0 + l1) + l2) + l3;
  for (; i < n; ++i) total = total + a[i] * b[i];
  return total;
}

// kernels.zig:118-158: a row's codes are decoded once into scratch and dotted
// with every token's activation row.
int32_t orc_linear_quantized(float* out, const float* x, int format, const uint8_t* scales, const uint8_t* data,
                             uint32_t rows, uint32_t cols, uint32_t tokens, int threads) {
  if (cols % kGroup != 0) return kShapeMismatch;
  const size_t groups = cols / kGroup;
  const size_t data_row = groups * orc_data_bytes_per_group(format);
  parallel_rows(rows, threads, size_t(cols) * tokens, [&](size_t begin, size_t end) {
    std::vector<float> scratch(cols);
    for (size_t r = begin; r < end; ++r) {
      orc_dequantize_row(format, scales + r * groups * 2, data + r * data_row, cols, scratch.data());
      for (uint32_t t = 0; t < tokens; ++t) {
        out[size_t(t) * rows + r] = orc_dot_f32(scratch.data(), x + size_t(t) * cols, cols);
      }
    }
  });
  return kOk;
}

// kernels.zig:288-300 -> math.zig:120-130
void orc_rmsnorm(float* x, const float* weight, uint32_t width, uint32_t tokens, float eps) {
  for (uint32_t t = 0; t < tokens; ++t) {
    float* row = x + size_t(t) * width;
    float sum_squares = 0.0f;
    for (uint32_t i = 0; i < width; ++i) sum_squares = sum_squares + row[i] * row[i];
    const float mean_square = sum_squares / static_cast<float>(width);
    const float inverse_rms = 1.0f / std::sqrt(mean_square + eps);
    for (uint32_t i = 0; i < width; ++i) row[i] = row[i] * inverse_rms * weight[i];
  }
}

// math.zig:69-71
float orc_silu(float x) { return x / (1.0f + std::exp(-x)); }

// kernels.zig:233-239
void orc_silu_mul(float* out, const float* gate, const float* up, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = orc_silu(gate[i]) * up[i];
}

// math.zig:77-93
void orc_softmax(float* row, size_t n) {
  float row_max = row[0];
  for (size_t i = 1; i < n; ++i) row_max = std::max(row_max, row[i]);
  float total = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    row[i] = std::exp(row[i] - row_max);
    total = total + row[i];
  }
  const float inverse_total = 1.0f / total;
  for (size_t i = 0; i < n; ++i) row[i] *= inverse_total;
}

// std.math.pow(f32, x, y) as Zig's standard library computes it (the
// published algorithm of Go's math.Pow: x^y = exp(yf*log x) * x^yi by
// repeated squaring, all in f32), restricted to finite x > 0 and finite y,
// which is the only domain kernels.zig:561-564 reaches.
float orc_pow_f32(float x, float y) {
  if (y == 0.0f || x == 1.0f) return 1.0f;
  if (std::isnan(x) || std::isnan(y)) return std::nanf("");
  if (y == 1.0f) return x;
  if (y == 0.5f) return std::sqrt(x);
  if (y == -0.5f) return 1.0f / std::sqrt(x);
  float yi_part;
  float yf = std::modf(std::fabs(y), &yi_part);
  float yi = yi_part;
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
    const int32_t overflow_shift = 8 + 1;
    if (xe < -(1 << overflow_shift) || (1 << overflow_shift) < xe) {
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

// kernels.zig:561-564
float orc_inverse_frequency(uint32_t index, uint32_t head_dim, float theta) {
  const float exponent = -2.0f * static_cast<float>(index) / static_cast<float>(head_dim);
  return orc_pow_f32(theta, exponent);
}

// kernels.zig:534-558
void orc_build_rope_tables(float* cos_table, float* sin_table, uint32_t half, float theta, uint32_t max_positions,
                           uint32_t stride) {
  const uint32_t head_dim = half * 2;
  for (uint32_t position = 0; position < max_positions; ++position) {
    for (uint32_t index = 0; index < half; ++index) {
      const float angle = static_cast<float>(position) * orc_inverse_frequency(index, head_dim, theta);
      const size_t offset = size_t(position) * stride + index;
      cos_table[offset] = std::cos(angle);
      sin_table[offset] = std::sin(angle);
    }
  }
}

// kernels.zig:495-527 (rotate_half pairing)
void orc_rope(float* rotated, const uint32_t* positions, uint32_t n_positions, uint32_t heads, uint32_t head_dim,
              const float* cos_table, const float* sin_table, uint32_t table_stride) {
  const uint32_t width = heads * head_dim;
  const uint32_t half = head_dim / 2;
  for (uint32_t token = 0; token < n_positions; ++token) {
    const float* cos_row = cos_table + size_t(positions[token]) * table_stride;
    const float* sin_row = sin_table + size_t(positions[token]) * table_stride;
    for (uint32_t head = 0; head < heads; ++head) {
      float* row = rotated + size_t(token) * width + size_t(head) * head_dim;
      for (uint32_t i = 0; i < half; ++i) {
        const float low = row[i];
        const float high = row[i + half];
        row[i] = low * cos_row[i] - high * sin_row[i];
        row[i + half] = high * cos_row[i] + low * sin_row[i];
      }
    }
  }
}

// kernels.zig:572-627
int32_t orc_decode_attention_f32(float* out, const float* query, const float* keys, const float* values,
                                 uint32_t cached, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, float* scores) {
  if (heads % kv_heads != 0) return kShapeMismatch;
  const uint32_t kv_width = kv_heads * head_dim;
  const uint32_t groups = heads / kv_heads;
  const float scaling = 1.0f / std::sqrt(static_cast<float>(head_dim));
  for (uint32_t head = 0; head < heads; ++head) {
    const float* head_query = query + size_t(head) * head_dim;
    const uint32_t kv_head = head / groups;
    for (uint32_t p = 0; p < cached; ++p) {
      scores[p] = orc_dot_f32(head_query, keys + size_t(p) * kv_width + size_t(kv_head) * head_dim, head_dim) * scaling;
    }
    orc_softmax(scores, cached);
    float* head_out = out + size_t(head) * head_dim;
    std::memset(head_out, 0, sizeof(float) * head_dim);
    for (uint32_t p = 0; p < cached; ++p) {
      const float* value_row = values + size_t(p) * kv_width + size_t(kv_head) * head_dim;
      const float weight = scores[p];
      for (uint32_t i = 0; i < head_dim; ++i) head_out[i] = head_out[i] + value_row[i] * weight;
    }
  }
  return kOk;
}

// kernels.zig:697-767
int32_t orc_decode_attention_q8(float* out, const float* query, const uint8_t* keys_scales, const uint8_t* keys_codes,
                                const uint8_t* values_scales, const uint8_t* values_codes, uint32_t cached,
                                uint32_t heads, uint32_t kv_heads, uint32_t head_dim, float* scores) {
  if (head_dim % kGroup != 0 || heads % kv_heads != 0) return kShapeMismatch;
  const uint32_t kv_width = kv_heads * head_dim;
  const uint32_t groups_per_row = kv_width / kGroup;
  const uint32_t groups = heads / kv_heads;
  const uint32_t groups_per_head = head_dim / kGroup;
  const float scaling = 1.0f / std::sqrt(static_cast<float>(head_dim));
  for (uint32_t head = 0; head < heads; ++head) {
    const float* head_query = query + size_t(head) * head_dim;
    const uint32_t kv_head = head / groups;
    const size_t head_group = size_t(kv_head) * head_dim / kGroup;
    for (uint32_t p = 0; p < cached; ++p) {
      const size_t row_group = size_t(p) * groups_per_row + head_group;
      const uint8_t* codes = keys_codes + size_t(p) * kv_width + size_t(kv_head) * head_dim;
      scores[p] = scaling * q8_group_dot(head_query, codes, keys_scales, row_group, groups_per_head);
    }
    orc_softmax(scores, cached);
    float* head_out = out + size_t(head) * head_dim;
    std::memset(head_out, 0, sizeof(float) * head_dim);
    for (uint32_t p = 0; p < cached; ++p) {
      const size_t row_group = size_t(p) * groups_per_row + head_group;
      const uint8_t* codes = values_codes + size_t(p) * kv_width + size_t(kv_head) * head_dim;
      q8_group_accumulate(head_out, codes, values_scales, row_group, groups_per_head, scores[p]);
    }
  }
  return kOk;
}

// decoder.zig:290-301: strict `>`, so the first (lowest) index of equal maxima wins.
uint32_t orc_argmax(const float* values, size_t n) {
  uint32_t best = 0;
  float best_value = values[0];
  for (size_t i = 1; i < n; ++i) {
    if (values[i] > best_value) {
      best_value = values[i];
      best = static_cast<uint32_t>(i);
    }
  }
  return best;
}

// selftest.zig:73-126 (the quantizer half of checkQuantization): FNV-1a 64
// over the q4, q5 and q8 planes of cos(i * 0.19) * 1.75, 128 values.
uint64_t orc_quant_hash(void) {
  const size_t cols = 128;
  float values[cols];
  for (size_t i = 0; i < cols; ++i) values[i] = std::cos(static_cast<float>(i) * 0.19f) * 1.75f;
  uint64_t hash = 0xcbf29ce484222325ull;
  auto update = [&](const uint8_t* bytes, size_t len) {
    for (size_t i = 0; i < len; ++i) {
      hash ^= bytes[i];
      hash *= 0x100000001b3ull;
    }
  };
  const int formats[3] = {ORC_Q4, ORC_Q5, ORC_Q8};
  for (int format : formats) {
    uint8_t scales[cols / kGroup * 2];
    uint8_t data[cols / kGroup * 64];
    const size_t data_len = cols / kGroup * orc_data_bytes_per_group(format);
    orc_quantize_row(format, values, cols, scales, data);
    update(scales, sizeof(scales));
    update(data, data_len);
  }
  return hash;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// The decoder: model.zig (weights, scratch, KV layout) and decoder.zig.
// ---------------------------------------------------------------------------

namespace {

// model_config.zig:110-177, byte for byte.
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
static_assert(sizeof(Config) == 160, "Config is 160 bytes (model_config.zig:364)");
static_assert(offsetof(Config, text_hidden_size) == 60, "model_config.zig:372");
static_assert(offsetof(Config, token_audio_start) == 104, "model_config.zig:373");
static_assert(offsetof(Config, flags) == 144, "model_config.zig:374");

// container.zig:333-376 (decoder part)
enum Kind : uint32_t {
  kEmbedTokens = 30,
  kFinalNorm = 31,
  kOutput = 32,
  kQ = 33,
  kK = 34,
  kV = 35,
  kO = 36,
  kQNorm = 37,
  kKNorm = 38,
  kAttnNorm = 39,
  kFfnNorm = 40,
  kGate = 41,
  kUp = 42,
  kDown = 43,
};

// kernels.zig:161-168 (the quantized arm; f32 vectors for norms)
struct Matrix {
  int format = -1;
  uint32_t rows = 0, cols = 0;
  const uint8_t* scales = nullptr;
  const uint8_t* data = nullptr;
  const float* f32 = nullptr;
  bool present() const { return format >= 0; }
};

struct Layer {
  Matrix q, k, v, o, gate, up, down;
  const float* q_norm = nullptr;
  const float* k_norm = nullptr;
  const float* attn_norm = nullptr;
  const float* ffn_norm = nullptr;
};

}  // namespace

struct OrcModel {
  Config config;
  uint32_t cache_format = 1;
  int threads = 1;
  bool finished = false;
  Matrix embed, output;
  const float* final_norm = nullptr;
  std::vector<Layer> layers;
  // model.zig:154-203 (decoder part)
  std::vector<float> hidden, normed, query, key, value, attention_out, gate, up, position_scores, logits, rope_cos,
      rope_sin, cache_keys, cache_values;
  std::vector<uint8_t> cache_keys_q8, cache_values_q8;
  uint32_t position = 0;

  uint32_t kv_width() const { return config.text_key_value_heads * config.text_head_dim; }
  uint32_t q_width() const { return config.text_attention_heads * config.text_head_dim; }
};

namespace {

int32_t apply(const OrcModel* m, const Matrix& w, float* out, const float* x) {
  return orc_linear_quantized(out, x, w.format, w.scales, w.data, w.rows, w.cols, 1, m->threads);
}

// decoder.zig:58-65
struct CachePlane {
  size_t scales, codes, stride;
};

CachePlane cache_plane(const OrcModel* m) {
  const size_t groups_per_row = m->kv_width() / kGroup;
  const size_t scales = size_t(m->config.max_positions) * groups_per_row * 2;
  const size_t codes = size_t(m->config.max_positions) * m->kv_width();
  return {scales, codes, scales + codes};
}

// decoder.zig:68-106
void append_cache_row(OrcModel* m, uint32_t layer, uint32_t position, const float* key, const float* value) {
  const uint32_t row_width = m->kv_width();
  if (m->cache_format == 0) {
    const size_t stride = size_t(m->config.max_positions) * row_width;
    const size_t offset = size_t(layer) * stride + size_t(position) * row_width;
    std::memcpy(m->cache_keys.data() + offset, key, row_width * sizeof(float));
    std::memcpy(m->cache_values.data() + offset, value, row_width * sizeof(float));
    return;
  }
  const CachePlane plane = cache_plane(m);
  const size_t layer_offset = size_t(layer) * plane.stride;
  const size_t scale_bytes = size_t(row_width / kGroup) * 2;
  const size_t scale_offset = layer_offset + size_t(position) * scale_bytes;
  const size_t code_offset = layer_offset + plane.scales + size_t(position) * row_width;
  orc_quantize_row(ORC_Q8, key, row_width, m->cache_keys_q8.data() + scale_offset,
                   m->cache_keys_q8.data() + code_offset);
  orc_quantize_row(ORC_Q8, value, row_width, m->cache_values_q8.data() + scale_offset,
                   m->cache_values_q8.data() + code_offset);
}

// decoder.zig:346-376 (quantized arm)
void embedding_row(const OrcModel* m, uint32_t row, float* out) {
  const Matrix& e = m->embed;
  const uint32_t cols = m->config.text_hidden_size;
  const size_t groups = cols / kGroup;
  orc_dequantize_row(e.format, e.scales + size_t(row) * groups * 2,
                     e.data + size_t(row) * groups * orc_data_bytes_per_group(e.format), cols, out);
}

// quant.zig:144-176 with a 16-byte-aligned base: scales at 0, codes at the next 16-byte boundary.
bool bind_planes(Matrix& m, int format, uint32_t rows, uint32_t cols, const void* payload, size_t len) {
  if (cols % kGroup != 0) return false;
  const size_t groups = size_t(rows) * (cols / kGroup);
  const size_t scales_len = groups * 2;
  const size_t data_offset = (scales_len + 15) / 16 * 16;
  const size_t data_len = groups * orc_data_bytes_per_group(format);
  if (len < data_offset + data_len) return false;
  m.format = format;
  m.rows = rows;
  m.cols = cols;
  m.scales = static_cast<const uint8_t*>(payload);
  m.data = static_cast<const uint8_t*>(payload) + data_offset;
  return true;
}

}  // namespace

extern "C" {

OrcModel* orc_model_new(const void* config, uint32_t config_len, uint32_t cache_format) {
  if (config_len != sizeof(Config) || cache_format > 1) return nullptr;
  auto* m = new OrcModel();
  std::memcpy(&m->config, config, sizeof(Config));
  m->cache_format = cache_format;
  m->layers.resize(m->config.text_layers);
  return m;
}

void orc_model_free(OrcModel* model) { delete model; }

void orc_model_set_threads(OrcModel* model, int threads) { model->threads = threads < 1 ? 1 : threads; }

int32_t orc_model_set_tensor(OrcModel* m, uint32_t kind, uint32_t layer, uint32_t format, uint32_t rows, uint32_t cols,
                             const void* payload, size_t len) {
  const bool vector_kind = kind == kFinalNorm || kind == kQNorm || kind == kKNorm || kind == kAttnNorm ||
                           kind == kFfnNorm;
  if (vector_kind) {
    if (format != ORC_F32 || len < size_t(rows) * cols * 4) return kShapeMismatch;
    const float* values = static_cast<const float*>(payload);
    if (kind == kFinalNorm) {
      m->final_norm = values;
      return kOk;
    }
    if (layer < 1 || layer > m->config.text_layers) return kInvalidArgument;
    Layer& l = m->layers[layer - 1];
    if (kind == kQNorm) l.q_norm = values;
    if (kind == kKNorm) l.k_norm = values;
    if (kind == kAttnNorm) l.attn_norm = values;
    if (kind == kFfnNorm) l.ffn_norm = values;
    return kOk;
  }
  if (format != ORC_Q4 && format != ORC_Q5 && format != ORC_Q8) return kUnsupportedModel;
  Matrix mat;
  if (!bind_planes(mat, static_cast<int>(format), rows, cols, payload, len)) return kShapeMismatch;
  if (kind == kEmbedTokens) {
    m->embed = mat;
    return kOk;
  }
  if (kind == kOutput) {
    m->output = mat;
    return kOk;
  }
  if (layer < 1 || layer > m->config.text_layers) return kInvalidArgument;
  Layer& l = m->layers[layer - 1];
  switch (kind) {
    case kQ: l.q = mat; break;
    case kK: l.k = mat; break;
    case kV: l.v = mat; break;
    case kO: l.o = mat; break;
    case kGate: l.gate = mat; break;
    case kUp: l.up = mat; break;
    case kDown: l.down = mat; break;
    default: return kInvalidArgument;
  }
  return kOk;
}

// model.zig:316-409 (decoder part) and allocateScratch (:1011-1088)
int32_t orc_model_finish(OrcModel* m) {
  const Config& c = m->config;
  if (!m->embed.present() || m->final_norm == nullptr) return kNotFound;
  const bool tied = (c.flags & 1u) != 0;
  if (!tied) {
    if (!m->output.present()) return kNotFound;
  } else {
    m->output = m->embed;  // model.zig:391-394
  }
  for (const Layer& l : m->layers) {
    if (!l.q.present() || !l.k.present() || !l.v.present() || !l.o.present() || !l.gate.present() ||
        !l.up.present() || !l.down.present() || !l.q_norm || !l.k_norm || !l.attn_norm || !l.ffn_norm) {
      return kNotFound;
    }
  }
  if (c.max_positions == 0 || c.max_positions > 8192) return kLimitExceeded;  // model.zig:62, :1006-1009
  const size_t hidden = c.text_hidden_size;
  m->hidden.assign(hidden, 0.0f);
  m->normed.assign(std::max<size_t>(hidden, 1), 0.0f);
  m->query.assign(m->q_width(), 0.0f);
  m->key.assign(m->kv_width(), 0.0f);
  m->value.assign(m->kv_width(), 0.0f);
  m->attention_out.assign(m->q_width(), 0.0f);
  m->gate.assign(c.text_ffn_dim, 0.0f);
  m->up.assign(c.text_ffn_dim, 0.0f);
  m->position_scores.assign(c.max_positions, 0.0f);
  m->logits.assign(c.vocab_size, 0.0f);
  const uint32_t half = c.text_head_dim / 2;
  m->rope_cos.assign(size_t(c.max_positions) * half, 0.0f);
  m->rope_sin.assign(size_t(c.max_positions) * half, 0.0f);
  orc_build_rope_tables(m->rope_cos.data(), m->rope_sin.data(), half, c.rope_theta, c.max_positions, half);
  if (m->cache_format == 0) {
    m->cache_keys.assign(size_t(c.text_layers) * c.max_positions * m->kv_width(), 0.0f);
    m->cache_values.assign(m->cache_keys.size(), 0.0f);
  } else {
    const CachePlane plane = cache_plane(m);
    m->cache_keys_q8.assign(size_t(c.text_layers) * plane.stride, 0);
    m->cache_values_q8.assign(m->cache_keys_q8.size(), 0);
  }
  m->position = 0;
  m->finished = true;
  return kOk;
}

// decoder.zig:109-121
void orc_decoder_reset(OrcModel* m) {
  m->position = 0;
  std::fill(m->cache_keys.begin(), m->cache_keys.end(), 0.0f);
  std::fill(m->cache_values.begin(), m->cache_values.end(), 0.0f);
  std::fill(m->cache_keys_q8.begin(), m->cache_keys_q8.end(), 0);
  std::fill(m->cache_values_q8.begin(), m->cache_values_q8.end(), 0);
}

uint32_t orc_decoder_position(const OrcModel* m) { return m->position; }

int32_t orc_decoder_set_state(OrcModel* m, const uint8_t* keys, const uint8_t* values, uint64_t len,
                              uint32_t position) {
  if (!m->finished || m->cache_format != 1) return kInvalidState;
  if (len != m->cache_keys_q8.size() || position > m->config.max_positions) return kShapeMismatch;
  std::memcpy(m->cache_keys_q8.data(), keys, len);
  std::memcpy(m->cache_values_q8.data(), values, len);
  m->position = position;
  return kOk;
}

// decoder.zig:133-287
int32_t orc_forward_token(OrcModel* m, uint32_t token, const float* audio_row, int want_logits) {
  if (!m->finished) return kInvalidState;
  const Config& c = m->config;
  const uint32_t hidden_size = c.text_hidden_size;
  if (m->position >= c.max_positions) return kLimitExceeded;  // PositionExceeded
  float* hidden = m->hidden.data();
  if (audio_row) {
    std::memcpy(hidden, audio_row, hidden_size * sizeof(float));
  } else {
    if (token >= m->embed.rows) return kShapeMismatch;
    embedding_row(m, token, hidden);
  }
  float* normed = m->normed.data();
  float* query = m->query.data();
  float* key = m->key.data();
  float* value = m->value.data();
  const uint32_t kv_width = m->kv_width();
  const uint32_t half_head = c.text_head_dim / 2;
  for (uint32_t li = 0; li < c.text_layers; ++li) {
    const Layer& layer = m->layers[li];
    // rmsNormInto: copy then normalize in place.
    std::memcpy(normed, hidden, hidden_size * sizeof(float));
    orc_rmsnorm(normed, layer.attn_norm, hidden_size, 1, c.text_rms_norm_eps);
    apply(m, layer.q, query, normed);
    apply(m, layer.k, key, normed);
    apply(m, layer.v, value, normed);
    orc_rmsnorm(query, layer.q_norm, c.text_head_dim, c.text_attention_heads, c.text_rms_norm_eps);
    orc_rmsnorm(key, layer.k_norm, c.text_head_dim, c.text_key_value_heads, c.text_rms_norm_eps);
    const uint32_t single_position[1] = {m->position};
    orc_rope(query, single_position, 1, c.text_attention_heads, c.text_head_dim, m->rope_cos.data(),
             m->rope_sin.data(), half_head);
    orc_rope(key, single_position, 1, c.text_key_value_heads, c.text_head_dim, m->rope_cos.data(), m->rope_sin.data(),
             half_head);
    append_cache_row(m, li, m->position, key, value);
    if (m->cache_format == 0) {
      const size_t layer_offset = size_t(li) * c.max_positions * kv_width;
      orc_decode_attention_f32(m->attention_out.data(), query, m->cache_keys.data() + layer_offset,
                               m->cache_values.data() + layer_offset, m->position + 1, c.text_attention_heads,
                               c.text_key_value_heads, c.text_head_dim, m->position_scores.data());
    } else {
      const CachePlane plane = cache_plane(m);
      const size_t layer_offset = size_t(li) * plane.stride;
      orc_decode_attention_q8(m->attention_out.data(), query, m->cache_keys_q8.data() + layer_offset,
                              m->cache_keys_q8.data() + layer_offset + plane.scales,
                              m->cache_values_q8.data() + layer_offset,
                              m->cache_values_q8.data() + layer_offset + plane.scales, m->position + 1,
                              c.text_attention_heads, c.text_key_value_heads, c.text_head_dim,
                              m->position_scores.data());
    }
    apply(m, layer.o, normed, m->attention_out.data());
    for (uint32_t i = 0; i < hidden_size; ++i) hidden[i] = hidden[i] + normed[i];
    std::memcpy(normed, hidden, hidden_size * sizeof(float));
    orc_rmsnorm(normed, layer.ffn_norm, hidden_size, 1, c.text_rms_norm_eps);
    apply(m, layer.gate, m->gate.data(), normed);
    apply(m, layer.up, m->up.data(), normed);
    orc_silu_mul(m->gate.data(), m->gate.data(), m->up.data(), c.text_ffn_dim);
    apply(m, layer.down, normed, m->gate.data());
    for (uint32_t i = 0; i < hidden_size; ++i) hidden[i] = hidden[i] + normed[i];
  }
  m->position += 1;
  if (!want_logits) return kOk;
  std::memcpy(normed, hidden, hidden_size * sizeof(float));
  orc_rmsnorm(normed, m->final_norm, hidden_size, 1, c.text_rms_norm_eps);
  apply(m, m->output, m->logits.data(), normed);
  return kOk;
}

uint32_t orc_argmax_logits(const OrcModel* m) { return orc_argmax(m->logits.data(), m->logits.size()); }

// decoder.zig:308-333
int32_t orc_prefill(OrcModel* m, const uint32_t* tokens, uint32_t n_tokens, const float* audio, uint32_t audio_steps,
                    uint32_t* next_out) {
  if (n_tokens == 0) return kShapeMismatch;
  const uint32_t hidden_size = m->config.text_hidden_size;
  uint32_t audio_index = 0;
  for (uint32_t i = 0; i < n_tokens; ++i) {
    const int is_last = (i + 1 == n_tokens) ? 1 : 0;
    int32_t status;
    if (tokens[i] == m->config.token_audio_pad) {
      if (audio_index >= audio_steps) return kShapeMismatch;  // PromptMismatch
      status = orc_forward_token(m, tokens[i], audio + size_t(audio_index) * hidden_size, is_last);
      audio_index += 1;
    } else {
      status = orc_forward_token(m, tokens[i], nullptr, is_last);
    }
    if (status != kOk) return status;
  }
  if (audio_index != audio_steps) return kShapeMismatch;
  *next_out = orc_argmax_logits(m);
  return kOk;
}

// decoder.zig:336-339
int32_t orc_step(OrcModel* m, uint32_t token, uint32_t* next_out) {
  const int32_t status = orc_forward_token(m, token, nullptr, 1);
  if (status != kOk) return status;
  *next_out = orc_argmax_logits(m);
  return kOk;
}

const float* orc_logits(const OrcModel* m) { return m->logits.data(); }
const float* orc_hidden(const OrcModel* m) { return m->hidden.data(); }

const float* orc_scratch(const OrcModel* m, int which, uint32_t* count_out) {
  const std::vector<float>* v = nullptr;
  switch (which) {
    case 0: v = &m->hidden; break;
    case 1: v = &m->query; break;
    case 2: v = &m->key; break;
    case 3: v = &m->value; break;
    case 4: v = &m->attention_out; break;
    case 5: v = &m->gate; break;
    default: *count_out = 0; return nullptr;
  }
  *count_out = static_cast<uint32_t>(v->size());
  return v->data();
}

const uint8_t* orc_cache_keys_q8(const OrcModel* m, uint64_t* len_out) {
  *len_out = m->cache_keys_q8.size();
  return m->cache_keys_q8.data();
}

const uint8_t* orc_cache_values_q8(const OrcModel* m, uint64_t* len_out) {
  *len_out = m->cache_values_q8.size();
  return m->cache_values_q8.data();
}

const float* orc_rope_cos(const OrcModel* m) { return m->rope_cos.data(); }
const float* orc_rope_sin(const OrcModel* m) { return m->rope_sin.data(); }

}  // extern "C"

// qwc_device.cuh -- device helpers for the sm_100a decoder kernels.
//
// Dequantization strategy (exact): a 4-bit code u sits at bit offset 4*i of a
// 32-bit word. OR-ing the masked nibble into the mantissa of 2^23 gives the
// float 2^23 + u*16^i exactly (i <= 4; nibbles 5..7 are shifted down by 12
// first). Subtracting 2^23 + 8*16^i leaves (u - 8)*16^i exactly, and the
// matching activation is pre-scaled by 16^-i, so every product equals the
// reference's (u - 8) * x (src/core/quant.zig:315-345) before rounding. q8
// bytes go through one byte-permute into 2^23 + b the same way. The
// arithmetic runs on the packed fma.rn.f32x2 / add.rn.f32x2 of sm_100.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>

namespace qwc {

__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ float2 unpack2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

__device__ __forceinline__ float bits_f32(uint32_t b) { return __uint_as_float(b); }

constexpr uint32_t kMagic = 0x4B000000u;  // 2^23
// -(2^23 + 8 * 16^i): the q4 bias of nibble position i after the magic OR.
constexpr float kNegM0 = -8388616.0f;
constexpr float kNegM1 = -8388736.0f;
constexpr float kNegM2 = -8390656.0f;
constexpr float kNegM3 = -8421376.0f;
constexpr float kNegM4 = -8912896.0f;
constexpr float kNegQ8 = -8388736.0f;  // -(2^23 + 128)

// Pre-scale of the activation paired with nibble position i of a word:
// 16^-i for i <= 4, 16^-(i-3) for the shifted nibbles 5..7.
__host__ __device__ constexpr float q4_xscale(int i) {
  return i == 0 ? 1.0f
       : i == 1 ? 0.0625f
       : i == 2 ? 0.00390625f
       : i == 3 ? 0.000244140625f
       : i == 4 ? 0.0000152587890625f
       : i == 5 ? 0.00390625f
       : i == 6 ? 0.000244140625f
                : 0.0000152587890625f;
}

// 1 / (kQ4SubScale * q4_xscale(i)): undoes the q4 activation prescale.
__host__ __device__ constexpr float q4_unscale(int i) {
  return i == 0 ? 0x1p-74f : i == 1 ? 0x1p-70f : (i == 2 || i == 5) ? 0x1p-66f : (i == 3 || i == 6) ? 0x1p-62f
                                                                                                     : 0x1p-58f;
}

// (w & MASK) | magic in one lop3 (LUT 0xEA = (a & b) | c).
template <uint32_t MASK>
__device__ __forceinline__ uint32_t and_or(uint32_t w, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "n"(MASK), "r"(magic));
  return r;
}

// The magic constant in a register the compiler will not fold back into an
// immediate (so each nibble costs one lop3).
__device__ __forceinline__ uint32_t magic_reg() {
  uint32_t m = kMagic;
  asm volatile("" : "+r"(m));
  return m;
}

// Accumulates 8 nibbles of `w` against 4 packed pre-scaled activation pairs.
__device__ __forceinline__ void q4_word(uint32_t w, uint32_t magic, const uint64_t* x2, uint64_t& acc) {
  const uint32_t h = w >> 12;
  const uint64_t v01 = pack2(bits_f32(and_or<0x0000000Fu>(w, magic)), bits_f32(and_or<0x000000F0u>(w, magic)));
  const uint64_t v23 = pack2(bits_f32(and_or<0x00000F00u>(w, magic)), bits_f32(and_or<0x0000F000u>(w, magic)));
  const uint64_t v45 = pack2(bits_f32(and_or<0x000F0000u>(w, magic)), bits_f32(and_or<0x00000F00u>(h, magic)));
  const uint64_t v67 = pack2(bits_f32(and_or<0x0000F000u>(h, magic)), bits_f32(and_or<0x000F0000u>(h, magic)));
  acc = fma2(add2(v01, pack2(kNegM0, kNegM1)), x2[0], acc);
  acc = fma2(add2(v23, pack2(kNegM2, kNegM3)), x2[1], acc);
  acc = fma2(add2(v45, pack2(kNegM4, kNegM2)), x2[2], acc);
  acc = fma2(add2(v67, pack2(kNegM3, kNegM4)), x2[3], acc);
}

// 32 q4 weights (one 16-byte chunk) against 16 packed activation pairs.
__device__ __forceinline__ float q4_chunk_dot(uint4 w, const uint64_t* x2, uint32_t magic) {
  uint64_t a = 0, b = 0;
  q4_word(w.x, magic, x2 + 0, a);
  q4_word(w.y, magic, x2 + 4, b);
  q4_word(w.z, magic, x2 + 8, a);
  q4_word(w.w, magic, x2 + 12, b);
  const float2 fa = unpack2(a), fb = unpack2(b);
  return (fa.x + fa.y) + (fb.x + fb.y);
}

__device__ __forceinline__ float q4_chunk_dot(uint4 w, const uint64_t* x2) { return q4_chunk_dot(w, x2, magic_reg()); }

// The same eight nibbles as subnormal floats: (w & 0xF << p) read as f32 is
// exactly u * 2^(p - 149), with no bias constant to remove. Against
// activations prescaled by 2^(74 - p) the products are u * x * 2^-75, so
// one power-of-two multiply of the sum restores sum(u * x); the bias comes
// out separately as 8 * sum(x) (q4_chunk_xsum). Needs subnormals kept
// (no flush-to-zero), which is the compiler's default.
constexpr float kQ4SubScale = 0x1p74f;   // activation prescale on top of q4_xscale
constexpr float kQ4SubUnscale = 0x1p75f;  // sum(u * x) = kQ4SubUnscale * sum of products
__device__ __forceinline__ void q4_word_sub(uint32_t w, const uint64_t* x2, uint64_t& acc) {
  const uint32_t h = w >> 12;
  acc = fma2(pack2(bits_f32(w & 0xFu), bits_f32(w & 0xF0u)), x2[0], acc);
  acc = fma2(pack2(bits_f32(w & 0xF00u), bits_f32(w & 0xF000u)), x2[1], acc);
  acc = fma2(pack2(bits_f32(w & 0xF0000u), bits_f32(h & 0xF00u)), x2[2], acc);
  acc = fma2(pack2(bits_f32(h & 0xF000u), bits_f32(h & 0xF0000u)), x2[3], acc);
}

// sum(u * x) * 2^-75 over 32 q4 weights (one 16-byte chunk).
__device__ __forceinline__ float q4_chunk_dot_sub(uint4 w, const uint64_t* x2) {
  uint64_t a = 0, b = 0;
  q4_word_sub(w.x, x2 + 0, a);
  q4_word_sub(w.y, x2 + 4, b);
  q4_word_sub(w.z, x2 + 8, a);
  q4_word_sub(w.w, x2 + 12, b);
  const float2 fa = unpack2(a), fb = unpack2(b);
  return (fa.x + fa.y) + (fb.x + fb.y);
}

// sum(x) over the chunk's 32 activations, from their prescaled pairs.
__device__ __forceinline__ float q4_chunk_xsum(const uint64_t* x2) {
  // Undo kQ4SubScale * q4_xscale per pair position: nibble positions
  // (0, 4), (8, 12), (16, 8), (12, 16) bits.
  const uint64_t d0 = pack2(0x1p-74f, 0x1p-70f), d1 = pack2(0x1p-66f, 0x1p-62f);
  const uint64_t d2 = pack2(0x1p-58f, 0x1p-66f), d3 = pack2(0x1p-62f, 0x1p-58f);
  uint64_t a = 0, b = 0;
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    a = fma2(x2[4 * t + 0], d0, a);
    b = fma2(x2[4 * t + 1], d1, b);
    a = fma2(x2[4 * t + 2], d2, a);
    b = fma2(x2[4 * t + 3], d3, b);
  }
  const float2 fa = unpack2(a), fb = unpack2(b);
  return (fa.x + fa.y) + (fb.x + fb.y);
}

// q5 (quant.zig:253-269, 327-335): a group's 32 bytes of low nibbles (the q4
// layout: weight 2i in the low nibble of byte i, 2i + 1 in the high one), then
// 8 bytes of fifth bits (bit i % 8 of byte i / 8 for weight i); the code is
// low | fifth << 4, bias 16. One half group, 32 weights: the low nibbles in
// four words (weight 8 w + p at nibble p of word w), the fifth bits in one word
// (bit i for weight i). (2^23 + u) - (2^23 + 16) = u - 16 is exact in f32.
constexpr float kNegQ5 = -8388624.0f;  // -(2^23 + 16)
__device__ __forceinline__ float q5_half_dot(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t fifth,
                                             const float* x) {
  const uint32_t lo[4] = {w0, w1, w2, w3};
  float a = 0.0f, b = 0.0f;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      const int i = 8 * w + p;
      const uint32_t u = ((lo[w] >> (4 * p)) & 0xFu) | (((fifth >> i) & 1u) << 4);
      const float v = bits_f32(kMagic | u) + kNegQ5;
      if (p & 1) {
        b = fmaf(v, x[i], b);
      } else {
        a = fmaf(v, x[i], a);
      }
    }
  }
  return a + b;
}

// Code of weight i (0..63) of one q5 group starting at `g`.
__device__ __forceinline__ int q5_code(const uint8_t* g, uint32_t i) {
  const uint32_t lo = (i & 1u) ? (g[i / 2] >> 4) : (g[i / 2] & 0x0Fu);
  const uint32_t hi = (g[32 + i / 8] >> (i % 8)) & 1u;
  return static_cast<int>(lo | (hi << 4)) - 16;
}

__device__ __forceinline__ void q8_word(uint32_t w, const uint64_t* x2, uint64_t& acc) {
  const uint64_t v01 = pack2(bits_f32(__byte_perm(w, kMagic, 0x7440)), bits_f32(__byte_perm(w, kMagic, 0x7441)));
  const uint64_t v23 = pack2(bits_f32(__byte_perm(w, kMagic, 0x7442)), bits_f32(__byte_perm(w, kMagic, 0x7443)));
  const uint64_t bias = pack2(kNegQ8, kNegQ8);
  acc = fma2(add2(v01, bias), x2[0], acc);
  acc = fma2(add2(v23, bias), x2[1], acc);
}

// 16 q8 weights (one 16-byte chunk) against 8 packed activation pairs.
__device__ __forceinline__ float q8_chunk_dot(uint4 w, const uint64_t* x2) {
  uint64_t a = 0, b = 0;
  q8_word(w.x, x2 + 0, a);
  q8_word(w.y, x2 + 2, b);
  q8_word(w.z, x2 + 4, a);
  q8_word(w.w, x2 + 6, b);
  const float2 fa = unpack2(a), fb = unpack2(b);
  return (fa.x + fa.y) + (fb.x + fb.y);
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t bits) { return __half2float(__ushort_as_half(bits)); }

// f16 -> f32 on the integer and FMA pipes: the exponent/mantissa bits moved
// into f32 position read as 2^-112 times the value (an f32 subnormal for an
// f16 subnormal), and the exact multiply by 2^112 restores it. Exact for
// every finite f16, zero and subnormals included (FTZ must be off).
__device__ __forceinline__ float f16_bits_to_f32_fast(uint32_t bits) {
  const float magnitude = __uint_as_float((bits & 0x7FFFu) << 13) * 0x1p112f;
  return __uint_as_float(__float_as_uint(magnitude) | ((bits & 0x8000u) << 16));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sums four per-lane values across the warp with 6 shuffles (a transposing
// butterfly): afterwards lanes 8q..8q+7 hold the total of value q.
__device__ __forceinline__ float warp_sum4(float v0, float v1, float v2, float v3) {
  const unsigned lane = threadIdx.x & 31u;
  const bool hi16 = (lane & 16u) != 0;
  float a = hi16 ? v2 : v0, b = hi16 ? v3 : v1;
  const float sa = hi16 ? v0 : v2, sb = hi16 ? v1 : v3;
  a += __shfl_xor_sync(0xffffffffu, sa, 16);
  b += __shfl_xor_sync(0xffffffffu, sb, 16);
  const bool hi8 = (lane & 8u) != 0;
  float r = hi8 ? b : a;
  r += __shfl_xor_sync(0xffffffffu, hi8 ? a : b, 8);
  r += __shfl_xor_sync(0xffffffffu, r, 4);
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// Sums two per-lane values across the warp with 5 shuffles: afterwards lanes
// 0..15 hold the total of v0 and lanes 16..31 the total of v1.
__device__ __forceinline__ float warp_sum2(float v0, float v1) {
  const bool hi16 = (threadIdx.x & 16u) != 0;
  float r = hi16 ? v1 : v0;
  r += __shfl_xor_sync(0xffffffffu, hi16 ? v0 : v1, 16);
  r += __shfl_xor_sync(0xffffffffu, r, 8);
  r += __shfl_xor_sync(0xffffffffu, r, 4);
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// L2-coherent loads for data other CTAs wrote during this launch.
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ld_cg4(const float4* p) { return __ldcg(p); }

__device__ __forceinline__ uint4 ld_nc4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier and bulk async copy (sm_90+ PTX; no multicast) ----

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `hint_ns` pass, instead of spinning on the issue slots
// its warp shares with the scheduler's other warps.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return done != 0;
}

// Bulk copy global -> shared, completing on `bar` (cp.async.bulk, non-multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// One box of a 3-D tensor map (no multicast) into shared memory, completing
// on `bar`. x is the innermost coordinate in elements; x * element size must
// be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* map, int32_t x, int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Orders this thread's generic-proxy global accesses before later async-proxy
// (bulk copy / TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Waits on an mbarrier phase for at most `timeout_ns` of wall-clock time.
// Returns false (and sets *error) if the bound is hit or another CTA already
// reported an error. The clock is read only once the phase has not completed
// on the first attempts, so waits that are already satisfied stay cheap.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* error, uint64_t timeout_ns,
                                                  int32_t code) {
#pragma unroll 1
  for (int spin = 0; spin < 32; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  const uint64_t deadline = global_timer_ns() + timeout_ns;
  // Each try sleeps up to 20 us unless the phase completes first, so the
  // error word and the clock are checked on every pass of the loop.
  while (!mbar_try_wait_sleep(bar, parity, 20000u)) {
    if (*reinterpret_cast<volatile int32_t*>(error) != 0) return false;
    if (global_timer_ns() > deadline) {
      atomicCAS(error, 0, code);
      return false;
    }
  }
  return true;
}

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream drains.
// Every thread waits here for the previous kernels to complete (their memory
// visible) before touching data they produced or still read, then lets the
// next kernel's CTAs be scheduled. Without the launch attribute both are
// no-ops.
__device__ __forceinline__ void pdl_wait_and_trigger() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

__device__ __forceinline__ uint32_t atom_add_acq_rel(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Named barrier over the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumer_sync(uint32_t threads) {
  asm volatile("bar.sync 1, %0;" ::"r"(threads) : "memory");
}

// ---- arithmetic in the reference's order ----
//
// The reference's CPU path rounds every f32 product and sum separately (no
// contraction into FMAs) and sums its reductions sequentially. The helpers
// below use the _rn intrinsics, which nvcc never contracts, so code built on
// them gives the same bits as that path on the same inputs.

// exp of an f32 as the host C library's expf computes it: the table-driven
// method of ARM's optimized-routines (Szabolcs Nagy, 2017; glibc >= 2.27
// ships it, built with FMA on x86-64): x * 32 / ln 2 = k + r rounded to the
// nearest integer k, exp(x) = 2^(k/32) * p(r) with p a cubic in double, the
// 2^(i/32) factors from a 32-entry table. The table entries are the doubles
// nearest 2^(i/32), minus i << 47 so that adding k << 47 forms 2^(k/32).
// The CPU oracle calls that expf, and this restatement was checked against it
// on every non-NaN f32 input.
// 2^(i/32) of the table below, as global memory: a warp's lanes index it
// with different i, which the constant cache would serialize; global loads of
// its two 128-byte lines do not.
static __device__ const uint64_t kExpRefTab[32] = {
      0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
      0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
      0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
      0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
      0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
      0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
      0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
      0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull,
  };

__device__ __forceinline__ float exp_ref(float x) {
  constexpr double kInvLn2N = 0x1.71547652b82fep+0 * 32;
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
  constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
  constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / 32;
  const uint32_t bits = __float_as_uint(x);
  const uint32_t abstop = (bits >> 20) & 0x7FFu;
  if (abstop >= 0x42Bu) {  // |x| >= 88, or not finite
    if (bits == 0xFF800000u) return 0.0f;                 // exp(-inf)
    if (abstop >= 0x7F8u) return x + x;                   // +inf, NaN
    if (x > 0x1.62e42ep6f) return __int_as_float(0x7F800000);  // overflow: log(2^128) ~ 88.72
    if (x < -0x1.9fe368p6f) return 0.0f;                  // underflow: log(2^-150) ~ -103.97
  }
  const double xd = static_cast<double>(x);
  double kd = __fma_rn(kInvLn2N, xd, kShift);
  const uint64_t ki = static_cast<uint64_t>(__double_as_longlong(kd));
  kd = __dsub_rn(kd, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const uint64_t t = __ldg(&kExpRefTab[ki % 32]) + (ki << 47);
  const double s = __longlong_as_double(static_cast<long long>(t));
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(kC2, r, 1.0);
  y = __fma_rn(z, r2, y);
  y = __dmul_rn(y, s);
  return __double2float_rn(y);
}

// 1 / sqrt(mean_square + eps) with mean_square = sum / width
// (math.zig:120-130): every step correctly rounded.
__device__ __forceinline__ float rms_inverse(float sum_squares, uint32_t width, float eps) {
  const float mean = __fdiv_rn(sum_squares, static_cast<float>(width));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// sum_squares over n values in order (math.zig:123): s = s + v * v, each
// product and sum rounded. `v` is read from shared or global memory.
__device__ __forceinline__ float sum_squares_seq(const float* v, uint32_t n) {
  float s = 0.0f;
  uint32_t i = 0;
  for (; i + 8 <= n; i += 8) {
    float t[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) t[e] = v[i + e];
#pragma unroll
    for (int e = 0; e < 8; ++e) s = __fadd_rn(s, __fmul_rn(t[e], t[e]));
  }
  for (; i < n; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
  return s;
}

// rotate_half RoPE of one element (kernels.zig:519-520): dims below half take
// lo * cos - hi * sin, the others hi * cos + lo * sin; products rounded first.
__device__ __forceinline__ float rope_rn(bool low_half, float lo, float hi, float cs, float sn) {
  return low_half ? __fsub_rn(__fmul_rn(lo, cs), __fmul_rn(hi, sn)) : __fadd_rn(__fmul_rn(hi, cs), __fmul_rn(lo, sn));
}

// quant.zig:280-288 for q8 (bias 128): round half away from zero against the
// stored f16 scale, then clamp into [-128, 127].
__device__ __forceinline__ uint8_t q8_code(float value, float stored_scale) {
  if (stored_scale == 0.0f) return 128;
  const float scaled = __fdiv_rn(value, stored_scale);
  const float rounded = scaled >= 0.0f ? floorf(__fadd_rn(scaled, 0.5f)) : ceilf(__fsub_rn(scaled, 0.5f));
  int code;
  if (rounded <= -128.0f) code = -128;
  else if (rounded >= 127.0f) code = 127;
  else code = static_cast<int>(rounded);
  return static_cast<uint8_t>(code + 128);
}

// Launches `kernel` with programmatic stream serialization (see
// pdl_wait_and_trigger); inside stream capture this becomes a programmatic
// edge of the graph.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace qwc

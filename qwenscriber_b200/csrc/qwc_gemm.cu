// qwc_gemm.cu -- quantized-weight GEMM for independent decode streams on the
// 5th-generation tensor cores (tcgen05, sm_100a).
//
// out[s][r] = sum_k W[r][k] * x[s][k] for up to 64 streams s at once: the
// projections of kernels.linearQuantized (src/core/qwen3_asr/kernels.zig:118-158)
// for a batch of streams. W stays in the reference's two-plane q4/q8 layout
// (src/core/quant.zig:144-176). Per CTA: two tiles of 128 weight rows (each
// activation block feeds both) and a range of K, in blocks of 64 (one
// quantization group):
//
//   warp 0   TMA producer: raw code and scale boxes of the tile, and the
//            activation box, into a 6-stage shared-memory ring (mbarrier
//            complete_tx);
//   warp 1   TMEM owner and MMA issuer: tcgen05.mma kind::f16 with the
//            weights from TMEM and the activations from shared memory,
//            M=128, K=16, accumulating in TMEM; tcgen05.commit frees stages;
//   warps 2-9 dequantize each raw block straight into TMEM (tcgen05.st, one
//            tile row per TMEM lane; the four warps of tile t cover its lane
//            quarters), 2 stages deep; then read tile t's accumulator back
//            (tcgen05.ld) and store f32 results.
//
// Keeping the dequantized weights out of shared memory leaves its bandwidth
// to the TMA boxes and the activation reads of the MMAs.
//
// Exactness: a dequantized weight (code - bias) * scale is split into
// hi = f16(w) and lo = w - hi, which is exact in f16 (at most 8 significant
// bits remain); each activation into hi = f16(x) and lo = f16(x - hi). The
// activation box holds the 64 hi rows, then the 64 lo rows. Per K step two
// MMAs (weights hi, then lo) take all 128 columns; the epilogue adds the two
// column halves. Products are thus those of the exact weights with 22-bit
// activations. Measured and not kept: leaving out the lo x lo product (no
// faster), and four N = 64 MMAs into one 64-column accumulator per tile with
// three dequantized stages in TMEM (slower: 3.67 against 3.36 ms per
// 64-stream step).
//
// Activations arrive by TMA in 128-byte-swizzled rows; the dequantized weights
// are written by the threads in the no-swizzle core-matrix layout.
//
// K order inside every 8-value chunk is permuted the same way for weights
// and activations, [0 4 1 5 2 6 3 7], so one lop3 extracts two values of a
// 32-bit q4 code word at once. The sum over K does not depend on the order.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>
#include <cstring>

#include "../../include/qwenscriber_cuda.h"
#include "qwc_device.cuh"
#include "qwc_internal.h"

namespace qwc {
namespace {

constexpr int kGemmThreads = 320;
constexpr int kDequantWarps = 8;
constexpr int kRawStages = 6;
constexpr int kAStages = 2;  // dequantized operands (TMEM) in flight between the dequant warps and the MMAs
constexpr uint32_t kTileM = 128;
constexpr uint32_t kTilesPerCta = 2;
constexpr uint32_t kCtaRows = kTileM * kTilesPerCta;
constexpr uint32_t kStreamCols = 64;                      // streams per launch
constexpr uint32_t kTileN = 2 * kStreamCols;              // hi rows then lo rows
constexpr uint32_t kKBlock = 64;
constexpr uint32_t kBStageBytes = kTileN * kKBlock * 2;   // 16 KB of f16, one 128-byte swizzle atom column
constexpr uint32_t kCodeStageBytes = kCtaRows * kKBlock;  // q8: 64 B per row; q4 uses half
constexpr uint32_t kScaleStageBytes = kCtaRows * 16;      // one 16-byte box column of scales
// TMEM: tile t's f32 accumulator in columns [128 t, 128 t + 128); A stage i
// in columns 256 + 128 i: per tile (64 columns each) weights hi (4 K steps x
// 8 columns of f16 pairs), then lo.
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = kTilesPerCta * kTileN;
constexpr uint32_t kTmemAStage = 64 * kTilesPerCta;

struct __align__(1024) GemmSmem {
  uint8_t b[kRawStages][kBStageBytes];
  uint8_t codes[kRawStages][kCodeStageBytes];
  uint8_t scales[kRawStages][kScaleStageBytes];
  uint64_t w_full[kRawStages];  // the stage's weight codes and scales landed
  uint64_t b_full[kRawStages];  // the stage's activation box landed
  uint64_t raw_empty[kRawStages];
  uint64_t a_full[kAStages];
  uint64_t a_empty[kAStages];
  uint64_t acc_full;
  uint32_t tmem_base;
};
static_assert(offsetof(GemmSmem, b) % 1024 == 0 && offsetof(GemmSmem, codes) % 128 == 0 &&
                  offsetof(GemmSmem, scales) % 128 == 0,
              "TMA destinations need 128-byte alignment (swizzled boxes 1024)");
static_assert(kTmemA + kAStages * kTmemAStage <= kTmemCols, "TMEM budget");

// ---- tcgen05 wrappers ----

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major. No swizzle: core matrices of
// 8 rows x 16 bytes stored contiguously, `lbo` = byte distance between the
// two 8-element K halves of an MMA, `sbo` = byte distance between 8-row
// groups. 128-byte swizzle: rows of 128 bytes, `sbo` = 1024 (8 rows), the
// atom 1024-byte aligned; K steps inside the atom advance the start address.
constexpr uint32_t kLayoutSw128 = 2;
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;  // base offset 0, absolute leading-offset mode
}

// Instruction descriptor: f16 x f16 -> f32, both K-major, M = 128, N = 128
// (activation hi and lo columns).
constexpr uint32_t kIdescN128 = (1u << 4) | ((kTileN >> 3) << 17) | ((kTileM >> 4) << 24);

// D[tmem_d] (+)= A[tmem_a] * B[smem desc]: A read from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}


// 32 lanes x 32 columns of this warp's lane quarter from registers: one
// instruction for a row's whole K block of hi (or lo) values.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint4 (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
      "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w),
      "r"(v[4].x), "r"(v[4].y), "r"(v[4].z), "r"(v[4].w), "r"(v[5].x), "r"(v[5].y), "r"(v[5].z), "r"(v[5].w),
      "r"(v[6].x), "r"(v[6].y), "r"(v[6].z), "r"(v[6].w), "r"(v[7].x), "r"(v[7].y), "r"(v[7].z), "r"(v[7].w)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

// 32 lanes x 32 columns of f32 from TMEM (lane quarter of this warp).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- dequantization to f16 pairs ----

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t lop_and_or(uint32_t w, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(magic));
  return r;
}

__device__ __forceinline__ uint32_t hfma2_bits(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Two centred codes (exact f16) times the scale: hi = f16(c * s), lo = the
// exact remainder c * s - hi (one fused multiply-add).
__device__ __forceinline__ void split_pair(uint32_t c2, uint32_t scale2, uint32_t& hi, uint32_t& lo) {
  hi = hmul2_bits(c2, scale2);
  lo = hfma2_bits(c2, scale2, hi ^ 0x80008000u);
}

// Eight q4 codes (one 32-bit word, K order 0..7) -> 16 bytes of f16 hi and
// lo in the chunk order [0 4 1 5 2 6 3 7].
__device__ __forceinline__ void dequant_q4_word(uint32_t w, uint32_t scale2, uint4& hi, uint4& lo) {
  const uint32_t magic = 0x64006400u;  // f16 1024 in both halves
  const uint32_t bias = 0x64086408u;   // f16 1032 = 1024 + 8
  const uint32_t mask = 0x000F000Fu;
  split_pair(hsub2_bits(lop_and_or(w, mask, magic), bias), scale2, hi.x, lo.x);
  split_pair(hsub2_bits(lop_and_or(w >> 4, mask, magic), bias), scale2, hi.y, lo.y);
  split_pair(hsub2_bits(lop_and_or(w >> 8, mask, magic), bias), scale2, hi.z, lo.z);
  split_pair(hsub2_bits(lop_and_or(w >> 12, mask, magic), bias), scale2, hi.w, lo.w);
}

// Eight q8 codes (two words, K order 0..7) -> the same chunk order.
__device__ __forceinline__ void dequant_q8_words(uint32_t w0, uint32_t w1, uint32_t scale2, uint4& hi, uint4& lo) {
  const uint32_t magic = 0x64006400u;
  const uint32_t bias = 0x64806480u;  // f16 1152 = 1024 + 128
  const uint32_t mask = 0x00FF00FFu;
  split_pair(hsub2_bits(lop_and_or(__byte_perm(w0, w1, 0x0400), mask, magic), bias), scale2, hi.x, lo.x);
  split_pair(hsub2_bits(lop_and_or(__byte_perm(w0, w1, 0x0501), mask, magic), bias), scale2, hi.y, lo.y);
  split_pair(hsub2_bits(lop_and_or(__byte_perm(w0, w1, 0x0602), mask, magic), bias), scale2, hi.z, lo.z);
  split_pair(hsub2_bits(lop_and_or(__byte_perm(w0, w1, 0x0703), mask, magic), bias), scale2, hi.w, lo.w);
}

// Code bytes a TMA box brings per row per K block, and the box's x
// coordinate. q4 and q8 groups (32, 64 bytes) start on 16-byte boundaries;
// a q5 group (40 bytes) starts 8 bytes past one when its index is odd, so
// its box is 48 bytes from the boundary at or below it (the group at byte
// offset (40 kb) & 15 within the box; the last box's overhang past the row
// reads the fill value and is never used).
__host__ __device__ constexpr uint32_t gemm_code_box(uint32_t format) {
  return format == kFormatQ4 ? 32u : format == kFormatQ5 ? 48u : 64u;
}
__device__ __forceinline__ uint32_t gemm_code_x(uint32_t format, uint32_t kb) {
  return format == kFormatQ5 ? (40u * kb) & ~15u : kb * gemm_code_box(format);
}

// Eight q5 weights of a group (K order 0..7): their low nibbles as one q4
// code word `w`, their fifth bits as byte `f` (bit k for weight k). The code
// is nibble | fifth << 4 with bias 16 (quant.zig:253-269, 327-335).
__device__ __forceinline__ void dequant_q5_word(uint32_t w, uint32_t f, uint32_t scale2, uint4& hi, uint4& lo) {
  const uint32_t magic = 0x64006400u;  // f16 1024 in both halves
  const uint32_t bias = 0x64106410u;   // f16 1040 = 1024 + 16
  const uint32_t mask = 0x000F000Fu;
  uint32_t pr[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // Pair (j, j + 4): fifth bits to bit 4 of each f16 half's mantissa.
    const uint32_t fifth = (((f >> j) & 1u) << 4) | (((f >> (j + 4)) & 1u) << 20);
    pr[j] = lop_and_or(w >> (4 * j), mask, magic) | fifth;  // f16 pair (1024 + code)
  }
  split_pair(hsub2_bits(pr[0], bias), scale2, hi.x, lo.x);
  split_pair(hsub2_bits(pr[1], bias), scale2, hi.y, lo.y);
  split_pair(hsub2_bits(pr[2], bias), scale2, hi.z, lo.z);
  split_pair(hsub2_bits(pr[3], bias), scale2, hi.w, lo.w);
}

// One weight matrix of a launch. A launch multiplies up to three matrices
// that share K and the activations (Q, K and V; gate and up).
struct GemmJob {
  uint32_t rows;        // M
  uint32_t mtiles;      // ceil(rows / 256): CTA tiles
  uint32_t format;      // q4 / q8
  uint32_t out_offset;  // first output column of this matrix in each output row
};

struct GemmParams {
  GemmJob job[3];
  uint32_t njobs;
  uint32_t cols;        // K (multiple of kKBlock)
  uint32_t streams;     // columns written, over all column blocks (blockIdx.z: 64 each); output rows per split
  uint32_t kb_per_split;
  float* out;           // [split][streams][out_ld]
  uint32_t out_ld;
  int32_t* error;
  uint64_t timeout_ns;
};

struct alignas(64) GemmMaps {
  CUtensorMap codes[3];
  CUtensorMap scales[3];
  CUtensorMap b;
};

enum GemmError : int32_t { kGemmErrWait = 1 };

// Bounded wait; on expiry the first failing thread also records where
// (error[1..3] = code site, block x, block y).
__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t parity, const GemmParams& p, int32_t site = 0) {
  if (mbar_wait_bounded(bar, parity, p.error, p.timeout_ns, kGemmErrWait + site)) return true;
  if (*reinterpret_cast<volatile int32_t*>(p.error) == kGemmErrWait + site) {
    p.error[1] = site;
    p.error[2] = static_cast<int32_t>(blockIdx.x);
    p.error[3] = static_cast<int32_t>(blockIdx.y);
  }
  return false;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_streams_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
  extern __shared__ __align__(1024) uint8_t gemm_smem_raw[];
  // The swizzle atoms need 1024-byte alignment in the shared window.
  const uint32_t pad = (1024u - (smem_addr(gemm_smem_raw) & 1023u)) & 1023u;
  GemmSmem* s = reinterpret_cast<GemmSmem*>(gemm_smem_raw + pad);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // Which matrix and which 256-row stretch of it this CTA takes.
  uint32_t tile = blockIdx.x, jb = 0;
  while (jb + 1 < p.njobs && tile >= p.job[jb].mtiles) tile -= p.job[jb++].mtiles;
  const GemmJob job = p.job[jb];
  const CUtensorMap* map_codes = &maps.codes[jb];
  const CUtensorMap* map_scales = &maps.scales[jb];
  const CUtensorMap* map_b = &maps.b;
  const uint32_t m0 = tile * kCtaRows;
  const uint32_t kblocks = p.cols / kKBlock;
  const uint32_t kb0 = blockIdx.y * p.kb_per_split;
  const uint32_t kb1 = min(kblocks, kb0 + p.kb_per_split);
  const uint32_t nkb = kb1 > kb0 ? kb1 - kb0 : 0;
  const bool q4 = job.format == kFormatQ4, q5 = job.format == kFormatQ5;
  const uint32_t code_box = gemm_code_box(job.format);  // bytes of codes per row per block

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(&s->w_full[i], 1);
      mbar_init(&s->b_full[i], 1);
      mbar_init(&s->raw_empty[i], 1);
    }
    for (int i = 0; i < kAStages; ++i) {
      mbar_init(&s->a_full[i], kDequantWarps);
      mbar_init(&s->a_empty[i], 1);
    }
    mbar_init(&s->acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s->tmem_base, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  bool ok = true;
  // Programmatic dependent launch, split by data: the weights never depend on
  // the previous kernel, so the first stages' weight boxes and their
  // dequantization start at once; only the producer's activation loads wait
  // for the previous kernel (which writes the activations and reads the
  // partial sums this launch overwrites). The MMAs and the epilogue follow
  // those loads, so they run after it too.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // ---- producer ----
    if (lane == 0) {
      auto load_weights = [&](uint32_t i) {
        const uint32_t st = i % kRawStages, kb = kb0 + i;
        mbar_arrive_expect_tx(&s->w_full[st], kCtaRows * code_box + kScaleStageBytes);
        tma_load_2d(s->codes[st], map_codes, static_cast<int32_t>(gemm_code_x(job.format, kb)), static_cast<int32_t>(m0),
                    &s->w_full[st]);
        // The 16-byte scale box holding this block's group.
        tma_load_2d(s->scales[st], map_scales, static_cast<int32_t>((kb * 2u) & ~15u), static_cast<int32_t>(m0),
                    &s->w_full[st]);
      };
      auto load_acts = [&](uint32_t i) {
        const uint32_t st = i % kRawStages;
        mbar_arrive_expect_tx(&s->b_full[st], kBStageBytes);
        tma_load_2d(s->b[st], map_b, static_cast<int32_t>((kb0 + i) * kKBlock), static_cast<int32_t>(blockIdx.z * kTileN),
                    &s->b_full[st]);
      };
      const uint32_t first = nkb < uint32_t(kRawStages) ? nkb : uint32_t(kRawStages);
      for (uint32_t i = 0; i < first; ++i) load_weights(i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (uint32_t i = 0; i < first; ++i) load_acts(i);
      uint32_t issued = first;
      for (uint32_t i = first; i < nkb && ok; ++i) {
        const uint32_t st = i % kRawStages;
        if (!wait_bounded(&s->raw_empty[st], ((i / kRawStages) - 1) & 1u, p, 10)) {
          ok = false;
          break;
        }
        load_weights(i);
        load_acts(i);
        issued = i + 1;
      }
      // Drain: the last stages issued must have landed before the CTA exits
      // (an earlier stage was consumed before its slot was loaded again).
      for (uint32_t i = issued > uint32_t(kRawStages) ? issued - kRawStages : 0u; i < issued; ++i) {
        const uint32_t st = i % kRawStages;
        wait_bounded(&s->w_full[st], (i / kRawStages) & 1u, p);
        wait_bounded(&s->b_full[st], (i / kRawStages) & 1u, p);
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    const uint64_t b_desc0 = umma_desc(smem_addr(s->b[0]), 16, 1024, kLayoutSw128);
    if (lane == 0) {
      for (uint32_t i = 0; i < nkb && ok; ++i) {
        const uint32_t st = i % kRawStages;
        const uint32_t at = i % kAStages;
        if (!wait_bounded(&s->b_full[st], (i / kRawStages) & 1u, p, 20) ||
            !wait_bounded(&s->a_full[at], (i / kAStages) & 1u, p, 30)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // A: 8 TMEM columns (16 f16 of K) per MMA. B: one swizzle atom of
        // 128 rows x 128 B; 32 B per K step (the descriptor's start-address
        // field advances in 16-byte units).
        const uint32_t a0 = tmem + kTmemA + at * kTmemAStage;
        const uint64_t bd0 = b_desc0 + ((uint64_t(st) * kBStageBytes) >> 4);
#pragma unroll
        for (uint32_t k = 0; k < kKBlock / 16; ++k) {
          const uint64_t bd = bd0 + 2 * k;
#pragma unroll
          for (uint32_t t = 0; t < kTilesPerCta; ++t) {
            // tile t: weights hi, then lo, against activations hi | lo
            const uint32_t d = tmem + t * kTileN;
            umma_f16_ts(d, a0 + 64 * t + 8 * k, bd, kIdescN128, (i > 0 || k > 0) ? 1u : 0u);
            umma_f16_ts(d, a0 + 64 * t + 32 + 8 * k, bd, kIdescN128, 1u);
          }
        }
        umma_commit(&s->a_empty[at]);
        umma_commit(&s->raw_empty[st]);
      }
      umma_commit(&s->acc_full);
      // MMAs still in flight must finish before TMEM is released.
      if (!ok) wait_bounded(&s->acc_full, 0, p);
    }
  } else {
    // ---- dequantize into TMEM, then epilogue ----
    const uint32_t quarter = static_cast<uint32_t>(warp % 4);
    const uint32_t t = static_cast<uint32_t>((warp - 2) / 4);  // tile of this warp
    const uint32_t r = t * kTileM + quarter * 32 + lane;       // row of the CTA's stretch
    const uint32_t lane_addr = (quarter * 32u) << 16;
    for (uint32_t i = 0; i < nkb && ok; ++i) {
      const uint32_t st = i % kRawStages;
      const uint32_t at = i % kAStages;
      bool ready = wait_bounded(&s->w_full[st], (i / kRawStages) & 1u, p, 40);
      if (ready && i >= kAStages) ready = wait_bounded(&s->a_empty[at], ((i / kAStages) - 1) & 1u, p, 50);
      if (!__all_sync(0xffffffffu, ready)) {  // tcgen05.st below is warp-collective
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t kb = kb0 + i;
      const uint16_t sb = *reinterpret_cast<const uint16_t*>(s->scales[st] + r * 16 + ((kb * 2u) & 15u));
      const uint32_t sc = static_cast<uint32_t>(sb) * 0x10001u;
      const uint32_t ahi = tmem + lane_addr + kTmemA + at * kTmemAStage + 64 * t;
      const uint32_t alo = ahi + 32;
      // The row's 64 K values as 32 columns of f16 pairs, hi and lo; each
      // goes to TMEM in one 32-column store.
      uint4 hv[8], lv[8];
      if (q5) {
        // The group's 32 bytes of nibbles (8 words of 8 weights) and 8 bytes of
        // fifth bits, at byte 0 or 8 of the row's 48-byte box: 8-byte loads.
        const uint2* g = reinterpret_cast<const uint2*>(s->codes[st] + r * 48u + ((40u * kb) & 15u));
        const uint2 n0 = g[0], n1 = g[1], n2 = g[2], n3 = g[3], fifth = g[4];
        const uint32_t nw[8] = {n0.x, n0.y, n1.x, n1.y, n2.x, n2.y, n3.x, n3.y};
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t fb = ((q < 4 ? fifth.x : fifth.y) >> (8 * (q & 3))) & 0xFFu;
          dequant_q5_word(nw[q], fb, sc, hv[q], lv[q]);
        }
      } else if (q4) {
        // Two 16-byte chunks of codes, 8 per word.
        const uint4* src = reinterpret_cast<const uint4*>(s->codes[st] + r * (kKBlock / 2));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint4 w = src[q];
          dequant_q4_word(w.x, sc, hv[4 * q], lv[4 * q]);
          dequant_q4_word(w.y, sc, hv[4 * q + 1], lv[4 * q + 1]);
          dequant_q4_word(w.z, sc, hv[4 * q + 2], lv[4 * q + 2]);
          dequant_q4_word(w.w, sc, hv[4 * q + 3], lv[4 * q + 3]);
        }
      } else {
        const uint4* src = reinterpret_cast<const uint4*>(s->codes[st] + r * kKBlock);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 w = src[q];
          dequant_q8_words(w.x, w.y, sc, hv[2 * q], lv[2 * q]);
          dequant_q8_words(w.z, w.w, sc, hv[2 * q + 1], lv[2 * q + 1]);
        }
      }
      tmem_st32(ahi, hv);
      tmem_st32(alo, lv);
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s->a_full[at]);
    }
    // Epilogue: TMEM lane = tile row; this warp reads tile t's accumulator in
    // its lane quarter: columns n (x hi) and 64 + n (x lo).
    bool go = ok && nkb > 0 && wait_bounded(&s->acc_full, 0, p, 60);
    go = __all_sync(0xffffffffu, go);  // tcgen05.ld is warp-collective
    if (go) {
      tc_fence_after();
      const uint32_t row = m0 + r;
      const uint32_t n_base = blockIdx.z * kStreamCols;  // this column block's first column
      float* out = p.out + (size_t(blockIdx.y) * p.streams + n_base) * p.out_ld + job.out_offset + row;
#pragma unroll
      for (uint32_t n0 = 0; n0 < kStreamCols; n0 += 32) {
        float v[32], vlo[32];
        tmem_ld32(tmem + lane_addr + t * kTileN + n0, v);
        tmem_ld32(tmem + lane_addr + t * kTileN + kStreamCols + n0, vlo);
        if (row < job.rows) {
#pragma unroll
          for (int n = 0; n < 32; ++n) {
            if (n_base + n0 + n < p.streams) out[size_t(n0 + n) * p.out_ld] = v[n] + vlo[n];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// x[s][k] f32 -> the activation box rows: column s of block b = s / 64 has
// its f16 hi values in row 128 b + s % 64 and its lo remainders in row
// 128 b + 64 + s % 64, chunks in the permuted order.
__global__ void pack_activations_kernel(const float* x, uint32_t streams, uint32_t cols, __half* out) {
  pdl_wait_and_trigger();
  const uint32_t chunks = cols / 8;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < streams * chunks; i += gridDim.x * blockDim.x) {
    const uint32_t col = i / chunks, c = i % chunks;
    const uint32_t sidx = (col / kStreamCols) * kTileN + col % kStreamCols;
    const float* src = x + size_t(col) * cols + c * 8;
    const int perm[8] = {0, 4, 1, 5, 2, 6, 3, 7};
    __align__(16) __half hi[8];
    __align__(16) __half lo[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = src[perm[j]];
      hi[j] = __float2half_rn(v);
      lo[j] = __float2half_rn(v - __half2float(hi[j]));
    }
    *reinterpret_cast<uint4*>(out + size_t(sidx) * cols + c * 8) = *reinterpret_cast<const uint4*>(hi);
    *reinterpret_cast<uint4*>(out + size_t(kStreamCols + sidx) * cols + c * 8) = *reinterpret_cast<const uint4*>(lo);
  }
}

__global__ void sum_splits_kernel(const float* parts, uint32_t splits, uint32_t n, float* out) {
  pdl_wait_and_trigger();
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    float acc = parts[i];
    for (uint32_t sp = 1; sp < splits; ++sp) acc += parts[size_t(sp) * n + i];
    out[i] = acc;
  }
}

// ---- dense f16 weights: the audio tower's convolutions as GEMMs ----
//
// out[split][n][m] = sum over the split's K blocks of W[m][k] * X[n][k]: W is
// f16 [rows][kpad] (exact: the convolution weights are stored in f16), X the
// activation rows of pack_activations_kernel's layout in natural K order (f16
// hi rows, then lo rows, per 64-column block). Both operands reach shared
// memory by TMA in 128-byte-swizzled boxes and feed tcgen05.mma directly (A
// from a shared-memory descriptor): per K step one MMA per 128-row tile over
// 128 columns (x hi | x lo); the epilogue adds the two halves.
// Warp 0: TMA producer; warp 1: MMA issuer; warps 2-9: epilogue (tile
// (warp - 2) / 4, TMEM lane quarter warp % 4).
constexpr int kDenseStages = 4;
constexpr uint32_t kDenseAStage = kTileM * kKBlock * 2;  // one 128-row tile: 16 KB

struct __align__(1024) DenseSmem {
  uint8_t a[kDenseStages][kTilesPerCta][kDenseAStage];
  uint8_t b[kDenseStages][kBStageBytes];
  uint64_t full[kDenseStages];
  uint64_t empty[kDenseStages];
  uint64_t acc_full;
  uint32_t tmem_base;
};
static_assert(offsetof(DenseSmem, b) % 1024 == 0 && kDenseAStage % 1024 == 0, "swizzled boxes need 1024 B alignment");

struct DenseParams {
  uint32_t rows;          // M
  uint32_t kb_per_split;  // K blocks per split (grid y)
  uint32_t kblocks;       // kpad / 64
  uint32_t columns;       // N over all column blocks (grid z)
  float* out;             // [split][columns][rows]
  int32_t* error;
  uint64_t timeout_ns;
};

struct alignas(64) DenseMaps {
  CUtensorMap a;
  CUtensorMap b;
};

// D[tmem_d] (+)= A[smem desc] * B[smem desc].
__device__ __forceinline__ void umma_f16_ss(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool dense_wait(uint64_t* bar, uint32_t parity, const DenseParams& p, int32_t site) {
  if (mbar_wait_bounded(bar, parity, p.error, p.timeout_ns, kGemmErrWait + site)) return true;
  if (*reinterpret_cast<volatile int32_t*>(p.error) == kGemmErrWait + site) {
    p.error[1] = site;
    p.error[2] = static_cast<int32_t>(blockIdx.x);
    p.error[3] = static_cast<int32_t>(blockIdx.y);
  }
  return false;
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_dense_kernel(const __grid_constant__ DenseMaps maps, const DenseParams p) {
  extern __shared__ __align__(1024) uint8_t dense_smem_raw[];
  const uint32_t pad = (1024u - (smem_addr(dense_smem_raw) & 1023u)) & 1023u;
  DenseSmem* s = reinterpret_cast<DenseSmem*>(dense_smem_raw + pad);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t m0 = blockIdx.x * kCtaRows;
  const uint32_t kb0 = blockIdx.y * p.kb_per_split;
  const uint32_t kb1 = min(p.kblocks, kb0 + p.kb_per_split);
  const uint32_t nkb = kb1 > kb0 ? kb1 - kb0 : 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kDenseStages; ++i) {
      mbar_init(&s->full[i], 1);
      mbar_init(&s->empty[i], 1);
    }
    mbar_init(&s->acc_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&s->tmem_base, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s->tmem_base;
  bool ok = true;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      // The weights never depend on the previous kernel: the first stages'
      // weight boxes go out before the dependency wait, the activations after.
      auto load_a = [&](uint32_t i) {
        const uint32_t st = i % kDenseStages, kb = kb0 + i;
        mbar_arrive_expect_tx(&s->full[st], kTilesPerCta * kDenseAStage + kBStageBytes);
        for (uint32_t t = 0; t < kTilesPerCta; ++t) {
          tma_load_2d(s->a[st][t], &maps.a, static_cast<int32_t>(kb * kKBlock), static_cast<int32_t>(m0 + t * kTileM),
                      &s->full[st]);
        }
      };
      auto load_b = [&](uint32_t i) {
        const uint32_t st = i % kDenseStages;
        tma_load_2d(s->b[st], &maps.b, static_cast<int32_t>((kb0 + i) * kKBlock),
                    static_cast<int32_t>(blockIdx.z * kTileN), &s->full[st]);
      };
      const uint32_t first = nkb < uint32_t(kDenseStages) ? nkb : uint32_t(kDenseStages);
      for (uint32_t i = 0; i < first; ++i) load_a(i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (uint32_t i = 0; i < first; ++i) load_b(i);
      uint32_t issued = first;
      for (uint32_t i = first; i < nkb && ok; ++i) {
        const uint32_t st = i % kDenseStages;
        if (!dense_wait(&s->empty[st], ((i / kDenseStages) - 1) & 1u, p, 10)) {
          ok = false;
          break;
        }
        load_a(i);
        load_b(i);
        issued = i + 1;
      }
      for (uint32_t i = issued > uint32_t(kDenseStages) ? issued - kDenseStages : 0u; i < issued; ++i) {
        dense_wait(&s->full[i % kDenseStages], (i / kDenseStages) & 1u, p, 11);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint64_t a_desc0 = umma_desc(smem_addr(s->a[0][0]), 16, 1024, kLayoutSw128);
      const uint64_t b_desc0 = umma_desc(smem_addr(s->b[0]), 16, 1024, kLayoutSw128);
      constexpr uint64_t kAStageUnits = (uint64_t(kTilesPerCta) * kDenseAStage) >> 4;
      for (uint32_t i = 0; i < nkb && ok; ++i) {
        const uint32_t st = i % kDenseStages;
        if (!dense_wait(&s->full[st], (i / kDenseStages) & 1u, p, 20)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + st * kAStageUnits;
        const uint64_t bd = b_desc0 + ((uint64_t(st) * kBStageBytes) >> 4);
#pragma unroll
        for (uint32_t k = 0; k < kKBlock / 16; ++k) {
#pragma unroll
          for (uint32_t t = 0; t < kTilesPerCta; ++t) {
            umma_f16_ss(tmem + t * kTileN, ad + ((uint64_t(t) * kDenseAStage) >> 4) + 2 * k, bd + 2 * k, kIdescN128,
                        (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma_commit(&s->empty[st]);
      }
      umma_commit(&s->acc_full);
      if (!ok) dense_wait(&s->acc_full, 0, p, 21);
    }
  } else {
    const uint32_t quarter = static_cast<uint32_t>(warp % 4);
    const uint32_t t = static_cast<uint32_t>((warp - 2) / 4);
    const uint32_t row = m0 + t * kTileM + quarter * 32 + lane;
    bool go = nkb > 0 && dense_wait(&s->acc_full, 0, p, 60);
    go = __all_sync(0xffffffffu, go);
    if (go) {
      tc_fence_after();
      const uint32_t n_base = blockIdx.z * kStreamCols;
      float* out = p.out + (size_t(blockIdx.y) * p.columns + n_base) * p.rows + row;
      const uint32_t taddr = tmem + ((quarter * 32u) << 16) + t * kTileN;
#pragma unroll
      for (uint32_t n0 = 0; n0 < kStreamCols; n0 += 32) {
        float v[32], vlo[32];
        tmem_ld32(taddr + n0, v);
        tmem_ld32(taddr + kStreamCols + n0, vlo);
        if (row < p.rows) {
#pragma unroll
          for (int n = 0; n < 32; ++n) {
            if (n_base + n0 + n < p.columns) out[size_t(n0 + n) * p.rows] = v[n] + vlo[n];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

int gemm_smem_bytes() { return static_cast<int>(sizeof(GemmSmem)) + 1024; }

int launch_pack_activations(const float* x, uint32_t columns, uint32_t cols, void* out, void* stream) {
  const uint32_t work = columns * (cols / 8);
  const uint32_t grid = std::min<uint32_t>(1184u, (work + 255) / 256);
  return static_cast<int>(launch_pdl(pack_activations_kernel, dim3(grid), dim3(256), 0,
                                     static_cast<cudaStream_t>(stream), x, columns, cols,
                                     static_cast<__half*>(out)));
}

int prepare_gemm_kernel() {
  return static_cast<int>(
      cudaFuncSetAttribute(gemm_streams_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes()));
}

// TMA descriptors of one weight matrix and of an activation buffer, with the
// box sizes the kernel's transaction counts assume.
int32_t gemm_weight_maps(uint32_t format, const void* codes, const void* scales, uint32_t rows, uint32_t cols,
                         uint8_t* codes_map, uint8_t* scales_map, uint32_t scale_stride) {
  const uint32_t groups = cols / kGroup;
  const uint64_t code_row = uint64_t(groups) * data_bytes_per_group(format);
  const uint64_t scale_row = scale_stride ? scale_stride : uint64_t(groups) * 2;
  const uint64_t dims_c[2] = {code_row, rows};
  const uint64_t str_c[1] = {code_row};
  const uint32_t box_c[2] = {gemm_code_box(format), kCtaRows};
  const uint64_t dims_s[2] = {scale_row, rows};
  const uint64_t str_s[1] = {scale_row};
  const uint32_t box_s[2] = {16, kCtaRows};
  const int32_t rc = encode_tensor_map(codes_map, kMapU8, 2, const_cast<void*>(codes), dims_c, str_c, box_c, false);
  if (rc != QWC_OK) return rc;
  return encode_tensor_map(scales_map, kMapU8, 2, const_cast<void*>(scales), dims_s, str_s, box_s, false);
}

int32_t gemm_act_map(void* base, uint32_t cols, uint8_t* out, uint32_t col_blocks) {
  const uint64_t dims[2] = {cols, uint64_t(kTileN) * col_blocks};
  const uint64_t str[1] = {uint64_t(cols) * 2};
  const uint32_t box[2] = {kKBlock, kTileN};
  return encode_tensor_map(out, kMapF16, 2, base, dims, str, box, true);
}

// Splits of K for a launch of `rows` x `cols`: the fewest waves of CTAs (one
// per SM) weighed against per-CTA fixed cost (about four K blocks of
// pipeline fill, TMEM set-up and epilogue) and the partial sums the next
// kernel reads.
uint32_t gemm_splits(uint32_t rows, uint32_t cols, int sms, uint32_t col_blocks) {
  const uint32_t mtiles = (rows + kCtaRows - 1) / kCtaRows * col_blocks;
  const uint32_t kblocks = cols / kKBlock;
  uint32_t best = 1;
  double best_cost = 1e30;
  for (uint32_t want = 1; want <= kblocks && want <= 32; ++want) {
    const uint32_t kps = (kblocks + want - 1) / want;
    const uint32_t splits = (kblocks + kps - 1) / kps;
    const uint32_t waves = (mtiles * splits + sms - 1) / sms;
    const double cost = double(waves) * (kps + 4.0) + 0.5 * splits;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = splits;
    }
  }
  return best;
}

// A launch over up to three matrices (maps: codes/scales per matrix, then
// the activations); `splits` divides K.
int launch_gemm_jobs(const uint8_t (*codes_maps)[128], const uint8_t (*scale_maps)[128], const uint32_t* rows,
                     const uint32_t* formats, const uint32_t* out_offsets, uint32_t njobs, const uint8_t* map_b,
                     uint32_t cols, uint32_t streams, uint32_t splits, float* out, uint32_t out_ld, int32_t* error,
                     void* stream, uint32_t col_blocks, uint64_t timeout_ns) {
  GemmMaps maps;
  GemmParams p{};
  uint32_t tiles = 0;
  for (uint32_t j = 0; j < njobs; ++j) {
    std::memcpy(&maps.codes[j], codes_maps[j], 128);
    std::memcpy(&maps.scales[j], scale_maps[j], 128);
    p.job[j] = GemmJob{rows[j], (rows[j] + kCtaRows - 1) / kCtaRows, formats[j], out_offsets[j]};
    tiles += p.job[j].mtiles;
  }
  for (uint32_t j = njobs; j < 3; ++j) {
    std::memcpy(&maps.codes[j], codes_maps[0], 128);
    std::memcpy(&maps.scales[j], scale_maps[0], 128);
  }
  std::memcpy(&maps.b, map_b, 128);
  const uint32_t kblocks = cols / kKBlock;
  p.njobs = njobs;
  p.cols = cols;
  p.streams = streams;
  p.kb_per_split = (kblocks + splits - 1) / splits;
  p.out = out;
  p.out_ld = out_ld;
  p.error = error;
  p.timeout_ns = timeout_ns;
  const uint32_t real_splits = (kblocks + p.kb_per_split - 1) / p.kb_per_split;
  const int smem = gemm_smem_bytes();
  return static_cast<int>(launch_pdl(gemm_streams_kernel, dim3(tiles, real_splits, col_blocks), dim3(kGemmThreads), smem,
                                     static_cast<cudaStream_t>(stream), maps, p));
}

int prepare_gemm_dense_kernel() {
  return static_cast<int>(cudaFuncSetAttribute(gemm_dense_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(sizeof(DenseSmem)) + 1024));
}

int32_t gemm_dense_weight_map(const void* weights, uint32_t rows, uint32_t kpad, uint8_t* out) {
  const uint64_t dims[2] = {kpad, rows};
  const uint64_t str[1] = {uint64_t(kpad) * 2};
  const uint32_t box[2] = {kKBlock, kTileM};
  return encode_tensor_map(out, kMapF16, 2, const_cast<void*>(weights), dims, str, box, true);
}

int launch_gemm_dense(const uint8_t* map_a, const uint8_t* map_b, uint32_t rows, uint32_t kpad, uint32_t columns,
                      uint32_t splits, float* out, int32_t* error, uint64_t timeout_ns, void* stream) {
  DenseMaps maps;
  std::memcpy(&maps.a, map_a, 128);
  std::memcpy(&maps.b, map_b, 128);
  DenseParams p{};
  p.rows = rows;
  p.kblocks = kpad / kKBlock;
  p.kb_per_split = (p.kblocks + splits - 1) / splits;
  p.columns = columns;
  p.out = out;
  p.error = error;
  p.timeout_ns = timeout_ns;
  const uint32_t real_splits = (p.kblocks + p.kb_per_split - 1) / p.kb_per_split;
  const dim3 grid((rows + kCtaRows - 1) / kCtaRows, real_splits, (columns + kStreamCols - 1) / kStreamCols);
  return static_cast<int>(launch_pdl(gemm_dense_kernel, grid, dim3(kGemmThreads),
                                     static_cast<int>(sizeof(DenseSmem)) + 1024, static_cast<cudaStream_t>(stream),
                                     maps, p));
}

int launch_gemm_streams(const uint8_t* map_codes, const uint8_t* map_scales, const uint8_t* map_b, uint32_t rows,
                        uint32_t cols, uint32_t format, uint32_t splits, float* out, int32_t* error, void* stream) {
  const uint8_t(*cm)[128] = reinterpret_cast<const uint8_t(*)[128]>(map_codes);
  const uint8_t(*sm)[128] = reinterpret_cast<const uint8_t(*)[128]>(map_scales);
  const uint32_t off = 0;
  return launch_gemm_jobs(cm, sm, &rows, &format, &off, 1, map_b, cols, kStreamCols, splits, out, rows, error, stream);
}

}  // namespace qwc

using namespace qwc;

namespace {

int32_t gemm_status(cudaError_t e) {
  if (e == cudaSuccess) return QWC_OK;
  cudaGetLastError();
  return e == cudaErrorMemoryAllocation ? QWC_OUT_OF_MEMORY : QWC_INVALID_STATE;
}

}  // namespace

extern "C" int32_t qwc_op_gemm_streams(uint32_t format, const void* scales, const void* codes, uint32_t rows,
                                       uint32_t cols, const float* x, uint32_t streams, float* out, void* stream) {
  if (!scales || !codes || !x || !out || rows == 0) return QWC_INVALID_ARGUMENT;
  if (format != kFormatQ4 && format != kFormatQ5 && format != kFormatQ8) return QWC_UNSUPPORTED;
  if (cols == 0 || cols % 512 != 0 || streams == 0 || streams > kStreamCols) return QWC_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(scales) % 16 != 0 || reinterpret_cast<uintptr_t>(codes) % 16 != 0) {
    return QWC_INVALID_ARGUMENT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int sms = 148;
  int device = 0;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const uint32_t kblocks = cols / kKBlock;
  const uint32_t want = gemm_splits(rows, cols, sms);
  const uint32_t kps = (kblocks + want - 1) / want;
  const uint32_t splits = (kblocks + kps - 1) / kps;

  // Workspace: error word, packed activations, split partials.
  const size_t xb_bytes = (size_t(kTileN) * cols * 2 + 255) / 256 * 256;
  const size_t part_bytes = size_t(splits) * streams * rows * 4;
  void* ws = nullptr;
  cudaError_t e = cudaMallocAsync(&ws, 256 + xb_bytes + part_bytes, st);
  if (e != cudaSuccess) return gemm_status(e);
  int32_t* err = static_cast<int32_t*>(ws);
  __half* xb = reinterpret_cast<__half*>(static_cast<uint8_t*>(ws) + 256);
  float* parts = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + 256 + xb_bytes);
  cudaMemsetAsync(ws, 0, 256 + xb_bytes, st);
  pack_activations_kernel<<<256, 256, 0, st>>>(x, streams, cols, xb);

  alignas(64) uint8_t maps[3][128];
  int32_t rc = gemm_weight_maps(format, codes, scales, rows, cols, maps[0], maps[1]);
  if (rc == QWC_OK) rc = gemm_act_map(xb, cols, maps[2]);
  if (rc != QWC_OK) {
    cudaFreeAsync(ws, st);
    return rc;
  }
  const uint32_t off = 0;
  int le = prepare_gemm_kernel();
  if (le == 0) le = launch_gemm_jobs(reinterpret_cast<const uint8_t(*)[128]>(maps[0]),
                            reinterpret_cast<const uint8_t(*)[128]>(maps[1]), &rows, &format, &off, 1, maps[2], cols,
                            streams, splits, parts, rows, err, st);
  e = static_cast<cudaError_t>(le);
  if (e == cudaSuccess) {
    sum_splits_kernel<<<256, 256, 0, st>>>(parts, splits, streams * rows, out);
    e = cudaGetLastError();
  }
  int32_t herr = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  cudaFreeAsync(ws, st);
  if (e != cudaSuccess) return gemm_status(e);
  return herr != 0 ? QWC_INVALID_STATE : QWC_OK;
}

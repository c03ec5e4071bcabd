// qwc_shard.cpp -- the `.qw` shard container (QWSHARD1) read in place.
//
// A restatement of the reference's container parse (src/core/container.zig):
// a 32-byte header, a tensor index of 40-byte entries sorted by (layer, kind),
// and a payload that starts on a 256-byte boundary with every tensor on a
// 16-byte boundary. Quantized tensors hold their f16 scale plane first and
// their code plane at the next 16-byte boundary (src/core/quant.zig:144-176).
// The parse validates everything container.File.parse and verifyChecksum do,
// with the same error-to-status mapping as src/wasm/abi.zig:91-147. It reads
// the caller's bytes and allocates nothing.

#include <cstdint>
#include <cstring>

#include "qwc_shard.h"
#include "qwenscriber_cuda.h"

namespace qwc {
namespace {

constexpr uint32_t kHeaderBytes = 32;        // container.zig:58
constexpr uint32_t kEntryBytes = 40;         // container.zig:59
constexpr uint32_t kFormatVersion = 1;       // container.zig:57
constexpr uint64_t kPayloadAlignment = 256;  // container.zig:62
constexpr uint64_t kTensorAlignment = 16;    // quant.zig:63
constexpr uint32_t kRankMax = 4;             // tensor.zig:20
constexpr uint32_t kDimsMax = 1u << 24;      // tensor.zig:21
constexpr uint32_t kGroupSize = 64;          // quant.zig:49

uint16_t rd16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t rd32(const uint8_t* p) { return uint32_t(p[0]) | (uint32_t(p[1]) << 8) | (uint32_t(p[2]) << 16) | (uint32_t(p[3]) << 24); }
uint64_t rd64(const uint8_t* p) { return uint64_t(rd32(p)) | (uint64_t(rd32(p + 4)) << 32); }

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// dtype.zig:17-23 and its element sizes; 0 for an unknown format.
uint32_t element_bytes(uint32_t format) {
  switch (format) {
    case QWC_FORMAT_F32:
      return 4;
    case QWC_FORMAT_F16:
    case QWC_FORMAT_BF16:
      return 2;
    default:
      return 0;
  }
}

uint32_t data_bytes_per_group(uint32_t format) {
  switch (format) {
    case QWC_FORMAT_Q4:
      return 32;
    case QWC_FORMAT_Q5:
      return 40;
    case QWC_FORMAT_Q8:
      return 64;
    default:
      return 0;
  }
}

bool quantized(uint32_t format) { return data_bytes_per_group(format) != 0; }
bool known(uint32_t format) { return quantized(format) || element_bytes(format) != 0; }

// Entry.validate (container.zig:142-160): a known format, a shape of rank 1..4
// with no zero or oversized extent, quantized formats only on matrices whose
// rows hold whole groups, and a recorded length equal to the shape's bytes.
int32_t validate_entry(const ShardEntry& e) {
  if (!known(e.format)) return QWC_UNSUPPORTED_MODEL;
  if (e.rank == 0 || e.rank > kRankMax) return QWC_SHAPE_MISMATCH;
  uint64_t count = 1;
  for (uint32_t i = 0; i < e.rank; ++i) {
    if (e.dims[i] == 0 || e.dims[i] > kDimsMax) return QWC_SHAPE_MISMATCH;
    if (count > UINT64_MAX / 8 / e.dims[i]) return QWC_SHAPE_MISMATCH;  // CountOverflow
    count *= e.dims[i];
  }
  uint64_t expected = 0;
  if (quantized(e.format)) {
    if (e.rank != 2 || e.dims[1] % kGroupSize != 0) return QWC_SHAPE_MISMATCH;
    const uint64_t groups = uint64_t(e.dims[0]) * (e.dims[1] / kGroupSize);
    expected = align_up(groups * 2, kTensorAlignment) + groups * data_bytes_per_group(e.format);
  } else {
    expected = count * element_bytes(e.format);
  }
  if (expected != e.len_bytes) return QWC_SHAPE_MISMATCH;  // ByteLengthMismatch
  return QWC_OK;
}

}  // namespace

// std.hash.Fnv1a_64 (offset basis 0xcbf29ce484222325, prime 0x100000001b3),
// truncated to its low 32 bits as the header stores it (container.zig:283-286).
uint32_t shard_checksum(const uint8_t* p, uint64_t n) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (uint64_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 0x100000001b3ull;
  }
  return static_cast<uint32_t>(h);
}

ShardEntry shard_entry(const ShardView& v, uint32_t i) {
  const uint8_t* p = v.index + size_t(i) * kEntryBytes;
  ShardEntry e;
  e.kind = rd16(p);
  e.layer = rd16(p + 2);
  e.format = p[4];
  e.rank = p[5];
  for (uint32_t d = 0; d < kRankMax; ++d) e.dims[d] = rd32(p + 8 + 4 * d);
  e.offset_bytes = rd64(p + 24);
  e.len_bytes = rd64(p + 32);
  return e;
}

int32_t parse_shard(const void* bytes, uint64_t len, ShardView* out) {
  if (!bytes || !out) return QWC_INVALID_ARGUMENT;
  // The readers alias the caller's buffer, which must be 16-byte aligned
  // (Error.Misaligned, mapped to invalid_argument).
  if (reinterpret_cast<uintptr_t>(bytes) % 16 != 0) return QWC_INVALID_ARGUMENT;
  const uint8_t* b = static_cast<const uint8_t*>(bytes);
  if (len < kHeaderBytes) return QWC_TRUNCATED;
  // Header.validate (container.zig:98-110).
  if (std::memcmp(b, "QWSHARD1", 8) != 0) return QWC_BAD_MAGIC;
  if (rd32(b + 8) != kFormatVersion) return QWC_BAD_VERSION;
  const uint32_t index_len = rd32(b + 12);
  const uint32_t payload_offset = rd32(b + 16);
  const uint32_t payload_len = rd32(b + 20);
  const uint32_t count = rd32(b + 24);
  const uint32_t checksum = rd32(b + 28);
  if (uint64_t(index_len) != uint64_t(count) * kEntryBytes) return QWC_TRUNCATED;
  if (uint64_t(payload_offset) < uint64_t(kHeaderBytes) + index_len) return QWC_TRUNCATED;
  if (payload_offset % kPayloadAlignment != 0) return QWC_TRUNCATED;
  // File.parse (container.zig:176-190).
  if (len < uint64_t(kHeaderBytes) + index_len) return QWC_TRUNCATED;
  if (len < uint64_t(payload_offset) + payload_len) return QWC_TRUNCATED;
  ShardView v;
  v.bytes = b;
  v.len = len;
  v.index = b + kHeaderBytes;
  v.count = count;
  v.payload = b + payload_offset;
  v.payload_len = payload_len;
  v.checksum = checksum;
  // File.validate (container.zig:192-216): every entry valid, keys strictly
  // ascending, ranges in order, inside the payload and 16-byte aligned.
  uint64_t previous_end = 0;
  uint32_t previous_key = 0;
  for (uint32_t i = 0; i < count; ++i) {
    const ShardEntry e = shard_entry(v, i);
    const int32_t rc = validate_entry(e);
    if (rc != QWC_OK) return rc;
    const uint32_t key = (uint32_t(e.layer) << 16) | e.kind;
    if (i > 0 && key <= previous_key) return QWC_INVALID_ARGUMENT;  // IndexNotSorted
    previous_key = key;
    if (e.offset_bytes < previous_end) return QWC_INVALID_ARGUMENT;  // TensorRangesOverlap
    const uint64_t end = e.offset_bytes + e.len_bytes;
    if (end < e.offset_bytes || end > payload_len) return QWC_TRUNCATED;
    previous_end = end;
    if (e.offset_bytes % kTensorAlignment != 0) return QWC_INVALID_ARGUMENT;  // TensorRangesOverlap
  }
  // verifyChecksum (container.zig:288-291), as addShard runs it (model.zig:160).
  if (shard_checksum(v.payload, payload_len) != checksum) return QWC_CHECKSUM_MISMATCH;
  *out = v;
  return QWC_OK;
}

}  // namespace qwc

extern "C" uint32_t qwc_shard_checksum(const void* bytes, uint64_t len) {
  return qwc::shard_checksum(static_cast<const uint8_t*>(bytes), bytes ? len : 0);
}

extern "C" int32_t qwc_shard_validate(const void* bytes, uint64_t len, uint32_t* tensor_count) {
  qwc::ShardView v;
  const int32_t rc = qwc::parse_shard(bytes, len, &v);
  if (rc == QWC_OK && tensor_count) *tensor_count = v.count;
  return rc;
}

// qwc_shard.h -- QWSHARD1 container parse shared by the model loader.
#pragma once

#include <cstdint>

namespace qwc {

// One index entry (src/core/container.zig:113-133).
struct ShardEntry {
  uint32_t kind, layer, format, rank;
  uint32_t dims[4];
  uint64_t offset_bytes, len_bytes;  // relative to the payload section
};

// A validated shard; every pointer aliases the caller's bytes.
struct ShardView {
  const uint8_t* bytes = nullptr;
  uint64_t len = 0;
  const uint8_t* index = nullptr;
  uint32_t count = 0;
  const uint8_t* payload = nullptr;
  uint32_t payload_len = 0;
  uint32_t checksum = 0;
};

// Full validation (header, index order and ranges, entry shapes and lengths,
// payload checksum); QWC_OK or the reference's status for the first failure.
int32_t parse_shard(const void* bytes, uint64_t len, ShardView* out);
ShardEntry shard_entry(const ShardView& v, uint32_t i);
uint32_t shard_checksum(const uint8_t* p, uint64_t n);

}  // namespace qwc

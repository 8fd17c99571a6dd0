// The persistent KV metadata table (kv_metadata.cu), shared with the store.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

#include "tpusync_b200.h"

namespace tsb {
namespace meta {

struct Record {
  int block_id;
  std::string hash;
  uint64_t seq;
};

uint64_t required_bytes(int num_blocks);

// A formatted or attached table on some region (not owned).
struct Table {
  void* base = nullptr;
  int blocks = 0;
  int format(void* region, uint64_t size, int num_blocks, const std::string& uid);
  int attach(void* region, uint64_t size, int num_blocks, const std::string& uid);
  int set(int block_id, const void* hash, size_t len, uint64_t seq);
  int clear(int block_id);
  std::vector<Record> valid_entries() const;
};

}  // namespace meta
}  // namespace tsb

struct ts_kv_metadata;
// The table behind a handle (kv_metadata.cu).
tsb::meta::Table* ts_kv_metadata_table(ts_kv_metadata* m);

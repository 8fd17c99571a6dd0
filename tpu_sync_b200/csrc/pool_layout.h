// Pool / region geometry shared by pool_layout.cu, the manager's pool copies
// and the pool reshard planner.
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include "tpusync_b200.h"

namespace tsb {
namespace pool {

// A strided run of live bytes inside one pool block (RegionSpec).
struct Region {
  std::string name;
  int64_t offset_bytes = 0;
  int64_t stride_bytes = 0;
  int64_t unit_bytes = 0;
  int64_t num_units = 0;
  int64_t units_per_stride = 1;

  int64_t live_bytes() const;        // INT64_MAX on overflow
  int64_t extent_end_bytes() const;  // INT64_MAX on overflow or negative geometry
  int validate(int64_t slot_bytes) const;
};

// num_blocks equally strided blocks of one storage, each with the same
// regions (PoolSpec).
struct Pool {
  std::string tag;
  int64_t storage_index = 0;
  int64_t base_offset_bytes = 0;
  int64_t block_stride_bytes = 0;
  int64_t num_blocks = 0;
  std::vector<Region> regions;
  std::string dtype_tag;

  int64_t storage_extent_end_bytes() const;
  int64_t block_live_end() const;  // max region extent end inside one block
  // storage_bytes < 0: internal consistency only.
  int validate(int64_t storage_bytes) const;
};

struct Extent {
  int64_t offset = 0;
  int64_t size = 0;
};

bool regions_cover_range(const std::vector<Region>& regions, uint64_t start, uint64_t end);
int copy_extents(const Pool& pool, const int64_t* ids, int64_t n, std::vector<Extent>* out);
int live_segments(const Pool& pool, std::vector<ts_live_segment>* out);
int physical_to_logical(const ts_live_segment* seg, int64_t n, int64_t phys, int64_t size,
                        int64_t* start, int64_t* end);
int translate_live_copy(const ts_live_segment* src, int64_t n_src, const ts_live_segment* dst,
                        int64_t n_dst, int64_t src_off, int64_t dst_off, int64_t size,
                        std::vector<ts_live_copy_chunk>* out);
int from_c(const ts_pool_spec* c, Pool* out);

}  // namespace pool
}  // namespace tsb

// Pool / region byte geometry (pure host logic, no CUDA calls).
//
// Restates tpu_sync/kv_cache/pool_layout.cc: RegionSpec / PoolSpec
// validation (:120-229), the storage extent (:231-254), RegionsCoverRange
// (:256-272), ComputePoolBlockCopyExtents (:274-374), ExpandPoolLiveSegments
// (:376-472), PhysicalLiveRangeToLogical (:474-493) and TranslateLiveCopy
// (:554-602), with the reference's status codes and messages (callers and
// tests match on them).  Every byte computation is overflow-checked in int64
// as there.

#include <algorithm>
#include <climits>
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "pool_layout.h"
#include "ts_internal.h"

namespace tsb {
namespace pool {

namespace {

constexpr int64_t kMax = INT64_MAX;
constexpr int64_t kMaxLiveSegments = int64_t{1} << 20;

bool mul_overflows(int64_t a, int64_t b) {
  if (a == 0 || b == 0) return false;
  return a > kMax / b;
}

// CheckedMul / CheckedAdd of pool_layout.cc:35-63: non-negative operands,
// result within int64; `what` names the quantity in the message.
int checked_mul(int64_t a, int64_t b, const std::string& what, int64_t* out) {
  if (a < 0 || b < 0) return set_error(TS_INVALID_ARGUMENT, what + " operands must be non-negative");
  if (mul_overflows(a, b)) return set_error(TS_INVALID_ARGUMENT, what + " overflows int64");
  *out = a * b;
  return TS_OK;
}

int checked_add(int64_t a, int64_t b, const std::string& what, int64_t* out) {
  if (a < 0 || b < 0) return set_error(TS_INVALID_ARGUMENT, what + " operands must be non-negative");
  if (a > kMax - b) return set_error(TS_INVALID_ARGUMENT, what + " overflows int64");
  *out = a + b;
  return TS_OK;
}

std::string S(int64_t v) { return std::to_string(v); }

// Which [segment_start, segment_end) of `r` holds `offset`, if any
// (RegionCoversOffset, pool_layout.cc:65-87).
bool region_covers(const Region& r, uint64_t offset, uint64_t* covered_end) {
  if (r.num_units <= 0) return false;
  const uint64_t base = uint64_t(r.offset_bytes);
  const uint64_t stride = uint64_t(r.stride_bytes);
  const uint64_t packed = uint64_t(r.unit_bytes) * uint64_t(r.units_per_stride);
  const uint64_t n = uint64_t(r.num_units);
  if (offset < base || packed == 0) return false;
  uint64_t unit = 0;
  if (n > 1) {
    if (stride == 0) return false;
    unit = (offset - base) / stride;
    if (unit >= n) return false;
  }
  const uint64_t start = base + unit * stride;
  const uint64_t end = start + packed;
  if (offset < start || offset >= end) return false;
  *covered_end = end;
  return true;
}

// Physical position of a compact-live offset and the bytes left in its run.
int locate(const ts_live_segment* seg, int64_t n, int64_t logical, int64_t* phys,
           int64_t* avail) {
  for (int64_t i = 0; i < n; ++i) {
    const ts_live_segment& s = seg[i];
    if (s.logical_offset <= logical && logical < s.logical_offset + s.size) {
      *phys = s.physical_offset + logical - s.logical_offset;
      *avail = s.logical_offset + s.size - logical;
      return TS_OK;
    }
  }
  return set_error(TS_INVALID_ARGUMENT, "Compact-live offset " + S(logical) + " is out of range");
}

}  // namespace

int64_t Region::live_bytes() const {
  if (mul_overflows(unit_bytes, num_units)) return kMax;
  const int64_t t = unit_bytes * num_units;
  if (mul_overflows(t, units_per_stride)) return kMax;
  return t * units_per_stride;
}

int64_t Region::extent_end_bytes() const {
  if (num_units == 0) return offset_bytes;
  if (num_units < 0 || stride_bytes < 0 || unit_bytes < 0 || units_per_stride < 0 ||
      offset_bytes < 0)
    return kMax;
  if (mul_overflows(num_units - 1, stride_bytes)) return kMax;
  const int64_t strided = (num_units - 1) * stride_bytes;
  if (mul_overflows(units_per_stride, unit_bytes)) return kMax;
  const int64_t packed = units_per_stride * unit_bytes;
  if (offset_bytes > kMax - strided) return kMax;
  const int64_t start = offset_bytes + strided;
  if (start > kMax - packed) return kMax;
  return start + packed;
}

int Region::validate(int64_t slot_bytes) const {
  const std::string r = "region " + name;
  if (name.empty()) return set_error(TS_INVALID_ARGUMENT, "region name must be non-empty");
  if (slot_bytes <= 0) return set_error(TS_INVALID_ARGUMENT, "slot_bytes must be positive");
  if (offset_bytes < 0) return set_error(TS_INVALID_ARGUMENT, r + " offset_bytes must be >= 0");
  if (stride_bytes < 0) return set_error(TS_INVALID_ARGUMENT, r + " stride_bytes must be >= 0");
  if (unit_bytes < 0) return set_error(TS_INVALID_ARGUMENT, r + " unit_bytes must be >= 0");
  if (num_units < 0) return set_error(TS_INVALID_ARGUMENT, r + " num_units must be >= 0");
  if (units_per_stride <= 0)
    return set_error(TS_INVALID_ARGUMENT, r + " units_per_stride must be positive");
  if (num_units > 0 && unit_bytes <= 0)
    return set_error(TS_INVALID_ARGUMENT, r + " unit_bytes must be positive");
  if (num_units > 1 && stride_bytes <= 0)
    return set_error(TS_INVALID_ARGUMENT, r + " stride_bytes must be positive");
  int64_t packed = 0, strided = 0, start = 0, end = 0;
  int rc = checked_mul(units_per_stride, unit_bytes, r + " packed unit bytes", &packed);
  if (rc != TS_OK) return rc;
  if (num_units > 0 && stride_bytes < packed)
    return set_error(TS_INVALID_ARGUMENT, r + " stride_bytes is smaller than packed units");
  rc = checked_mul(num_units > 0 ? num_units - 1 : 0, stride_bytes, r + " stride extent", &strided);
  if (rc != TS_OK) return rc;
  rc = checked_add(offset_bytes, strided, r + " extent start", &start);
  if (rc != TS_OK) return rc;
  rc = checked_add(start, packed, r + " extent end", &end);
  if (rc != TS_OK) return rc;
  if (end > slot_bytes)
    return set_error(TS_INVALID_ARGUMENT,
                     r + " exceeds slot bytes: end=" + S(end) + " slot=" + S(slot_bytes));
  return TS_OK;
}

int64_t Pool::storage_extent_end_bytes() const {
  if (base_offset_bytes < 0 || block_stride_bytes < 0 || num_blocks <= 0) return kMax;
  if (mul_overflows(num_blocks - 1, block_stride_bytes)) return kMax;
  const int64_t block_off = (num_blocks - 1) * block_stride_bytes;
  const int64_t live_end = block_live_end();
  if (base_offset_bytes > kMax - block_off) return kMax;
  const int64_t last = base_offset_bytes + block_off;
  if (live_end < 0 || last > kMax - live_end) return kMax;
  return last + live_end;
}

int64_t Pool::block_live_end() const {
  int64_t e = 0;
  for (const Region& r : regions) e = std::max(e, r.extent_end_bytes());
  return e;
}

int Pool::validate(int64_t storage_bytes) const {
  if (tag.empty()) return set_error(TS_INVALID_ARGUMENT, "pool tag must be non-empty");
  const std::string p = "pool " + tag;
  if (block_stride_bytes <= 0)
    return set_error(TS_INVALID_ARGUMENT, p + " block_stride_bytes must be positive");
  if (num_blocks <= 0) return set_error(TS_INVALID_ARGUMENT, p + " num_blocks must be positive");
  if (base_offset_bytes < 0)
    return set_error(TS_INVALID_ARGUMENT, p + " base_offset_bytes must be >= 0");
  if (regions.empty())
    return set_error(TS_INVALID_ARGUMENT, p + " must contain at least one region");
  for (const Region& r : regions) {
    if (r.validate(block_stride_bytes) != TS_OK)
      return set_error(TS_INVALID_ARGUMENT, p + ": " + ts_last_error());
  }
  if (storage_bytes >= 0) {
    const int64_t end = storage_extent_end_bytes();
    if (end == kMax)
      return set_error(TS_INVALID_ARGUMENT, p + " live storage extent overflows int64");
    if (end > storage_bytes)
      return set_error(TS_INVALID_ARGUMENT, p + " exceeds storage bytes (live regions): end=" +
                                                S(end) + " storage=" + S(storage_bytes));
  }
  return TS_OK;
}

bool regions_cover_range(const std::vector<Region>& regions, uint64_t start, uint64_t end) {
  uint64_t cursor = start;
  while (cursor < end) {
    uint64_t next = cursor;
    for (const Region& r : regions) {
      uint64_t covered = 0;
      if (region_covers(r, cursor, &covered)) next = std::max(next, std::min(covered, end));
    }
    if (next == cursor) return false;
    cursor = next;
  }
  return true;
}

int copy_extents(const Pool& pool, const int64_t* ids, int64_t n, std::vector<Extent>* out) {
  const std::string p = "pool " + pool.tag;
  std::vector<Extent> ext;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t id = ids[i];
    if (id < 0 || id >= pool.num_blocks)
      return set_error(TS_OUT_OF_RANGE, p + " block_id " + S(id) + " out of range [0, " +
                                            S(pool.num_blocks) + ")");
    int64_t delta = 0, base = 0;
    int rc = checked_mul(id, pool.block_stride_bytes, p + " block offset", &delta);
    if (rc == TS_OK) rc = checked_add(pool.base_offset_bytes, delta, p + " block base", &base);
    if (rc != TS_OK) return rc;
    for (const Region& r : pool.regions) {
      const std::string pr = p + " region " + r.name;
      int64_t packed = 0;
      rc = checked_mul(r.unit_bytes, r.units_per_stride, pr + " packed bytes", &packed);
      if (rc != TS_OK) return rc;
      if (r.num_units == 0 || packed == 0) continue;
      if (r.stride_bytes == packed) {
        // abutting units: one extent for the whole region
        int64_t bytes = 0, off = 0;
        rc = checked_mul(r.num_units, packed, pr + " live bytes", &bytes);
        if (rc == TS_OK) rc = checked_add(base, r.offset_bytes, pr + " offset", &off);
        if (rc != TS_OK) return rc;
        ext.push_back({off, bytes});
        continue;
      }
      for (int64_t u = 0; u < r.num_units; ++u) {
        int64_t ud = 0, rb = 0, off = 0;
        rc = checked_mul(u, r.stride_bytes, pr + " unit offset", &ud);
        if (rc == TS_OK) rc = checked_add(base, r.offset_bytes, pr + " base", &rb);
        if (rc == TS_OK) rc = checked_add(rb, ud, pr + " unit address", &off);
        if (rc != TS_OK) return rc;
        ext.push_back({off, packed});
      }
    }
  }
  std::sort(ext.begin(), ext.end(), [](const Extent& a, const Extent& b) {
    return a.offset != b.offset ? a.offset < b.offset : a.size < b.size;
  });
  std::vector<Extent> merged;
  merged.reserve(ext.size());
  for (const Extent& e : ext) {
    int64_t end = 0;
    int rc = checked_add(e.offset, e.size, p + " copy extent end", &end);
    if (rc != TS_OK) return rc;
    if (merged.empty()) {
      merged.push_back(e);
      continue;
    }
    Extent& prev = merged.back();
    int64_t prev_end = 0;
    rc = checked_add(prev.offset, prev.size, p + " previous copy extent end", &prev_end);
    if (rc != TS_OK) return rc;
    if (e.offset > prev_end) {
      merged.push_back(e);
      continue;
    }
    prev.size = std::max(prev_end, end) - prev.offset;
  }
  *out = std::move(merged);
  return TS_OK;
}

int live_segments(const Pool& pool, std::vector<ts_live_segment>* out) {
  const std::string p = "pool " + pool.tag;
  const int64_t stride = pool.block_stride_bytes;
  if (stride <= 0) return set_error(TS_INVALID_ARGUMENT, p + " has non-positive block stride");
  std::vector<std::pair<int64_t, int64_t>> iv;
  auto too_far = [&](int64_t end) {
    return set_error(TS_INVALID_ARGUMENT, p + " live region exceeds its block stride: end=" +
                                              S(end) + ", stride=" + S(stride));
  };
  for (const Region& r : pool.regions) {
    if (r.offset_bytes < 0 || r.stride_bytes < 0 || r.unit_bytes < 0 || r.num_units < 0)
      return set_error(TS_INVALID_ARGUMENT, p + " has negative region geometry");
    if (r.units_per_stride <= 0)
      return set_error(TS_INVALID_ARGUMENT, p + " has non-positive units_per_stride");
    if (mul_overflows(r.unit_bytes, r.units_per_stride))
      return set_error(TS_INVALID_ARGUMENT, p + " region byte geometry overflows");
    const int64_t packed = r.unit_bytes * r.units_per_stride;
    if (r.num_units > 0 && packed <= 0)
      return set_error(TS_INVALID_ARGUMENT, p + " has an empty live region");
    if (r.num_units > 1 && r.stride_bytes <= 0)
      return set_error(TS_INVALID_ARGUMENT, p + " has a non-positive region stride");
    if (r.num_units > 0 && r.stride_bytes < packed)
      return set_error(TS_INVALID_ARGUMENT, p + " has overlapping units within one region");
    if (int64_t(iv.size()) + r.num_units > kMaxLiveSegments)
      return set_error(TS_INVALID_ARGUMENT, p + " exceeds the live-region expansion bound");
    if (r.num_units > 0 && r.stride_bytes == packed) {
      if (mul_overflows(r.num_units, packed))
        return set_error(TS_INVALID_ARGUMENT, p + " region byte geometry overflows");
      const int64_t end = r.offset_bytes + r.num_units * packed;
      if (end > stride) return too_far(end);
      iv.emplace_back(r.offset_bytes, end);
      continue;
    }
    for (int64_t u = 0; u < r.num_units; ++u) {
      if (mul_overflows(u, r.stride_bytes))
        return set_error(TS_INVALID_ARGUMENT, p + " region byte geometry overflows");
      const int64_t start = r.offset_bytes + u * r.stride_bytes;
      const int64_t end = start + packed;
      if (end > stride) return too_far(end);
      iv.emplace_back(start, end);
    }
  }
  std::sort(iv.begin(), iv.end());
  std::vector<std::pair<int64_t, int64_t>> phys;
  for (const auto& [s, e] : iv) {
    if (!phys.empty() && s < phys.back().second)
      return set_error(TS_INVALID_ARGUMENT, p + " has overlapping live regions at byte " + S(s));
    if (!phys.empty() && s == phys.back().second)
      phys.back().second = e;
    else
      phys.emplace_back(s, e);
  }
  out->clear();
  out->reserve(phys.size());
  int64_t logical = 0;
  for (const auto& [s, e] : phys) {
    out->push_back({logical, s, e - s});
    logical += e - s;
  }
  return TS_OK;
}

int physical_to_logical(const ts_live_segment* seg, int64_t n, int64_t phys, int64_t size,
                        int64_t* start, int64_t* end) {
  if (phys < 0 || size <= 0)
    return set_error(TS_INVALID_ARGUMENT, "physical live range offset/size is invalid");
  const int64_t pend = phys + size;
  for (int64_t i = 0; i < n; ++i) {
    const ts_live_segment& s = seg[i];
    if (s.physical_offset <= phys && pend <= s.physical_offset + s.size) {
      *start = s.logical_offset + phys - s.physical_offset;
      *end = *start + size;
      return TS_OK;
    }
  }
  return set_error(TS_INVALID_ARGUMENT, "physical range [" + S(phys) + ", " + S(pend) +
                                            ") crosses padding or lies outside declared live "
                                            "regions");
}

int translate_live_copy(const ts_live_segment* src, int64_t n_src, const ts_live_segment* dst,
                        int64_t n_dst, int64_t src_off, int64_t dst_off, int64_t size,
                        std::vector<ts_live_copy_chunk>* out) {
  if (src_off < 0 || dst_off < 0 || size <= 0)
    return set_error(TS_INVALID_ARGUMENT, "Compact-live copy offsets/size are invalid");
  out->clear();
  int64_t left = size, sc = src_off, dc = dst_off;
  while (left > 0) {
    int64_t sp = 0, sa = 0, dp = 0, da = 0;
    int rc = locate(src, n_src, sc, &sp, &sa);
    if (rc == TS_OK) rc = locate(dst, n_dst, dc, &dp, &da);
    if (rc != TS_OK) return rc;
    const int64_t take = std::min({left, sa, da});
    out->push_back({sp, dp, take});
    if (int64_t(out->size()) > kMaxLiveSegments)
      return set_error(TS_INVALID_ARGUMENT, "Compact-live copy exceeds the segment expansion bound");
    sc += take;
    dc += take;
    left -= take;
  }
  return TS_OK;
}

int from_c(const ts_pool_spec* c, Pool* out) {
  if (!c) return set_error(TS_INVALID_ARGUMENT, "null pool spec");
  if (c->num_regions < 0 || (c->num_regions > 0 && !c->regions))
    return set_error(TS_INVALID_ARGUMENT, "pool regions must be a valid array");
  if (c->storage_index < 0)
    return set_error(TS_INVALID_ARGUMENT, std::string("pool ") + (c->tag ? c->tag : "") +
                                              " storage_index must be non-negative");
  out->tag = c->tag ? c->tag : "";
  out->dtype_tag = c->dtype_tag ? c->dtype_tag : "";
  out->storage_index = c->storage_index;
  out->base_offset_bytes = c->base_offset_bytes;
  out->block_stride_bytes = c->block_stride_bytes;
  out->num_blocks = c->num_blocks;
  out->regions.clear();
  for (int64_t i = 0; i < c->num_regions; ++i) {
    const ts_region_spec& r = c->regions[i];
    out->regions.push_back({r.name ? r.name : "", r.offset_bytes, r.stride_bytes, r.unit_bytes,
                            r.num_units, r.units_per_stride});
  }
  return TS_OK;
}

}  // namespace pool
}  // namespace tsb

using tsb::set_error;

namespace {

// Copies `v` into a caller array of capacity `cap`; *n_out = v.size().
template <typename T, typename F>
int emit(const std::vector<T>& v, int64_t cap, int64_t* n_out, F&& store) {
  if (n_out) *n_out = int64_t(v.size());
  if (int64_t(v.size()) > cap)
    return set_error(TS_RESOURCE_EXHAUSTED, "output capacity " + std::to_string(cap) +
                                                " is below the " + std::to_string(v.size()) +
                                                " results");
  for (size_t i = 0; i < v.size(); ++i) store(i, v[i]);
  return TS_OK;
}

std::vector<tsb::pool::Region> regions_from_c(const ts_region_spec* regions, int64_t n) {
  std::vector<tsb::pool::Region> rs;
  for (int64_t i = 0; i < n; ++i)
    rs.push_back({regions[i].name ? regions[i].name : "", regions[i].offset_bytes,
                  regions[i].stride_bytes, regions[i].unit_bytes, regions[i].num_units,
                  regions[i].units_per_stride});
  return rs;
}

}  // namespace

extern "C" int ts_pool_validate(const ts_pool_spec* pool, int64_t storage_bytes) {
  tsb::clear_error();
  tsb::pool::Pool p;
  int rc = tsb::pool::from_c(pool, &p);
  return rc != TS_OK ? rc : p.validate(storage_bytes);
}

extern "C" int ts_region_validate(const ts_region_spec* region, int64_t slot_bytes) {
  tsb::clear_error();
  if (!region) return set_error(TS_INVALID_ARGUMENT, "null region spec");
  return regions_from_c(region, 1)[0].validate(slot_bytes);
}

extern "C" int ts_pool_geometry(const ts_pool_spec* pool, int64_t* storage_extent_end,
                                int64_t* block_live_end, int64_t* live_bytes_per_block) {
  tsb::clear_error();
  tsb::pool::Pool p;
  int rc = tsb::pool::from_c(pool, &p);
  if (rc != TS_OK) return rc;
  if (storage_extent_end) *storage_extent_end = p.storage_extent_end_bytes();
  if (block_live_end) *block_live_end = p.block_live_end();
  if (live_bytes_per_block) {
    int64_t t = 0;
    for (const tsb::pool::Region& r : p.regions) {
      const int64_t lb = r.live_bytes();
      t = (lb == INT64_MAX || t > INT64_MAX - lb) ? INT64_MAX : t + lb;
    }
    *live_bytes_per_block = t;
  }
  return TS_OK;
}

extern "C" int ts_regions_cover_range(const ts_region_spec* regions, int64_t n, uint64_t start,
                                      uint64_t end, int* covered) {
  tsb::clear_error();
  if (!covered || n < 0 || (n > 0 && !regions))
    return set_error(TS_INVALID_ARGUMENT, "invalid regions or output");
  *covered = tsb::pool::regions_cover_range(regions_from_c(regions, n), start, end) ? 1 : 0;
  return TS_OK;
}

extern "C" int ts_pool_copy_extents(const ts_pool_spec* pool, const int64_t* block_ids,
                                    int64_t n_ids, ts_pool_extent* out, int64_t cap,
                                    int64_t* n_out) {
  tsb::clear_error();
  if (n_ids < 0 || (n_ids > 0 && !block_ids))
    return set_error(TS_INVALID_ARGUMENT, "block_ids must be a valid array");
  tsb::pool::Pool p;
  int rc = tsb::pool::from_c(pool, &p);
  if (rc != TS_OK) return rc;
  std::vector<tsb::pool::Extent> ext;
  rc = tsb::pool::copy_extents(p, block_ids, n_ids, &ext);
  if (rc != TS_OK) return rc;
  return emit(ext, out ? cap : 0, n_out, [&](size_t i, const tsb::pool::Extent& e) {
    out[i] = {e.offset, e.size};
  });
}

extern "C" int ts_pool_live_segments(const ts_pool_spec* pool, ts_live_segment* out, int64_t cap,
                                     int64_t* n_out) {
  tsb::clear_error();
  tsb::pool::Pool p;
  int rc = tsb::pool::from_c(pool, &p);
  if (rc != TS_OK) return rc;
  std::vector<ts_live_segment> seg;
  rc = tsb::pool::live_segments(p, &seg);
  if (rc != TS_OK) return rc;
  return emit(seg, out ? cap : 0, n_out,
              [&](size_t i, const ts_live_segment& s) { out[i] = s; });
}

extern "C" int ts_pool_physical_to_logical(const ts_live_segment* segments, int64_t n,
                                           int64_t physical_offset, int64_t size,
                                           int64_t* logical_start, int64_t* logical_end) {
  tsb::clear_error();
  if (n < 0 || (n > 0 && !segments) || !logical_start || !logical_end)
    return set_error(TS_INVALID_ARGUMENT, "invalid segments or output");
  return tsb::pool::physical_to_logical(segments, n, physical_offset, size, logical_start,
                                        logical_end);
}

extern "C" int ts_pool_translate_live_copy(const ts_live_segment* src, int64_t n_src,
                                           const ts_live_segment* dst, int64_t n_dst,
                                           int64_t src_offset, int64_t dst_offset, int64_t size,
                                           ts_live_copy_chunk* out, int64_t cap,
                                           int64_t* n_out) {
  tsb::clear_error();
  if (n_src < 0 || n_dst < 0 || (n_src > 0 && !src) || (n_dst > 0 && !dst))
    return set_error(TS_INVALID_ARGUMENT, "invalid segment arrays");
  std::vector<ts_live_copy_chunk> chunks;
  int rc = tsb::pool::translate_live_copy(src, n_src, dst, n_dst, src_offset, dst_offset, size,
                                          &chunks);
  if (rc != TS_OK) return rc;
  return emit(chunks, out ? cap : 0, n_out,
              [&](size_t i, const ts_live_copy_chunk& c) { out[i] = c; });
}

// Test driver around the REFERENCE pool geometry (tpu_sync/kv_cache/pool_layout.cc),
// compiled from the reference checkout by oracle/build_ref.py into
// oracle/_ref/pool_ref.  One request per stdin line, one result line out:
//
//   POOL   := tag storage base stride num_blocks dtype nreg {name off stride unit n ups}*
//   SEGS   := n {logical physical size}*
//   ext POOL k id*          -> "OK" {offset size}*          (ComputePoolBlockCopyExtents)
//   segs POOL               -> "OK" {logical physical size}* (ExpandPoolLiveSegments)
//   val POOL storage_bytes  -> "OK"                           (PoolSpec::Validate)
//   end POOL                -> "OK" storage_extent_end_bytes
//   p2l SEGS off size       -> "OK" start end                 (PhysicalLiveRangeToLogical)
//   xl SEGS SEGS so do size -> "OK" {src dst size}*           (TranslateLiveCopy)
//   cover nreg {region}* start end -> "OK" 0|1                (RegionsCoverRange)
// Errors print "ERR <absl code> <message>".  Names and tags contain no spaces
// ("-" stands for an empty string).
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "tpu_sync/kv_cache/pool_layout.h"

using namespace tpu_raiden::kv_cache;

static std::string unesc(const std::string& s) { return s == "-" ? "" : s; }

static RegionSpec read_region(std::istream& in) {
  RegionSpec r;
  std::string name;
  in >> name >> r.offset_bytes >> r.stride_bytes >> r.unit_bytes >> r.num_units >>
      r.units_per_stride;
  r.name = unesc(name);
  return r;
}

static PoolSpec read_pool(std::istream& in) {
  PoolSpec p;
  std::string tag, dtype;
  long long storage = 0;
  int nreg = 0;
  in >> tag >> storage >> p.base_offset_bytes >> p.block_stride_bytes >> p.num_blocks >> dtype >>
      nreg;
  p.tag = unesc(tag);
  p.storage_index = size_t(storage);
  p.dtype_tag = unesc(dtype);
  for (int i = 0; i < nreg; ++i) p.regions.push_back(read_region(in));
  return p;
}

static std::vector<PoolLiveSegment> read_segs(std::istream& in) {
  int n = 0;
  in >> n;
  std::vector<PoolLiveSegment> v(n);
  for (auto& s : v) in >> s.logical_offset >> s.physical_offset >> s.size;
  return v;
}

static void err(const absl::Status& s) {
  std::cout << "ERR " << int(s.code()) << " " << s.message() << "\n";
}

int main() {
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    std::string op;
    in >> op;
    if (op == "ext") {
      PoolSpec p = read_pool(in);
      int k = 0;
      in >> k;
      std::vector<int64_t> ids(k);
      for (auto& x : ids) in >> x;
      auto r = ComputePoolBlockCopyExtents(p, ids);
      if (!r.ok()) { err(r.status()); continue; }
      std::cout << "OK";
      for (const auto& e : *r) std::cout << " " << e.offset_bytes << " " << e.size_bytes;
      std::cout << "\n";
    } else if (op == "segs") {
      PoolSpec p = read_pool(in);
      auto r = ExpandPoolLiveSegments(p);
      if (!r.ok()) { err(r.status()); continue; }
      std::cout << "OK";
      for (const auto& s : *r)
        std::cout << " " << s.logical_offset << " " << s.physical_offset << " " << s.size;
      std::cout << "\n";
    } else if (op == "val") {
      PoolSpec p = read_pool(in);
      long long sb = 0;
      in >> sb;
      absl::Status s = p.Validate(sb);
      if (!s.ok()) { err(s); continue; }
      std::cout << "OK\n";
    } else if (op == "end") {
      PoolSpec p = read_pool(in);
      std::cout << "OK " << p.storage_extent_end_bytes() << "\n";
    } else if (op == "p2l") {
      auto segs = read_segs(in);
      long long off = 0, size = 0;
      in >> off >> size;
      auto r = PhysicalLiveRangeToLogical(segs, off, size);
      if (!r.ok()) { err(r.status()); continue; }
      std::cout << "OK " << r->first << " " << r->second << "\n";
    } else if (op == "xl") {
      auto a = read_segs(in);
      auto b = read_segs(in);
      long long so = 0, d = 0, size = 0;
      in >> so >> d >> size;
      auto r = TranslateLiveCopy(a, b, so, d, size);
      if (!r.ok()) { err(r.status()); continue; }
      std::cout << "OK";
      for (const auto& c : *r) std::cout << " " << c.src_physical << " " << c.dst_physical << " " << c.size;
      std::cout << "\n";
    } else if (op == "cover") {
      int n = 0;
      in >> n;
      std::vector<RegionSpec> rs;
      for (int i = 0; i < n; ++i) rs.push_back(read_region(in));
      unsigned long long s = 0, e = 0;
      in >> s >> e;
      std::cout << "OK " << (RegionsCoverRange(rs, s, e) ? 1 : 0) << "\n";
    } else {
      std::cout << "ERR -1 unknown op\n";
    }
    std::cout.flush();
  }
  return 0;
}

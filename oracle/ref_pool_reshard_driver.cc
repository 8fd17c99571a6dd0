// Test-oracle driver (TEST INFRASTRUCTURE ONLY): runs the reference's own
// pool reshard planning flow on requests read from stdin and prints each
// outcome as one JSON line.  Built by oracle/build_ref.py from the reference
// sources (pool_layout.cc, reshard/declaration_types.cc,
// reshard/work_unit_directory.cc, reshard/request_block_registry.cc,
// reshard/pool_reshard_planner.cc) with the stand-ins under oracle/shim.
//
// The flow is the reference service's: every unit is registered in a
// WorkUnitDirectory (WorkUnitDirectory::Validate + RegisterLocked,
// reshard/reshard_service.cc:335-343), every source unit registers its byte
// spans (RequestBlockRegistry::Register, reshard/reshard_service.cc:218),
// metadata comes from WorkUnitDirectory::LocalMetadata and the plan from
// BuildPoolReshardPlan (reshard/reshard_coordinator.cc:308-347).
//
// Input, whitespace-separated tokens (strings carry no spaces), per request:
//   REQ nu
//   nu x { transfer_parallelism transfer_rank n_pools pool* }
//   n_dst_pools pool*
//   n_tags tag*   n_ids id*   n_counts count* (-1: absent)
//   n_skips skip* (-1: absent)   parallelism (0: absent)
//   n_decls { unit tag version declared_bytes n_ids id* n_spans span* }
// pool = tag storage_index base_offset block_stride num_blocks dtype n_regions
//        { name offset stride unit_bytes num_units units_per_stride }*
// span = src_ordinal src_offset dst_index dst_offset size src_stride dst_stride count
//
// Unit u is RaidenId("src", "<u>", "kv", 0); the destination is
// RaidenId("dst", "0", "kv", 0).

#include <cstdint>
#include <iostream>
#include <map>
#include <sstream>
#include <string>
#include <vector>

#include "tpu_sync/kv_cache/reshard/declaration_types.h"
#include "tpu_sync/kv_cache/reshard/pool_reshard_planner.h"
#include "tpu_sync/kv_cache/reshard/request_block_registry.h"
#include "tpu_sync/kv_cache/reshard/work_unit_directory.h"

namespace rs = tpu_raiden::kv_cache::reshard;
using tpu_raiden::kv_cache::RaidenId;
using tpu_sync::rpc::PoolSpecProto;

namespace {

std::string Json(const std::string& s) {
  std::string o = "\"";
  for (char c : s) {
    if (c == '"' || c == '\\') {
      o += '\\';
      o += c;
    } else if (static_cast<unsigned char>(c) < 0x20) {
      char buf[8];
      snprintf(buf, sizeof(buf), "\\u%04x", c);
      o += buf;
    } else {
      o += c;
    }
  }
  return o + "\"";
}

template <typename T>
std::string List(const std::vector<T>& v) {
  std::ostringstream os;
  os << "[";
  for (size_t i = 0; i < v.size(); ++i) os << (i ? ", " : "") << v[i];
  os << "]";
  return os.str();
}

PoolSpecProto ReadPool(std::istream& in) {
  PoolSpecProto p;
  std::string tag, dtype;
  int64_t storage, base, stride, nb, nr;
  in >> tag >> storage >> base >> stride >> nb >> dtype >> nr;
  p.set_tag(tag);
  p.set_storage_index(storage);
  p.set_base_offset_bytes(base);
  p.set_block_stride_bytes(stride);
  p.set_num_blocks(nb);
  p.set_dtype_tag(dtype == "-" ? "" : dtype);  // "-" stands for an empty tag
  for (int64_t r = 0; r < nr; ++r) {
    std::string name;
    int64_t off, rs_, unit, num, ups;
    in >> name >> off >> rs_ >> unit >> num >> ups;
    auto* reg = p.add_regions();
    reg->set_name(name);
    reg->set_offset_bytes(off);
    reg->set_stride_bytes(rs_);
    reg->set_unit_bytes(unit);
    reg->set_num_units(num);
    reg->set_units_per_stride(ups);
  }
  return p;
}

std::vector<int64_t> ReadInts(std::istream& in, bool* present = nullptr) {
  int64_t n;
  in >> n;
  if (present) *present = n >= 0;
  std::vector<int64_t> v(n > 0 ? size_t(n) : 0);
  for (auto& x : v) in >> x;
  return v;
}

void Fail(const char* stage, const absl::Status& s) {
  std::cout << "{\"ok\": false, \"stage\": " << Json(stage) << ", \"code\": "
            << static_cast<int>(s.code()) << ", \"message\": " << Json(s.message()) << "}\n";
}

RaidenId Unit(const std::string& job, int idx) {
  RaidenId id;
  id.job_name = job;
  id.job_replica_id = std::to_string(idx);
  id.data_name = "kv";
  id.data_replica_idx = 0;
  return id;
}

void RunOne(std::istream& in, int64_t serial) {
  int nu;
  in >> nu;
  std::vector<int32_t> par(nu), rank(nu);
  std::vector<std::vector<PoolSpecProto>> src_pools(nu);
  for (int u = 0; u < nu; ++u) {
    int64_t np;
    in >> par[u] >> rank[u] >> np;
    for (int64_t i = 0; i < np; ++i) src_pools[u].push_back(ReadPool(in));
  }
  int64_t ndp;
  in >> ndp;
  std::vector<PoolSpecProto> dst_pools;
  for (int64_t i = 0; i < ndp; ++i) dst_pools.push_back(ReadPool(in));
  int64_t nt;
  in >> nt;
  std::vector<std::string> tags(nt);
  for (auto& t : tags) in >> t;
  std::vector<int64_t> ids = ReadInts(in);
  bool has_counts = false, has_skips = false;
  std::vector<int64_t> counts = ReadInts(in, &has_counts);
  std::vector<int64_t> skips = ReadInts(in, &has_skips);
  int32_t parallelism;
  in >> parallelism;
  int64_t nd;
  in >> nd;
  std::map<int, std::vector<rs::PoolSpanRegistration>> decls;
  for (int64_t d = 0; d < nd; ++d) {
    int unit;
    rs::PoolSpanRegistration r;
    in >> unit >> r.tag >> r.dst_space_version >> r.declared_bytes;
    r.block_ids = ReadInts(in);
    int64_t ns;
    in >> ns;
    for (int64_t s = 0; s < ns; ++s) {
      rs::PoolByteSpan sp;
      in >> sp.src_block_ordinal >> sp.src_offset_bytes >> sp.dst_block_index >>
          sp.dst_offset_bytes >> sp.size_bytes >> sp.src_stride_bytes >> sp.dst_stride_bytes >>
          sp.count;
      r.spans.push_back(sp);
    }
    decls[unit].push_back(std::move(r));
  }

  absl::Mutex mu;
  rs::WorkUnitDirectory dir(&mu);
  rs::RequestBlockRegistry registry(&dir, 3600.0, [] { return 0.0; });
  auto register_unit = [&](const RaidenId& id, const std::vector<PoolSpecProto>& pools,
                           int32_t p, int32_t r, const std::string& shard) -> absl::Status {
    rs::WorkUnitRegistration reg;
    reg.unit = id;
    reg.shards = {shard};
    reg.control_plane_rpc_address = "ctl-" + shard;
    reg.pool_manifest = pools;
    reg.layout_fingerprint = "layout-v1";
    reg.page_tokens = 16;
    reg.transfer_parallelism = p;
    reg.transfer_rank = r;
    absl::Status s = rs::WorkUnitDirectory::Validate(reg);
    if (!s.ok()) return s;
    absl::MutexLock lock(&mu);
    dir.RegisterLocked(reg);
    return absl::OkStatus();
  };
  std::vector<RaidenId> src_units;
  for (int u = 0; u < nu; ++u) {
    src_units.push_back(Unit("src", u));
    absl::Status s = register_unit(src_units.back(), src_pools[u], par[u], rank[u],
                                   "src-" + std::to_string(u));
    if (!s.ok()) return Fail("register_unit", s);
  }
  const RaidenId dst_unit = Unit("dst", 0);
  {
    absl::Status s = register_unit(dst_unit, dst_pools, 1, 0, "dst-0");
    if (!s.ok()) return Fail("register_unit", s);
  }
  const std::string req_id = "req-" + std::to_string(serial);
  const int64_t uuid = serial + 1;
  for (int u = 0; u < nu; ++u) {
    absl::Status s = registry.Register(req_id, uuid, src_units[u], {}, decls[u]);
    if (!s.ok()) return Fail("register_spans", s);
  }
  auto src_meta = dir.LocalMetadata(src_units);
  if (!src_meta.ok()) return Fail("metadata", src_meta.status());
  auto dst_meta = dir.LocalMetadata({dst_unit});
  if (!dst_meta.ok()) return Fail("metadata", dst_meta.status());

  rs::PlanRequest req;
  req.src_units = src_units;
  req.dst_units = {dst_unit};
  req.src_metadata = *src_meta;
  req.dst_metadata = *dst_meta;
  req.req_id = req_id;
  req.uuid = uuid;
  req.dst_device_block_ids = ids;
  req.transfer_pool_tags = tags;
  if (parallelism > 0) req.parallelism = parallelism;
  if (has_counts) req.dst_block_counts = counts;
  if (has_skips) req.dst_skip_bytes = skips;
  static int owner_tag = 0;
  auto plan = rs::BuildPoolReshardPlan(req, &registry, &owner_tag);
  if (!plan.ok()) return Fail("plan", plan.status());

  auto index_of = [&](const RaidenId& id) {
    for (int u = 0; u < nu; ++u)
      if (src_units[u] == id) return u;
    return -1;
  };
  std::ostringstream os;
  os << "{\"ok\": true, \"src_units\": [";
  for (size_t i = 0; i < plan->src_units.size(); ++i)
    os << (i ? ", " : "") << index_of(plan->src_units[i]);
  os << "], \"transfer_pool_indices\": " << List(plan->transfer_pool_indices)
     << ", \"expected_block_count\": " << plan->expected_block_count
     << ", \"expected_pushes_per_pool\": " << plan->expected_pushes_per_pool
     << ", \"parallelism\": " << plan->parallelism
     << ", \"dst_peer\": " << Json(plan->dst_peer)
     << ", \"dst_expected_extent_bytes\": " << List(plan->dst_expected_extent_bytes)
     << ", \"schedules\": {";
  bool first = true;
  for (const auto& [unit, entries] : plan->schedules) {
    os << (first ? "" : ", ") << "\"" << index_of(unit) << "\": [";
    first = false;
    for (size_t i = 0; i < entries.size(); ++i) {
      const rs::ScheduleEntry& e = entries[i];
      os << (i ? ", " : "") << "[" << e.src_block_id << ", " << e.dst_block_id << ", "
         << e.src_offset_bytes << ", " << e.dst_offset_bytes << ", " << e.size_bytes << ", "
         << e.pool_group << ", " << e.src_stride_bytes << ", " << e.dst_stride_bytes << ", "
         << e.count << ", " << e.dst_shard_idx << ", " << e.layer_idx << ", " << Json(e.dst_peer)
         << "]";
    }
    os << "]";
  }
  os << "}, \"groups\": [";
  for (size_t g = 0; g < plan->pool_groups.size(); ++g) {
    const rs::PlanPoolGroup& grp = plan->pool_groups[g];
    os << (g ? ", " : "") << "{\"pool_indices\": " << List(grp.pool_indices)
       << ", \"dst_device_block_ids\": " << List(grp.dst_device_block_ids)
       << ", \"expected_pushes\": " << grp.expected_pushes
       << ", \"dst_expected_extent_bytes\": " << List(grp.dst_expected_extent_bytes)
       << ", \"order_rank\": " << grp.order_rank << "}";
  }
  os << "], \"skipped_pool_counts\": {";
  first = true;
  for (const auto& [tag, n] : plan->skipped_pool_counts) {
    os << (first ? "" : ", ") << Json(tag) << ": " << n;
    first = false;
  }
  os << "}}";
  std::cout << os.str() << "\n";
}

}  // namespace

int main() {
  std::string word;
  int64_t serial = 0;
  while (std::cin >> word) {
    if (word != "REQ") {
      std::cerr << "expected REQ, got " << word << "\n";
      return 2;
    }
    RunOne(std::cin, serial++);
    std::cout.flush();
  }
  return 0;
}

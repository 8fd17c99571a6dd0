// Pool reshard: the prefill -> decode KV hand-off planner and its executor.
//
// Planner: restates the data-plane part of BuildPoolReshardPlan
// (tpu_sync/kv_cache/reshard/pool_reshard_planner.cc:132-859): manifest
// identity and geometry checks across source units, per-tag destination
// block split (dst_block_counts), destination clip (dst_skip_bytes), one live
// geometry per side and tag, page split of request-global spans
// (dst_space_version 1, :547-590), exactly-once prefix coverage of every
// destination block (:624-719), emission of (src block, dst block, src
// offset, dst offset, size) entries through TranslateLiveCopy in
// (dst block index, dst offset) order (:721-781) and the expected push
// counts.  Before planning it makes the checks the reference makes when the
// units and their byte-span declarations are registered
// (WorkUnitDirectory::Validate, kv_cache/reshard/work_unit_directory.cc:66-86;
// RequestBlockRegistry::Register, kv_cache/reshard/request_block_registry.cc:142-245),
// so a request fails with the message the reference gives at whichever step
// rejects it.  The registry claim, the units' network endpoints and the layout
// fingerprints are control plane and have no counterpart here; a source unit
// is named by its index (or a caller-given name) in messages.
//
// Executor: the reference D2Hs the source pool blocks, pushes them over TCP
// and the receiver H2Ds the entries' byte ranges (PoolReshardPush /
// OnPoolReceived, tpu_sync/core/kv_cache_manager_with_transfer.cc:1152-1335,
// :2665-2805).  Here one program per source GPU keeps, per pool group, the
// unit's entries merged into strided tasks relative to a pool (one device
// table) and the pools' block-0 addresses (a second, small table); one launch
// per group reads the source HBM and stores straight into the destination
// GPU's storages (peer pointers / IPC mappings over NVLink), one warp per
// (pool, task) of at most 64 KiB.  Every transferred pool's live extent is
// checked against the storage sizes the caller gives, so no task reaches
// outside a storage.

#include <cuda_runtime.h>

#include <algorithm>
#include <map>
#include <set>
#include <string>
#include <tuple>
#include <vector>

#include "pool_layout.h"
#include "ts_internal.h"

struct ts_pool_reshard_plan {
  struct Entry {
    int64_t src_block, dst_block, src_off, dst_off, size;
    int32_t group;
    int64_t src_stride = 0, dst_stride = 0;  // received plans: count repeats
    int32_t count = 1;
  };
  struct Group {
    std::vector<int32_t> pools;
    std::vector<int64_t> dst_ids;
    int32_t expected_pushes = 0;
    std::vector<int64_t> extents;
    int32_t order_rank = 0;
  };
  int64_t n_src_units = 0;
  std::vector<int64_t> active_units;                 // rank order, units with entries
  std::vector<std::vector<Entry>> schedules;         // per source unit
  std::vector<Group> groups;
  std::vector<int32_t> transfer_pool_indices;
  std::vector<std::pair<std::string, int64_t>> skipped;  // tag -> pools not transferred
  int32_t parallelism = 1;
  int64_t expected_block_count = 0;
  std::vector<tsb::pool::Pool> src_pools, dst_pools;  // geometry for the executor
};

namespace tsb {
// One merged run of entry bytes, relative to a pool: row r of `count` rows
// copies `bytes` from pool block src_block at src_off + r*src_stride to pool
// block dst_block at dst_off + r*dst_stride.
struct RelTask {
  int64_t src_block, src_off, dst_block, dst_off;
  int64_t src_stride, dst_stride;
  uint32_t bytes, count;
};
// Where one pool of the group lives: block 0 addresses and block strides.
struct PoolBase {
  uint64_t src, dst;
  int64_t src_stride, dst_stride;
};
}  // namespace tsb

struct ts_pool_reshard_program {
  int device = 0;
  struct Group {
    tsb::RelTask* d_tasks = nullptr;  // sorted by access width: 16-, 4-, 1-byte tasks
    tsb::PoolBase* d_pools = nullptr;
    int64_t n_tasks = 0, n_pools = 0;
    int64_t n16 = 0, n4 = 0;          // tasks of the first two widths
  };
  std::vector<Group> groups;
  int64_t n_tasks = 0;  // tasks x pools over all groups
  uint64_t bytes = 0;
};

namespace tsb {
namespace {

using Plan = ts_pool_reshard_plan;
constexpr int64_t kMaxLiveSegments = int64_t{1} << 20;

std::string S(int64_t v) { return std::to_string(v); }
std::string Q(const std::string& s) { return "'" + s + "'"; }

std::string int_list(const std::vector<int64_t>& v) {
  std::string out = "[";
  for (size_t i = 0; i < v.size(); ++i) out += (i ? ", " : "") + S(v[i]);
  return out + "]";
}

std::string geometry_signature(const pool::Pool& p) {
  std::string sig = p.tag + "\x1f" + S(p.storage_index) + "\x1f" + S(p.base_offset_bytes) +
                    "\x1f" + S(p.block_stride_bytes) + "\x1f" + S(p.num_blocks) + "\x1f" +
                    p.dtype_tag;
  for (const pool::Region& r : p.regions)
    sig += "\x1e" + r.name + "\x1f" + S(r.offset_bytes) + "\x1f" + S(r.stride_bytes) + "\x1f" +
           S(r.unit_bytes) + "\x1f" + S(r.num_units) + "\x1f" + S(r.units_per_stride);
  return sig;
}

struct Decl {
  int64_t unit = 0;
  std::vector<int64_t> block_ids;
  std::vector<ts_byte_span> spans;
  int64_t declared = 0;
  int32_t version = 0;
};

struct TagPre {
  std::vector<int32_t> selected;
  int64_t src_live = 0, dst_live = 0;
  std::vector<ts_live_segment> src_seg, dst_seg;
};

bool same_segments(const std::vector<ts_live_segment>& a, const std::vector<ts_live_segment>& b) {
  if (a.size() != b.size()) return false;
  for (size_t i = 0; i < a.size(); ++i)
    if (a[i].logical_offset != b[i].logical_offset || a[i].physical_offset != b[i].physical_offset ||
        a[i].size != b[i].size)
      return false;
  return true;
}

std::string S128(__int128 v) {
  if (v >= INT64_MIN && v <= INT64_MAX) return S(int64_t(v));
  const bool neg = v < 0;
  unsigned __int128 m = neg ? (unsigned __int128)(-(v + 1)) + 1 : (unsigned __int128)v;
  std::string d;
  while (m) {
    d.insert(d.begin(), char('0' + int(m % 10)));
    m /= 10;
  }
  return neg ? "-" + d : d;
}

// Unit registration (WorkUnitDirectory::Validate,
// kv_cache/reshard/work_unit_directory.cc:66-86): every source unit in
// order, then the destination.  A unit without an explicit
// transfer_parallelism declares the number of source units, without a rank
// its index.
int validate_unit_registrations(const ts_pool_reshard_request* rq, int64_t nu) {
  for (int64_t u = 0; u < nu; ++u) {
    if (rq->n_src_pools[u] <= 0)
      return set_error(TS_INVALID_ARGUMENT, "pool_manifest must not be empty");
    const int64_t par = rq->transfer_parallelism ? rq->transfer_parallelism[u] : nu;
    const int64_t rank = rq->transfer_ranks ? rq->transfer_ranks[u] : u;
    if (par <= 0) return set_error(TS_INVALID_ARGUMENT, "transfer_parallelism must be positive");
    if (rank < 0) return set_error(TS_INVALID_ARGUMENT, "transfer_rank must be non-negative");
    if (rank >= par)
      return set_error(TS_INVALID_ARGUMENT, "transfer_rank must be less than transfer_parallelism");
  }
  if (rq->n_dst_pools <= 0) return set_error(TS_INVALID_ARGUMENT, "pool_manifest must not be empty");
  return TS_OK;
}

// Byte-span registration (RequestBlockRegistry::Register,
// kv_cache/reshard/request_block_registry.cc:142-245): per source unit, in
// unit order, its declarations in the order given, against the live bytes of
// its manifest's pools per tag.  Arithmetic is widened so no overflow can
// let a span through.
template <typename UnitName>
int validate_span_registrations(const ts_pool_reshard_request* rq,
                                const std::vector<std::vector<pool::Pool>>& src,
                                const UnitName& unit_name) {
  constexpr int64_t kMaxSpanCount = int64_t{1} << 20;
  // a declaration of a unit the request does not have was never registered
  for (int64_t d = 0; d < rq->n_decls; ++d)
    if (rq->decls[d].src_unit < 0 || rq->decls[d].src_unit >= int64_t(src.size()))
      return set_error(TS_INVALID_ARGUMENT,
                       "Work unit is not registered: src unit " + S(rq->decls[d].src_unit));
  for (int64_t u = 0; u < int64_t(src.size()); ++u) {
    std::vector<const ts_span_decl*> mine;
    for (int64_t d = 0; d < rq->n_decls; ++d)
      if (rq->decls[d].src_unit == u) mine.push_back(&rq->decls[d]);
    if (mine.empty()) continue;
    std::map<std::string, int64_t> live_by_tag;
    for (const pool::Pool& p : src[size_t(u)]) {
      std::vector<ts_live_segment> seg;
      const int rc = pool::live_segments(p, &seg);
      if (rc != TS_OK) return rc;
      int64_t live = 0;
      for (const ts_live_segment& g : seg) live += g.size;
      auto [it, inserted] = live_by_tag.emplace(p.tag, live);
      if (!inserted && it->second != live)
        return set_error(TS_INVALID_ARGUMENT, "pools tagged " + p.tag + " disagree on live bytes for " +
                                                  unit_name(u) +
                                                  "; byte-span registration requires one geometry per tag");
    }
    std::set<std::string> seen;
    for (const ts_span_decl* sd : mine) {
      const std::string tag = sd->tag ? sd->tag : "";
      if (tag.empty()) return set_error(TS_INVALID_ARGUMENT, "pool span registration tag must not be empty");
      if (!seen.insert(tag).second)
        return set_error(TS_INVALID_ARGUMENT, "duplicate pool span registration tag: " + tag);
      auto live_it = live_by_tag.find(tag);
      if (live_it == live_by_tag.end())
        return set_error(TS_INVALID_ARGUMENT, "pool span registration " + tag +
                                                  " does not match any registered pool for " + unit_name(u));
      const int64_t live = live_it->second;
      const int64_t n_ids = sd->n_block_ids > 0 ? sd->n_block_ids : 0;
      for (int64_t i = 0; i < n_ids; ++i)
        if (sd->block_ids[i] < 0)
          return set_error(TS_INVALID_ARGUMENT, "pool span registration " + tag +
                                                    " block_ids must be non-negative");
      if (int64_t(std::set<int64_t>(sd->block_ids, sd->block_ids + n_ids).size()) != n_ids)
        return set_error(TS_INVALID_ARGUMENT, "pool span registration " + tag +
                                                  " block_ids must not contain duplicates");
      __int128 span_bytes = 0;
      for (int64_t k = 0; k < (sd->n_spans > 0 ? sd->n_spans : 0); ++k) {
        const ts_byte_span& sp = sd->spans[k];
        if (sp.size_bytes <= 0)
          return set_error(TS_INVALID_ARGUMENT, "byte span size_bytes must be positive (" + tag + ")");
        if (sp.count <= 0)
          return set_error(TS_INVALID_ARGUMENT, "byte span count must be positive (" + tag + ")");
        if (sp.count > kMaxSpanCount)
          return set_error(TS_INVALID_ARGUMENT, "byte span count " + S(sp.count) +
                                                    " exceeds the expansion bound (" + tag + ")");
        if (sp.src_offset_bytes < 0 || sp.dst_offset_bytes < 0 || sp.src_stride_bytes < 0 ||
            sp.dst_stride_bytes < 0 || sp.dst_block_index < 0)
          return set_error(TS_INVALID_ARGUMENT, "byte span fields must be non-negative (" + tag + ")");
        if (sp.src_block_ordinal < 0 || sp.src_block_ordinal >= n_ids)
          return set_error(TS_INVALID_ARGUMENT, "byte span ordinal " + S(sp.src_block_ordinal) +
                                                    " is outside the registration's " + S(n_ids) +
                                                    " block ids (" + tag + ")");
        const __int128 src_end = __int128(sp.src_offset_bytes) +
                                 __int128(sp.count - 1) * sp.src_stride_bytes + sp.size_bytes;
        if (src_end > live)
          return set_error(TS_INVALID_ARGUMENT, "byte span exceeds its source block live bytes (" + tag +
                                                    "): end=" + S128(src_end) + ", live=" + S(live));
        span_bytes += __int128(sp.size_bytes) * sp.count;
      }
      if (__int128(sd->declared_bytes) != span_bytes)
        return set_error(TS_INVALID_ARGUMENT, "pool span registration " + tag + " declared_bytes " +
                                                  S(sd->declared_bytes) + " disagrees with the span sum " +
                                                  S128(span_bytes));
    }
  }
  return TS_OK;
}

int build(const ts_pool_reshard_request* rq, Plan* plan) {
  const int64_t nu = rq->n_src_units;
  if (nu <= 0) return set_error(TS_INVALID_ARGUMENT, "src_units must not be empty");
  auto unit_name = [&](int64_t u) {
    return rq->unit_names && rq->unit_names[u] ? std::string(rq->unit_names[u])
                                               : "src unit " + S(u);
  };
  // registration-time checks first, as in the reference's flow
  if (int rc = validate_unit_registrations(rq, nu); rc != TS_OK) return rc;
  const int64_t np_dst = rq->n_dst_pools;
  std::vector<std::vector<pool::Pool>> src(static_cast<size_t>(nu));
  for (int64_t u = 0; u < nu; ++u) {
    if (rq->n_src_pools[u] <= 0)
      return set_error(TS_INVALID_ARGUMENT, "Missing explicit pool manifest for " + unit_name(u));
    for (int64_t i = 0; i < rq->n_src_pools[u]; ++i) {
      pool::Pool p;
      int rc = pool::from_c(&rq->src_pools[u][i], &p);
      if (rc != TS_OK) return rc;
      src[size_t(u)].push_back(std::move(p));
    }
  }
  std::vector<pool::Pool> dst;
  for (int64_t i = 0; i < np_dst; ++i) {
    pool::Pool p;
    int rc = pool::from_c(&rq->dst_pools[i], &p);
    if (rc != TS_OK) return rc;
    dst.push_back(std::move(p));
  }
  if (int rc = validate_span_registrations(rq, src, unit_name); rc != TS_OK) return rc;
  // BuildPoolReshardPlan proper
  std::vector<int64_t> dst_ids(rq->dst_block_ids, rq->dst_block_ids + rq->n_dst_block_ids);
  if (dst_ids.empty()) return set_error(TS_INVALID_ARGUMENT, "dst_device_block_ids must not be empty");
  for (int64_t b : dst_ids)
    if (b < 0) return set_error(TS_INVALID_ARGUMENT, "dst_device_block_ids must be non-negative");
  // canonical (tag, dtype_tag) manifests agree; source geometry agrees
  for (int64_t u = 0; u < nu; ++u) {
    bool same = src[size_t(u)].size() == dst.size();
    for (size_t i = 0; same && i < dst.size(); ++i)
      same = src[size_t(u)][i].tag == dst[i].tag && src[size_t(u)][i].dtype_tag == dst[i].dtype_tag;
    if (!same)
      return set_error(TS_INVALID_ARGUMENT,
                       "Canonical pool manifest mismatch between source and destination for " +
                           unit_name(u));
  }
  for (int64_t u = 1; u < nu; ++u)
    for (size_t i = 0; i < dst.size(); ++i)
      if (geometry_signature(src[size_t(u)][i]) != geometry_signature(src[0][i]))
        return set_error(TS_INVALID_ARGUMENT,
                         "Source pool geometry differs across ranks at " + unit_name(u));
  std::vector<std::string> tags;
  for (int64_t i = 0; i < rq->n_tags; ++i) tags.push_back(rq->tags[i] ? rq->tags[i] : "");
  if (tags.empty())
    return set_error(TS_INVALID_ARGUMENT, "transfer_pool_tags must name at least one pool tag");
  if (std::set<std::string>(tags.begin(), tags.end()).size() != tags.size()) {
    std::string l = "[";
    for (size_t i = 0; i < tags.size(); ++i) l += (i ? ", " : "") + Q(tags[i]);
    return set_error(TS_INVALID_ARGUMENT, "transfer_pool_tags must not repeat tags; got " + l + "]");
  }
  std::vector<int64_t> counts(rq->dst_block_counts, rq->dst_block_counts + rq->n_dst_block_counts);
  if (!counts.empty()) {
    if (counts.size() != tags.size())
      return set_error(TS_INVALID_ARGUMENT, "dst_block_counts must align 1:1 with transfer_pool_tags: " +
                                                S(int64_t(counts.size())) + " counts for " +
                                                S(int64_t(tags.size())) + " tags");
    int64_t sum = 0;
    bool bad = false;
    for (int64_t c : counts) {
      bad = bad || c <= 0;
      sum += c;
    }
    if (bad || sum != int64_t(dst_ids.size()))
      return set_error(TS_INVALID_ARGUMENT,
                       "dst_block_counts must be positive and sum to the destination block count: "
                       "counts=" + int_list(counts) + ", blocks=" + S(int64_t(dst_ids.size())));
  } else if (tags.size() == 1) {
    counts = {int64_t(dst_ids.size())};
  } else {
    return set_error(TS_INVALID_ARGUMENT,
                     "Multi-tag transfers must split dst_device_block_ids with dst_block_counts");
  }
  std::vector<std::vector<int64_t>> tag_dst;
  for (size_t c = 0, cur = 0; c < counts.size(); cur += size_t(counts[c]), ++c)
    tag_dst.emplace_back(dst_ids.begin() + long(cur), dst_ids.begin() + long(cur + size_t(counts[c])));
  std::vector<int64_t> skips(tags.size(), 0);
  if (rq->n_dst_skip_bytes > 0) {
    if (rq->n_dst_skip_bytes != int64_t(tags.size()))
      return set_error(TS_INVALID_ARGUMENT, "dst_skip_bytes must align 1:1 with transfer_pool_tags: " +
                                                S(rq->n_dst_skip_bytes) + " skips for " +
                                                S(int64_t(tags.size())) + " tags");
    for (size_t i = 0; i < tags.size(); ++i) {
      if (rq->dst_skip_bytes[i] < 0)
        return set_error(TS_INVALID_ARGUMENT, "dst_skip_bytes must be non-negative; tag " +
                                                  Q(tags[i]) + " requested " +
                                                  S(rq->dst_skip_bytes[i]));
      skips[i] = rq->dst_skip_bytes[i];
    }
  }
  {
    std::set<std::string> avail;
    for (const pool::Pool& p : dst) avail.insert(p.tag);
    for (const std::string& t : tags)
      if (!avail.count(t))
        return set_error(TS_INVALID_ARGUMENT,
                         "transfer_pool_tags do not match any registered pool: [" + Q(t) + "]");
  }
  std::set<int64_t> par;
  std::map<int64_t, int64_t> ranks;  // rank -> unit
  for (int64_t u = 0; u < nu; ++u) {
    par.insert(rq->transfer_parallelism ? rq->transfer_parallelism[u] : nu);
    ranks[rq->transfer_ranks ? rq->transfer_ranks[u] : u] = u;
  }
  if (par.size() != 1 || *par.begin() <= 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "All source ranks must declare one consistent positive transfer_parallelism");
  const int64_t topo = *par.begin();
  if (int64_t(ranks.size()) != nu)
    return set_error(TS_INVALID_ARGUMENT, "Source transfer_rank values must be unique");
  {
    int64_t want = 0;
    for (const auto& [r, u] : ranks)
      if (r != want++)
        return set_error(TS_INVALID_ARGUMENT, "Source transfer_rank values must be contiguous from zero");
  }
  const int64_t parallelism = rq->parallelism > 0 ? rq->parallelism : topo;
  if (rq->parallelism < 0) return set_error(TS_INVALID_ARGUMENT, "parallelism must be positive");
  if (parallelism > topo)
    return set_error(TS_INVALID_ARGUMENT, "parallelism exceeds source admission: requested=" +
                                              S(parallelism) + ", admitted=" + S(topo));

  // per-tag prechecks (before any planning)
  std::vector<TagPre> pre;
  for (size_t g = 0; g < tags.size(); ++g) {
    const std::vector<int64_t>& ids = tag_dst[g];
    if (std::set<int64_t>(ids.begin(), ids.end()).size() != ids.size())
      return set_error(TS_INVALID_ARGUMENT, "dst_device_block_ids for tag " + Q(tags[g]) +
                                                " must not contain duplicates");
    TagPre tp;
    for (size_t i = 0; i < dst.size(); ++i)
      if (dst[i].tag == tags[g]) tp.selected.push_back(int32_t(i));
    std::set<int64_t> sl, dl;
    std::vector<std::vector<ts_live_segment>> smaps, dmaps;
    for (int32_t pi : tp.selected) {
      std::vector<ts_live_segment> ss, ds;
      int rc = pool::live_segments(src[0][size_t(pi)], &ss);
      if (rc == TS_OK) rc = pool::live_segments(dst[size_t(pi)], &ds);
      if (rc != TS_OK) return rc;
      int64_t s_live = 0, d_live = 0;
      for (const auto& x : ss) s_live += x.size;
      for (const auto& x : ds) d_live += x.size;
      if (s_live <= 0 || d_live <= 0)
        return set_error(TS_INVALID_ARGUMENT, "Pool " + S(pi) + " has no declared live bytes");
      sl.insert(s_live);
      dl.insert(d_live);
      bool seen = false;
      for (const auto& m : smaps) seen = seen || same_segments(m, ss);
      if (!seen) smaps.push_back(ss);
      seen = false;
      for (const auto& m : dmaps) seen = seen || same_segments(m, ds);
      if (!seen) dmaps.push_back(ds);
    }
    if (sl.size() != 1 || dl.size() != 1) {
      std::vector<int64_t> a(sl.begin(), sl.end()), b(dl.begin(), dl.end());
      return set_error(TS_INVALID_ARGUMENT, "Pools tagged " + tags[g] +
                                                " must share one geometry per side; src=" +
                                                int_list(a) + " dst=" + int_list(b));
    }
    if (smaps.size() != 1 || dmaps.size() != 1)
      return set_error(TS_INVALID_ARGUMENT,
                       "Pools tagged " + tags[g] + " must share one live-region map per side");
    tp.src_live = *sl.begin();
    tp.dst_live = *dl.begin();
    if (skips[g] % tp.dst_live != 0)
      return set_error(TS_INVALID_ARGUMENT,
                       "dst_skip_bytes must be a whole multiple of the destination page live bytes "
                       "for tag " + Q(tags[g]) + ": skip=" + S(skips[g]) +
                           ", page_live_bytes=" + S(tp.dst_live));
    tp.src_seg = std::move(smaps[0]);
    tp.dst_seg = std::move(dmaps[0]);
    pre.push_back(std::move(tp));
  }

  plan->n_src_units = nu;
  plan->schedules.assign(size_t(nu), {});
  std::vector<int32_t> union_sel;
  int64_t emitted = 0;
  for (size_t g = 0; g < tags.size(); ++g) {
    const std::string& tag = tags[g];
    const std::vector<int64_t>& ids = tag_dst[g];
    const TagPre& tp = pre[g];
    const int64_t src_live = tp.src_live, dst_live = tp.dst_live, skip = skips[g];
    // declarations of this tag, in source-unit order then declaration order
    std::vector<Decl> declared;
    for (int64_t u = 0; u < nu; ++u)
      for (int64_t d = 0; d < rq->n_decls; ++d) {
        const ts_span_decl& sd = rq->decls[d];
        if (sd.src_unit != u || !sd.tag || tag != sd.tag || sd.n_spans <= 0) continue;
        Decl x;
        x.unit = u;
        x.block_ids.assign(sd.block_ids, sd.block_ids + sd.n_block_ids);
        x.spans.assign(sd.spans, sd.spans + sd.n_spans);
        x.declared = sd.declared_bytes;
        x.version = sd.dst_space_version;
        declared.push_back(std::move(x));
      }
    if (declared.empty())
      return set_error(TS_INVALID_ARGUMENT, "No byte-span declarations are registered for tag " + tag);
    // request-global (v1) spans: split at destination pages, clip, re-base
    int64_t clipped = 0, global_end = 0;
    for (Decl& x : declared) {
      if (x.version == 0) {
        if (skip > 0)
          return set_error(TS_INVALID_ARGUMENT,
                           "dst_skip_bytes requires destination-page-agnostic (dst_space_version=1) "
                           "declarations for tag " + Q(tag) + " (declared by " + unit_name(x.unit) + ")");
        continue;
      }
      std::vector<ts_byte_span> split;
      for (const ts_byte_span& sp : x.spans) {
        if (sp.count > 1 || sp.src_stride_bytes != 0 || sp.dst_stride_bytes != 0)
          return set_error(TS_INVALID_ARGUMENT,
                           "Global-space byte spans must be plain contiguous ranges (declared by " +
                               unit_name(x.unit) + ")");
        if (sp.dst_block_index != 0)
          return set_error(TS_INVALID_ARGUMENT,
                           "Global-space byte spans must leave dst_block_index zero (declared by " +
                               unit_name(x.unit) + ")");
        global_end = std::max(global_end, sp.dst_offset_bytes + sp.size_bytes);
        int64_t adv = 0;
        if (sp.dst_offset_bytes + sp.size_bytes <= skip) {
          clipped += sp.size_bytes;
          continue;
        }
        if (sp.dst_offset_bytes < skip) {
          adv = skip - sp.dst_offset_bytes;
          clipped += adv;
        }
        int64_t left = sp.size_bytes - adv, goff = sp.dst_offset_bytes + adv - skip;
        int64_t soff = sp.src_offset_bytes + adv;
        while (left > 0) {
          const int64_t page = goff / dst_live, in_page = goff % dst_live;
          const int64_t take = std::min(left, dst_live - in_page);
          ts_byte_span s{};
          s.src_block_ordinal = sp.src_block_ordinal;
          s.src_offset_bytes = soff;
          s.dst_block_index = page;
          s.dst_offset_bytes = in_page;
          s.size_bytes = take;
          s.count = 1;
          split.push_back(s);
          goff += take;
          soff += take;
          left -= take;
        }
      }
      x.spans = std::move(split);
      x.version = 0;
    }
    if (skip > 0 && skip >= global_end)
      return set_error(TS_INVALID_ARGUMENT, "dst_skip_bytes removes the entire tag " + Q(tag) +
                                                ": skip=" + S(skip) + ", declared_extent=" +
                                                S(global_end) +
                                                "; a full local hit must not reach the planner");
    for (int32_t pi : tp.selected) {
      for (const Decl& x : declared) {
        const int64_t limit = src[size_t(x.unit)][size_t(pi)].num_blocks;
        for (int64_t b : x.block_ids)
          if (b >= limit)
            return set_error(TS_INVALID_ARGUMENT, "Source block id is out of range for pool " +
                                                      S(pi) + " at " + unit_name(x.unit));
      }
      for (int64_t b : ids)
        if (b >= dst[size_t(pi)].num_blocks)
          return set_error(TS_INVALID_ARGUMENT,
                           "Destination block id is out of range for pool " + S(pi));
    }
    // coverage: every destination block covered exactly once, as a prefix
    std::vector<std::vector<std::pair<int64_t, int64_t>>> cov(ids.size());
    int64_t repeats = 0, declared_total = 0, covered_total = 0;
    for (const Decl& x : declared) {
      declared_total += x.declared;
      for (const ts_byte_span& sp : x.spans) {
        if (sp.dst_block_index >= int64_t(ids.size()))
          return set_error(TS_INVALID_ARGUMENT,
                           "Byte span destination index " + S(sp.dst_block_index) +
                               " exceeds the transfer's " + S(int64_t(ids.size())) +
                               " destination blocks for tag " + Q(tag) + " (declared by " +
                               unit_name(x.unit) + ")");
        const int64_t src_end =
            sp.src_offset_bytes + int64_t(sp.count - 1) * sp.src_stride_bytes + sp.size_bytes;
        if (src_end > src_live)
          return set_error(TS_INVALID_ARGUMENT, "Byte span exceeds its source block live bytes: end=" +
                                                    S(src_end) + ", live=" + S(src_live) +
                                                    " (declared by " + unit_name(x.unit) + ")");
        const int64_t dst_end =
            sp.dst_offset_bytes + int64_t(sp.count - 1) * sp.dst_stride_bytes + sp.size_bytes;
        if (dst_end > dst_live)
          return set_error(TS_INVALID_ARGUMENT,
                           "Byte span exceeds its destination block live bytes: end=" + S(dst_end) +
                               ", live=" + S(dst_live) + " (declared by " + unit_name(x.unit) + ")");
        repeats += sp.count;
        if (repeats > kMaxLiveSegments)
          return set_error(TS_INVALID_ARGUMENT, "Byte span plan exceeds the repeat expansion bound");
        for (int32_t r = 0; r < sp.count; ++r) {
          const int64_t start = sp.dst_offset_bytes + int64_t(r) * sp.dst_stride_bytes;
          cov[size_t(sp.dst_block_index)].emplace_back(start, start + sp.size_bytes);
          covered_total += sp.size_bytes;
        }
      }
    }
    std::vector<int64_t> extents;
    for (size_t i = 0; i < ids.size(); ++i) {
      auto& iv = cov[i];
      std::sort(iv.begin(), iv.end());
      if (iv.empty())
        return set_error(TS_INVALID_ARGUMENT, "Destination block index " + S(int64_t(i)) +
                                                  " has no declared coverage for tag " + Q(tag));
      int64_t until = 0;
      for (const auto& [s, e] : iv) {
        if (s != until)
          return set_error(TS_INVALID_ARGUMENT,
                           std::string("Declared byte spans have a destination coverage ") +
                               (s < until ? "overlap" : "gap") + " at byte " +
                               S(std::min(s, until)) + " of destination block index " +
                               S(int64_t(i)));
        until = e;
      }
      if (i != ids.size() - 1 && until != dst_live)
        return set_error(TS_INVALID_ARGUMENT, "Destination block index " + S(int64_t(i)) +
                                                  " is covered to " + S(until) + " of " +
                                                  S(dst_live) +
                                                  " live bytes; only the final block may be partial");
      extents.push_back(until);
    }
    if (declared_total != covered_total + clipped) {
      std::string m = "Declared byte totals disagree with coverage: declared=" + S(declared_total) +
                      ", covered=" + S(covered_total);
      if (clipped != 0) m += ", clipped=" + S(clipped);
      return set_error(TS_INVALID_ARGUMENT, m);
    }
    // emission, ordered by (dst block index, dst offset); stable in
    // declaration order
    struct Ordered {
      const ts_byte_span* sp;
      const Decl* x;
    };
    std::vector<Ordered> ord;
    for (const Decl& x : declared)
      for (const ts_byte_span& sp : x.spans) ord.push_back({&sp, &x});
    std::stable_sort(ord.begin(), ord.end(), [](const Ordered& a, const Ordered& b) {
      return std::tie(a.sp->dst_block_index, a.sp->dst_offset_bytes) <
             std::tie(b.sp->dst_block_index, b.sp->dst_offset_bytes);
    });
    std::map<int64_t, std::set<std::pair<int64_t, int64_t>>> pairs;
    std::vector<ts_live_copy_chunk> chunks;
    for (const Ordered& o : ord) {
      const ts_byte_span& sp = *o.sp;
      if (sp.src_block_ordinal < 0 || sp.src_block_ordinal >= int64_t(o.x->block_ids.size()))
        return set_error(TS_INVALID_ARGUMENT, "Byte span source ordinal " +
                                                  S(sp.src_block_ordinal) + " is out of range (declared by " +
                                                  unit_name(o.x->unit) + ")");
      const int64_t sb = o.x->block_ids[size_t(sp.src_block_ordinal)];
      const int64_t db = ids[size_t(sp.dst_block_index)];
      for (int32_t r = 0; r < sp.count; ++r) {
        int rc = pool::translate_live_copy(
            tp.src_seg.data(), int64_t(tp.src_seg.size()), tp.dst_seg.data(),
            int64_t(tp.dst_seg.size()), sp.src_offset_bytes + int64_t(r) * sp.src_stride_bytes,
            sp.dst_offset_bytes + int64_t(r) * sp.dst_stride_bytes, sp.size_bytes, &chunks);
        if (rc != TS_OK) return rc;
        emitted += int64_t(chunks.size());
        if (emitted > kMaxLiveSegments)
          return set_error(TS_INVALID_ARGUMENT, "Byte-span plan exceeds the live-region expansion bound");
        for (const ts_live_copy_chunk& c : chunks)
          plan->schedules[size_t(o.x->unit)].push_back(
              {sb, db, c.src_physical, c.dst_physical, c.size, int32_t(g)});
      }
      pairs[o.x->unit].insert({sb, db});
    }
    int64_t pushes = 0;
    for (const auto& [u, p] : pairs) pushes += std::min(parallelism, int64_t(p.size()));
    if (pushes <= 0)
      return set_error(TS_INVALID_ARGUMENT,
                       "Pool reshard plan contains no source pushes for tag " + Q(tag));
    Plan::Group grp;
    grp.pools = tp.selected;
    grp.dst_ids = ids;
    grp.expected_pushes = int32_t(pushes);
    grp.extents = extents;
    grp.order_rank = g == 0 ? 0 : 1;
    plan->groups.push_back(std::move(grp));
    union_sel.insert(union_sel.end(), tp.selected.begin(), tp.selected.end());
  }
  if (std::set<int32_t>(union_sel.begin(), union_sel.end()).size() != union_sel.size())
    return set_error(TS_INVALID_ARGUMENT,
                     "Requested tags select overlapping pool indices; tags must partition their pools");
  {
    std::set<int32_t> sel(union_sel.begin(), union_sel.end());
    std::map<std::string, int64_t> skipped;
    for (size_t i = 0; i < dst.size(); ++i)
      if (!sel.count(int32_t(i))) skipped[dst[i].tag] += 1;
    plan->skipped.assign(skipped.begin(), skipped.end());
  }
  for (const auto& [r, u] : ranks)
    if (!plan->schedules[size_t(u)].empty()) plan->active_units.push_back(u);
  plan->transfer_pool_indices = union_sel;
  plan->parallelism = int32_t(parallelism);
  plan->expected_block_count = int64_t(dst_ids.size());
  plan->src_pools = src[0];
  plan->dst_pools = dst;
  return TS_OK;
}

// Tasks are cut to at most kTaskBytes (whole rows when a row fits, else
// 64 KiB column chunks of single rows) so one warp's share stays bounded.
constexpr uint64_t kTaskBytes = 64 * 1024;
constexpr int kThreads = 256;

void push_split(std::vector<RelTask>* out, const RelTask& t) {
  if (t.bytes == 0 || t.count == 0) return;
  if (t.bytes >= kTaskBytes) {
    for (uint32_t r = 0; r < t.count; ++r)
      for (uint64_t o = 0; o < t.bytes; o += kTaskBytes)
        out->push_back({t.src_block, t.src_off + int64_t(r) * t.src_stride + int64_t(o),
                        t.dst_block, t.dst_off + int64_t(r) * t.dst_stride + int64_t(o), 0, 0,
                        uint32_t(std::min<uint64_t>(kTaskBytes, t.bytes - o)), 1});
    return;
  }
  const uint32_t rows = uint32_t(kTaskBytes / t.bytes);
  for (uint32_t r = 0; r < t.count; r += rows) {
    RelTask h = t;
    h.src_off = t.src_off + int64_t(r) * t.src_stride;
    h.dst_off = t.dst_off + int64_t(r) * t.dst_stride;
    h.count = std::min(rows, t.count - r);
    out->push_back(h);
  }
}

// One warp per (pool, task) item; rows and access words flattened across
// the lanes, eight loads in flight per lane before its stores.  A lane walks
// its elements (lane, lane + 32, ...) by keeping its column and byte offset
// and advancing 32 elements with two adds and one wrap test -- no division
// or multiply per element; the store pass repeats the same walk.
template <typename W>
__device__ __forceinline__ void copy_rows(uint64_t src, uint64_t dst, const RelTask& t, int lane) {
  constexpr int64_t kW = int64_t(sizeof(W));
  const uint32_t per_row = t.bytes / uint32_t(kW);
  const uint32_t total = per_row * t.count;
  const uint32_t adv_c = 32u % per_row, adv_r = 32u / per_row;
  const int64_t s_adv = int64_t(adv_r) * t.src_stride + int64_t(adv_c) * kW;
  const int64_t d_adv = int64_t(adv_r) * t.dst_stride + int64_t(adv_c) * kW;
  const int64_t s_wrap = t.src_stride - int64_t(per_row) * kW;
  const int64_t d_wrap = t.dst_stride - int64_t(per_row) * kW;
  uint32_t col0 = uint32_t(lane) % per_row;
  const uint32_t row0 = uint32_t(lane) / per_row;
  int64_t s0 = int64_t(row0) * t.src_stride + int64_t(col0) * kW;
  int64_t d0 = int64_t(row0) * t.dst_stride + int64_t(col0) * kW;
  for (uint32_t base = 0; base < total; base += 256) {
    W v[8];
    uint32_t col = col0;
    int64_t so = s0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (base + uint32_t(lane + 32 * i) < total) v[i] = *reinterpret_cast<const W*>(src + so);
      col += adv_c;
      so += s_adv;
      if (col >= per_row) {
        col -= per_row;
        so += s_wrap;
      }
    }
    col = col0;
    int64_t dof = d0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (base + uint32_t(lane + 32 * i) < total) *reinterpret_cast<W*>(dst + dof) = v[i];
      col += adv_c;
      dof += d_adv;
      if (col >= per_row) {
        col -= per_row;
        dof += d_wrap;
      }
    }
    col0 = col;
    s0 = so;
    d0 = dof;
  }
}

// 16-byte path: 80 registers (3 CTAs per SM); narrower paths fit 4.
template <typename W>
__global__ void __launch_bounds__(kThreads, sizeof(W) == 16 ? 3 : 4)
    pool_reshard_kernel(const RelTask* __restrict__ tasks, int64_t n_tasks,
                        const PoolBase* __restrict__ pools, int64_t n_pools) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (int64_t(gridDim.x) * kThreads) >> 5;
  const int64_t items = n_tasks * n_pools;
  for (int64_t i = warp; i < items; i += nwarps) {
    const int64_t p = i / n_tasks;
    const RelTask t = tasks[i - p * n_tasks];
    const PoolBase pb = pools[p];
    copy_rows<W>(pb.src + uint64_t(t.src_block * pb.src_stride + t.src_off),
                 pb.dst + uint64_t(t.dst_block * pb.dst_stride + t.dst_off), t, lane);
  }
}

// Widest access (16, 4 or 1 bytes) every address of `t` allows in every pool
// of the group.
int task_class(const RelTask& t, uint64_t pool_bits) {
  const uint64_t bits = pool_bits | uint64_t(t.src_off) |
                        uint64_t(t.dst_off) | uint64_t(t.src_stride) | uint64_t(t.dst_stride) |
                        uint64_t(t.bytes);
  return (bits & 15) == 0 ? 16 : (bits & 3) == 0 ? 4 : 1;
}

// ---------------------------------------------------------------------------
// Plans that arrive from a controller: the executor's own checks
// (ValidatePoolReshardPlan + ValidatePoolReshardReceiverCoverage,
// tpu_sync/core/kv_cache_manager_with_transfer.cc:742-1150) against the local
// pool table.  The transport identity checks (req_id, uuid,
// use_block_chunks) belong to the control plane and are not repeated.
// ---------------------------------------------------------------------------

// StridedSpanFitsBlock / StridedSpanFitsRegions (:115-142).
bool span_fits_block(int64_t off, int64_t stride, int64_t size, int64_t count, int64_t block) {
  if (off < 0 || stride < 0 || size <= 0 || count <= 0 || block <= 0 || off > block ||
      size > block - off)
    return false;
  if (count == 1) return true;
  const int64_t remaining = block - off - size;
  return stride <= remaining / (count - 1);
}

bool span_fits_regions(int64_t off, int64_t stride, int64_t size, int64_t count,
                       const pool::Pool& p) {
  if (!span_fits_block(off, stride, size, count, p.block_stride_bytes)) return false;
  for (int64_t r = 0; r < count; ++r) {
    const int64_t start = off + r * stride;
    if (!pool::regions_cover_range(p.regions, uint64_t(start), uint64_t(start + size)))
      return false;
  }
  return true;
}

int receiver_coverage(const ts_received_plan* rp, const std::vector<pool::Pool>& pools) {
  constexpr int64_t kMaxRepeats = int64_t{1} << 20;
  std::set<int64_t> grouped;
  for (int64_t g = 0; g < rp->n_groups; ++g)
    for (int64_t i = 0; i < rp->groups[g].n_pool_indices; ++i) {
      const int32_t pi = rp->groups[g].pool_indices[i];
      if (pi < 0 || !grouped.insert(pi).second)
        return set_error(TS_INVALID_ARGUMENT, "group pool indices must be unique and non-negative");
    }
  bool partition = int64_t(grouped.size()) == rp->n_transfer_pools;
  for (int64_t i = 0; partition && i < rp->n_transfer_pools; ++i)
    partition = grouped.count(rp->transfer_pool_indices[i]) > 0;
  if (!partition)
    return set_error(TS_INVALID_ARGUMENT,
                     "group pool indices do not partition the plan's transfer pools");
  const int64_t par = rp->parallelism;
  if (par <= 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "receiver plans require positive parallelism for push accounting");
  struct State {
    std::vector<ts_live_segment> seg;
    int64_t live = 0;
    std::map<int64_t, size_t> ordinal;
    std::vector<std::vector<std::pair<int64_t, int64_t>>> cov;
    std::map<int32_t, std::set<std::tuple<int32_t, int64_t, int64_t>>> pairs;
  };
  std::vector<State> st(size_t(rp->n_groups));
  for (int64_t g = 0; g < rp->n_groups; ++g) {
    const ts_received_group& grp = rp->groups[g];
    State& s = st[size_t(g)];
    if (grp.n_pool_indices == 0)
      return set_error(TS_INVALID_ARGUMENT, "group " + S(g) + " declares no pools");
    for (int64_t i = 0; i < grp.n_pool_indices; ++i) {
      const int32_t pi = grp.pool_indices[i];
      if (pi >= int32_t(pools.size()))
        return set_error(TS_INVALID_ARGUMENT, "group pool index out of range: " + S(pi));
      std::vector<ts_live_segment> seg;
      int rc = pool::live_segments(pools[size_t(pi)], &seg);
      if (rc != TS_OK) return rc;
      if (s.seg.empty()) {
        s.seg = seg;
      } else if (!same_segments(s.seg, seg)) {
        return set_error(TS_INVALID_ARGUMENT, "group " + S(g) +
                                                  " pools must share one live-region map; pool " +
                                                  S(pi) + " disagrees");
      }
    }
    for (const auto& x : s.seg) s.live += x.size;
    if (s.live <= 0)
      return set_error(TS_INVALID_ARGUMENT, "group " + S(g) + " has no live destination bytes");
    if (grp.n_extents == 0)
      return set_error(TS_INVALID_ARGUMENT, "receiver plans require dst_expected_extent_bytes");
    if (grp.n_extents != grp.n_dst_block_ids)
      return set_error(TS_INVALID_ARGUMENT, "group " + S(g) +
                                                " extents do not match its destination block "
                                                "count: got " + S(grp.n_extents) +
                                                ", expected " + S(grp.n_dst_block_ids));
    for (int64_t o = 0; o < grp.n_extents; ++o) {
      const int64_t e = grp.extents[o];
      if (e <= 0 || e > s.live)
        return set_error(TS_INVALID_ARGUMENT, "extent " + S(e) + " for destination block ordinal " +
                                                  S(o) + " of group " + S(g) +
                                                  " is outside (0, " + S(s.live) + "]");
      if (o != grp.n_extents - 1 && e != s.live)
        return set_error(TS_INVALID_ARGUMENT,
                         "extents must cover every destination block fully except the final one");
    }
    for (int64_t o = 0; o < grp.n_dst_block_ids; ++o) s.ordinal[grp.dst_block_ids[o]] = size_t(o);
    s.cov.resize(size_t(grp.n_dst_block_ids));
  }
  int64_t repeats = 0;
  for (int64_t i = 0; i < rp->n_entries; ++i) {
    const ts_received_entry& e = rp->entries[i];
    if (e.pool_group < 0 || e.pool_group >= rp->n_groups)
      return set_error(TS_INVALID_ARGUMENT,
                       "reshard entry declares an unknown pool group " + S(e.pool_group));
    State& s = st[size_t(e.pool_group)];
    auto it = s.ordinal.find(e.dst_block_id);
    if (it == s.ordinal.end())
      return set_error(TS_INVALID_ARGUMENT, "reshard entry targets destination block " +
                                                S(e.dst_block_id) + " outside its group " +
                                                S(e.pool_group) + " destination set");
    const int64_t extent = rp->groups[e.pool_group].extents[it->second];
    repeats += e.count;
    if (repeats > kMaxRepeats)
      return set_error(TS_INVALID_ARGUMENT, "receiver plan exceeds the repeat expansion bound");
    for (int64_t r = 0; r < e.count; ++r) {
      int64_t a = 0, b = 0;
      if (pool::physical_to_logical(s.seg.data(), int64_t(s.seg.size()),
                                    e.dst_offset_bytes + r * e.dst_stride_bytes, e.size_bytes, &a,
                                    &b) != TS_OK)
        return set_error(TS_INVALID_ARGUMENT, "reshard entry for destination block " +
                                                  S(e.dst_block_id) +
                                                  " crosses padding or lies outside declared live "
                                                  "regions: " + ts_last_error());
      if (b > extent)
        return set_error(TS_INVALID_ARGUMENT, "reshard entry exceeds destination block " +
                                                  S(e.dst_block_id) + " declared live tail: end=" +
                                                  S(b) + " extent=" + S(extent));
      s.cov[it->second].emplace_back(a, b);
    }
    s.pairs[e.source_rank].insert({e.dst_peer, e.src_block_id, e.dst_block_id});
  }
  for (int64_t g = 0; g < rp->n_groups; ++g) {
    State& s = st[size_t(g)];
    const ts_received_group& grp = rp->groups[g];
    int64_t pushes = 0;
    for (const auto& [rank, pr] : s.pairs) pushes += std::min(par, int64_t(pr.size()));
    if (pushes != grp.expected_pushes)
      return set_error(TS_INVALID_ARGUMENT, "expected pushes for group " + S(g) +
                                                " do not match the received schedules: declared=" +
                                                S(grp.expected_pushes) +
                                                " recomputed=" + S(pushes));
    for (int64_t o = 0; o < grp.n_dst_block_ids; ++o) {
      auto& iv = s.cov[size_t(o)];
      std::sort(iv.begin(), iv.end());
      int64_t until = 0;
      for (const auto& [a, b] : iv) {
        if (a != until)
          return set_error(TS_INVALID_ARGUMENT,
                           std::string("receiver schedule has a destination coverage ") +
                               (a < until ? "overlap" : "gap") + " for block " +
                               S(grp.dst_block_ids[o]) + " at byte " + S(a));
        until = b;
      }
      if (until != grp.extents[o])
        return set_error(TS_INVALID_ARGUMENT,
                         "receiver schedule does not cover the exact live bytes for destination "
                         "block " + S(grp.dst_block_ids[o]) + ": covered=" + S(until) +
                             " expected=" + S(grp.extents[o]));
    }
  }
  return TS_OK;
}

int validate_received(const ts_received_plan* rp, const std::vector<pool::Pool>& pools,
                      int64_t num_shards, const int64_t* local_ids, int64_t n_local,
                      bool is_sender) {
  if (rp->n_transfer_pools <= 0)
    return set_error(TS_INVALID_ARGUMENT, "reshard plan must declare transfer_pool_indices");
  if (rp->n_groups <= 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "reshard plans must declare pool_groups (a plan is a list of groups; entries "
                     "name their group)");
  for (int64_t g = 0; g < rp->n_groups; ++g)
    if (rp->groups[g].expected_pushes <= 0)
      return set_error(TS_INVALID_ARGUMENT, "every pool group must expect a positive push count");
  if (rp->n_pool_dtype_tags != int64_t(pools.size()))
    return set_error(TS_INVALID_ARGUMENT, "reshard plan must declare one dtype tag per pool: plan=" +
                                              S(rp->n_pool_dtype_tags) +
                                              " local=" + S(int64_t(pools.size())));
  if (n_local <= 0) return set_error(TS_INVALID_ARGUMENT, "local block ids must not be empty");
  std::set<int64_t> local(local_ids, local_ids + n_local);
  for (int64_t i = 0; i < n_local; ++i)
    if (local_ids[i] < 0 || local_ids[i] > INT32_MAX)
      return set_error(TS_INVALID_ARGUMENT, "local block ids must be non-negative and fit in int");
  if (!is_sender) {
    int64_t cur = 0;
    for (int64_t g = 0; g < rp->n_groups; ++g) {
      std::set<int64_t> ids;
      for (int64_t i = 0; i < rp->groups[g].n_dst_block_ids; ++i) {
        const int64_t b = rp->groups[g].dst_block_ids[i];
        if (!ids.insert(b).second)
          return set_error(TS_INVALID_ARGUMENT, "group destination block ids must be unique");
        if (cur >= n_local || local_ids[cur] != b)
          return set_error(TS_INVALID_ARGUMENT,
                           "pool group block ids must concatenate to the plan's local block ids");
        ++cur;
      }
    }
    if (cur != n_local)
      return set_error(TS_INVALID_ARGUMENT,
                       "pool group block ids must cover the plan's local block ids");
  }
  std::set<int32_t> declared;
  for (int64_t i = 0; i < rp->n_transfer_pools; ++i) {
    const int32_t pi = rp->transfer_pool_indices[i];
    if (pi < 0) return set_error(TS_INVALID_ARGUMENT, "transfer pool index must be non-negative");
    if (!declared.insert(pi).second)
      return set_error(TS_INVALID_ARGUMENT, "duplicate transfer pool index " + S(pi));
    if (pi >= int32_t(pools.size()))
      return set_error(TS_INVALID_ARGUMENT, "transfer pool index out of range: " + S(pi));
    const pool::Pool& p = pools[size_t(pi)];
    const char* tag = rp->pool_dtype_tags[pi] ? rp->pool_dtype_tags[pi] : "";
    if (p.dtype_tag != tag)
      return set_error(TS_INVALID_ARGUMENT, "plan dtype tag mismatch for pool " + S(pi) + " (" +
                                                p.tag + "): plan=" + tag + " local=" + p.dtype_tag);
    for (int64_t b : local)
      if (b >= p.num_blocks)
        return set_error(TS_INVALID_ARGUMENT, "local block id " + S(b) +
                                                  " is out of range for pool " + S(pi));
  }
  if (rp->n_schedules <= 0)
    return set_error(TS_INVALID_ARGUMENT, "reshard plan must contain shard push schedules");
  std::set<int64_t> zero_start;
  for (int64_t i = 0; i < rp->n_entries; ++i) {
    const ts_received_entry& e = rp->entries[i];
    if (e.source_rank < 0)
      return set_error(TS_INVALID_ARGUMENT, "reshard schedule source rank must be non-negative");
    if (e.dst_peer < 0) return set_error(TS_INVALID_ARGUMENT, "reshard entry dst_peer must be non-empty");
    if (e.src_block_id < 0 || e.src_block_id > INT32_MAX || e.dst_block_id < 0 ||
        e.dst_block_id > INT32_MAX || e.dst_shard_idx < 0 || e.src_offset_bytes < 0 ||
        e.dst_offset_bytes < 0 || e.size_bytes <= 0 || e.src_stride_bytes < 0 ||
        e.dst_stride_bytes < 0 || e.count <= 0 || e.count > (1 << 20))
      return set_error(TS_INVALID_ARGUMENT,
                       "reshard entry contains invalid ids, offsets, sizes, or strides");
    if (e.count > 1 && (e.src_stride_bytes == 0 || e.dst_stride_bytes == 0))
      return set_error(TS_INVALID_ARGUMENT, "multi-chunk reshard entries require positive strides");
    if (!is_sender && e.dst_shard_idx >= num_shards)
      return set_error(TS_INVALID_ARGUMENT, "destination shard index " + S(e.dst_shard_idx) +
                                                " is out of range: receiver has " + S(num_shards) +
                                                " shards");
    const int64_t id = is_sender ? e.src_block_id : e.dst_block_id;
    if (!local.count(id))
      return set_error(TS_INVALID_ARGUMENT, std::string(is_sender ? "source" : "destination") +
                                                " block id " + S(id) +
                                                " is absent from the local block-id list");
    const int64_t off = is_sender ? e.src_offset_bytes : e.dst_offset_bytes;
    const int64_t stride = is_sender ? e.src_stride_bytes : e.dst_stride_bytes;
    if (!is_sender && e.dst_offset_bytes == 0) zero_start.insert(e.dst_block_id);
    if (e.pool_group < 0 || e.pool_group >= rp->n_groups)
      return set_error(TS_INVALID_ARGUMENT,
                       "reshard entry declares an unknown pool group " + S(e.pool_group));
    const ts_received_group& grp = rp->groups[e.pool_group];
    for (int64_t k = 0; k < grp.n_pool_indices; ++k) {
      const int32_t pi = grp.pool_indices[k];
      if (pi < 0 || pi >= int32_t(pools.size()))
        return set_error(TS_INVALID_ARGUMENT, "group pool index out of range: " + S(pi));
      const pool::Pool& p = pools[size_t(pi)];
      if (!span_fits_regions(off, stride, e.size_bytes, e.count, p))
        return set_error(TS_INVALID_ARGUMENT,
                         std::string(is_sender ? "source" : "destination") +
                             " span exceeds declared pool " + S(pi) + " live regions in block " +
                             S(id) + ": offset=" + S(off) + " stride=" + S(stride) +
                             " size=" + S(e.size_bytes) + " count=" + S(e.count) +
                             " block_stride_bytes=" + S(p.block_stride_bytes));
    }
  }
  if (rp->n_entries == 0) return set_error(TS_INVALID_ARGUMENT, "reshard plan contains no entries");
  if (!is_sender) {
    for (int64_t b : local)
      if (!zero_start.count(b))
        return set_error(TS_INVALID_ARGUMENT,
                         "destination block " + S(b) +
                             " has no transfer entry starting at offset 0; partial-page "
                             "destination preservation is not implemented");
    return receiver_coverage(rp, pools);
  }
  return TS_OK;
}

int pools_from_c(const ts_pool_spec* c, int64_t n, std::vector<pool::Pool>* out) {
  out->clear();
  for (int64_t i = 0; i < n; ++i) {
    pool::Pool p;
    int rc = pool::from_c(&c[i], &p);
    if (rc != TS_OK) return rc;
    out->push_back(std::move(p));
  }
  return TS_OK;
}

}  // namespace
}  // namespace tsb

using tsb::set_error;

extern "C" int ts_pool_reshard_plan_build(const ts_pool_reshard_request* request,
                                          ts_pool_reshard_plan** out) {
  tsb::clear_error();
  if (!request || !out) return set_error(TS_INVALID_ARGUMENT, "null request or output");
  *out = nullptr;
  auto* plan = new ts_pool_reshard_plan();
  int rc = tsb::build(request, plan);
  if (rc != TS_OK) {
    delete plan;
    return rc;
  }
  *out = plan;
  return TS_OK;
}

extern "C" void ts_pool_reshard_plan_destroy(ts_pool_reshard_plan* plan) { delete plan; }

extern "C" int ts_pool_reshard_plan_info(const ts_pool_reshard_plan* plan, int64_t* info) {
  tsb::clear_error();
  if (!plan || !info) return set_error(TS_INVALID_ARGUMENT, "null plan or output");
  info[0] = int64_t(plan->groups.size());
  info[1] = int64_t(plan->active_units.size());
  info[2] = plan->expected_block_count;
  info[3] = plan->parallelism;
  info[4] = plan->groups.empty() ? 0 : plan->groups[0].expected_pushes;
  info[5] = int64_t(plan->transfer_pool_indices.size());
  int64_t n = 0;
  for (const auto& s : plan->schedules) n += int64_t(s.size());
  info[6] = n;
  info[7] = plan->n_src_units;
  return TS_OK;
}

extern "C" int ts_pool_reshard_plan_entries(const ts_pool_reshard_plan* plan, int64_t src_unit,
                                            ts_schedule_entry* out, int64_t cap, int64_t* n_out) {
  tsb::clear_error();
  if (!plan || !n_out) return set_error(TS_INVALID_ARGUMENT, "null plan or output");
  if (src_unit < 0 || src_unit >= plan->n_src_units)
    return set_error(TS_OUT_OF_RANGE, "source unit out of range");
  const auto& v = plan->schedules[size_t(src_unit)];
  *n_out = int64_t(v.size());
  if (!out || cap < int64_t(v.size()))
    return v.empty() ? TS_OK : set_error(TS_RESOURCE_EXHAUSTED, "entry capacity too small");
  for (size_t i = 0; i < v.size(); ++i)
    out[i] = {v[i].src_block, v[i].dst_block, v[i].src_off, v[i].dst_off, v[i].size, v[i].group, 0};
  return TS_OK;
}

extern "C" int ts_pool_reshard_plan_units(const ts_pool_reshard_plan* plan, int64_t* units,
                                          int32_t* pool_indices) {
  tsb::clear_error();
  if (!plan) return set_error(TS_INVALID_ARGUMENT, "null plan");
  if (units)
    for (size_t i = 0; i < plan->active_units.size(); ++i) units[i] = plan->active_units[i];
  if (pool_indices)
    for (size_t i = 0; i < plan->transfer_pool_indices.size(); ++i)
      pool_indices[i] = plan->transfer_pool_indices[i];
  return TS_OK;
}

extern "C" int ts_pool_reshard_plan_group(const ts_pool_reshard_plan* plan, int64_t group,
                                          int64_t* sizes, int32_t* pool_indices,
                                          int64_t* dst_ids, int64_t* extents) {
  tsb::clear_error();
  if (!plan || !sizes) return set_error(TS_INVALID_ARGUMENT, "null plan or output");
  if (group < 0 || group >= int64_t(plan->groups.size()))
    return set_error(TS_OUT_OF_RANGE, "pool group out of range");
  const auto& g = plan->groups[size_t(group)];
  sizes[0] = int64_t(g.pools.size());
  sizes[1] = int64_t(g.dst_ids.size());
  sizes[2] = g.expected_pushes;
  sizes[3] = g.order_rank;
  if (pool_indices) std::copy(g.pools.begin(), g.pools.end(), pool_indices);
  if (dst_ids) std::copy(g.dst_ids.begin(), g.dst_ids.end(), dst_ids);
  if (extents) std::copy(g.extents.begin(), g.extents.end(), extents);
  return TS_OK;
}

extern "C" int ts_pool_reshard_validate(const ts_received_plan* plan,
                                        const ts_pool_spec* local_pools, int64_t n_local_pools,
                                        int64_t num_shards, const int64_t* local_block_ids,
                                        int64_t n_local_block_ids, int is_sender) {
  tsb::clear_error();
  if (!plan || (n_local_pools > 0 && !local_pools) ||
      (n_local_block_ids > 0 && !local_block_ids))
    return set_error(TS_INVALID_ARGUMENT, "null plan, pools or block ids");
  std::vector<tsb::pool::Pool> pools;
  int rc = tsb::pools_from_c(local_pools, n_local_pools, &pools);
  if (rc != TS_OK) return rc;
  return tsb::validate_received(plan, pools, num_shards, local_block_ids, n_local_block_ids,
                                is_sender != 0);
}

extern "C" int ts_pool_reshard_plan_from_received(
    const ts_received_plan* plan, const ts_pool_spec* src_pools, const ts_pool_spec* dst_pools,
    int64_t n_pools, const int64_t* src_block_ids, int64_t n_src_block_ids,
    const int64_t* dst_block_ids, int64_t n_dst_block_ids, int64_t dst_num_shards,
    ts_pool_reshard_plan** out) {
  tsb::clear_error();
  if (!plan || !out || (n_pools > 0 && (!src_pools || !dst_pools)))
    return set_error(TS_INVALID_ARGUMENT, "null plan, pools or output");
  *out = nullptr;
  std::vector<tsb::pool::Pool> sp, dp;
  int rc = tsb::pools_from_c(src_pools, n_pools, &sp);
  if (rc == TS_OK) rc = tsb::pools_from_c(dst_pools, n_pools, &dp);
  if (rc != TS_OK) return rc;
  // both ends' checks: every source span inside the sender's pool regions,
  // every destination span inside the receiver's and exactly covered
  rc = tsb::validate_received(plan, sp, 1, src_block_ids, n_src_block_ids, true);
  if (rc != TS_OK) return set_error(rc, std::string("sender: ") + ts_last_error());
  rc = tsb::validate_received(plan, dp, dst_num_shards, dst_block_ids, n_dst_block_ids, false);
  if (rc != TS_OK) return set_error(rc, std::string("receiver: ") + ts_last_error());
  auto* p = new ts_pool_reshard_plan();
  int64_t max_rank = 0;
  for (int64_t i = 0; i < plan->n_entries; ++i)
    max_rank = std::max<int64_t>(max_rank, plan->entries[i].source_rank);
  p->n_src_units = max_rank + 1;
  p->schedules.assign(size_t(p->n_src_units), {});
  for (int64_t i = 0; i < plan->n_entries; ++i) {
    const ts_received_entry& e = plan->entries[i];
    ts_pool_reshard_plan::Entry x{e.src_block_id, e.dst_block_id, e.src_offset_bytes,
                                  e.dst_offset_bytes, e.size_bytes, e.pool_group};
    x.src_stride = e.src_stride_bytes;
    x.dst_stride = e.dst_stride_bytes;
    x.count = e.count;
    p->schedules[size_t(e.source_rank)].push_back(x);
  }
  for (int64_t g = 0; g < plan->n_groups; ++g) {
    const ts_received_group& rg = plan->groups[g];
    ts_pool_reshard_plan::Group grp;
    grp.pools.assign(rg.pool_indices, rg.pool_indices + rg.n_pool_indices);
    grp.dst_ids.assign(rg.dst_block_ids, rg.dst_block_ids + rg.n_dst_block_ids);
    grp.extents.assign(rg.extents, rg.extents + rg.n_extents);
    grp.expected_pushes = rg.expected_pushes;
    grp.order_rank = rg.order_rank;
    p->groups.push_back(std::move(grp));
  }
  for (int64_t u = 0; u < p->n_src_units; ++u)
    if (!p->schedules[size_t(u)].empty()) p->active_units.push_back(u);
  p->transfer_pool_indices.assign(plan->transfer_pool_indices,
                                  plan->transfer_pool_indices + plan->n_transfer_pools);
  p->parallelism = plan->parallelism;
  p->expected_block_count = n_dst_block_ids;
  p->src_pools = std::move(sp);
  p->dst_pools = std::move(dp);
  *out = p;
  return TS_OK;
}

extern "C" int ts_pool_reshard_program_create(const ts_pool_reshard_plan* plan, int64_t src_unit,
                                              int device, const uint64_t* src_storage_ptrs,
                                              const uint64_t* dst_storage_ptrs,
                                              const uint64_t* src_storage_bytes,
                                              const uint64_t* dst_storage_bytes,
                                              int64_t n_storages,
                                              ts_pool_reshard_program** out) {
  tsb::clear_error();
  if (!plan || !out || !src_storage_ptrs || !dst_storage_ptrs || !src_storage_bytes ||
      !dst_storage_bytes)
    return set_error(TS_INVALID_ARGUMENT, "null plan, storages or output");
  *out = nullptr;
  if (src_unit < 0 || src_unit >= plan->n_src_units)
    return set_error(TS_OUT_OF_RANGE, "source unit out of range");
  for (int32_t pi : plan->transfer_pool_indices) {
    const tsb::pool::Pool& sp = plan->src_pools[size_t(pi)];
    const tsb::pool::Pool& dp = plan->dst_pools[size_t(pi)];
    if (sp.storage_index >= n_storages || dp.storage_index >= n_storages)
      return set_error(TS_OUT_OF_RANGE, "pool storage_index beyond the given storages");
    if (sp.validate(int64_t(src_storage_bytes[sp.storage_index])) != TS_OK)
      return set_error(TS_OUT_OF_RANGE, "source " + std::string(ts_last_error()));
    if (dp.validate(int64_t(dst_storage_bytes[dp.storage_index])) != TS_OK)
      return set_error(TS_OUT_OF_RANGE, "destination " + std::string(ts_last_error()));
  }
  auto* prog = new ts_pool_reshard_program();
  prog->device = device;
  auto fail = [&](int rc) {
    for (auto& g : prog->groups) {
      if (g.d_tasks) cudaFree(g.d_tasks);
      if (g.d_pools) cudaFree(g.d_pools);
    }
    delete prog;
    return rc;
  };
  tsb::DeviceGuard guard(device);
  const auto& entries = plan->schedules[size_t(src_unit)];
  for (size_t gi = 0; gi < plan->groups.size(); ++gi) {
    // This unit's entries of the group.  Their destination bytes are
    // disjoint (exactly-once coverage), so they may run in any order: sort by
    // (src block, dst block, src offset) and merge rows that repeat with
    // constant source and destination deltas into strided tasks.
    std::vector<const ts_pool_reshard_plan::Entry*> es;
    for (const auto& e : entries)
      if (e.group == int32_t(gi)) es.push_back(&e);
    if (es.empty()) continue;
    std::stable_sort(es.begin(), es.end(), [](const auto* a, const auto* b) {
      return std::tie(a->src_block, a->dst_block, a->src_off) <
             std::tie(b->src_block, b->dst_block, b->src_off);
    });
    std::vector<tsb::RelTask> merged;
    uint64_t group_bytes = 0;
    for (const auto* e : es) {
      group_bytes += uint64_t(e->size) * uint64_t(e->count);
      if (e->count > 1) {  // a received entry with its own repeats
        for (int64_t o = 0; o < e->size; o += int64_t(1) << 30)
          merged.push_back({e->src_block, e->src_off + o, e->dst_block, e->dst_off + o,
                            e->src_stride, e->dst_stride,
                            uint32_t(std::min<int64_t>(e->size - o, int64_t(1) << 30)),
                            uint32_t(e->count)});
        continue;
      }
      for (int64_t o = 0; o < e->size; o += int64_t(1) << 30) {
        const uint32_t n = uint32_t(std::min<int64_t>(e->size - o, int64_t(1) << 30));
        tsb::RelTask t{e->src_block, e->src_off + o, e->dst_block, e->dst_off + o, 0, 0, n, 1};
        if (!merged.empty()) {
          tsb::RelTask& b = merged.back();
          if (b.src_block == t.src_block && b.dst_block == t.dst_block && b.bytes == n &&
              b.count < UINT32_MAX) {
            if (b.count == 1) {
              b.src_stride = t.src_off - b.src_off;
              b.dst_stride = t.dst_off - b.dst_off;
              b.count = 2;
              continue;
            }
            if (t.src_off == b.src_off + int64_t(b.count) * b.src_stride &&
                t.dst_off == b.dst_off + int64_t(b.count) * b.dst_stride) {
              ++b.count;
              continue;
            }
          }
        }
        merged.push_back(t);
      }
    }
    std::vector<tsb::RelTask> tasks;
    for (const tsb::RelTask& t : merged) tsb::push_split(&tasks, t);
    std::vector<tsb::PoolBase> bases;
    for (int32_t pi : plan->groups[gi].pools) {
      const tsb::pool::Pool& sp = plan->src_pools[size_t(pi)];
      const tsb::pool::Pool& dp = plan->dst_pools[size_t(pi)];
      bases.push_back({src_storage_ptrs[sp.storage_index] + uint64_t(sp.base_offset_bytes),
                       dst_storage_ptrs[dp.storage_index] + uint64_t(dp.base_offset_bytes),
                       sp.block_stride_bytes, dp.block_stride_bytes});
    }
    // Block-0 addresses and block strides of every pool enter each task's
    // addresses, so they bound the access width of all of the group's tasks.
    uint64_t pool_bits = 0;
    for (const tsb::PoolBase& pb : bases)
      pool_bits |= pb.src | pb.dst | uint64_t(pb.src_stride) | uint64_t(pb.dst_stride);
    std::stable_sort(tasks.begin(), tasks.end(), [&](const tsb::RelTask& a, const tsb::RelTask& b) {
      return tsb::task_class(a, pool_bits) > tsb::task_class(b, pool_bits);
    });
    ts_pool_reshard_program::Group g;
    g.n_tasks = int64_t(tasks.size());
    g.n_pools = int64_t(bases.size());
    for (const tsb::RelTask& t : tasks) {
      const int c = tsb::task_class(t, pool_bits);
      g.n16 += c == 16;
      g.n4 += c == 4;
    }
    cudaError_t e = cudaMalloc(&g.d_tasks, sizeof(tsb::RelTask) * tasks.size());
    if (e == cudaSuccess) e = cudaMalloc(&g.d_pools, sizeof(tsb::PoolBase) * bases.size());
    if (e == cudaSuccess)
      e = cudaMemcpy(g.d_tasks, tasks.data(), sizeof(tsb::RelTask) * tasks.size(),
                     cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
      e = cudaMemcpy(g.d_pools, bases.data(), sizeof(tsb::PoolBase) * bases.size(),
                     cudaMemcpyHostToDevice);
    prog->groups.push_back(g);
    if (e != cudaSuccess) return fail(tsb::cuda_error(e, "pool reshard task table"));
    prog->n_tasks += g.n_tasks * g.n_pools;
    prog->bytes += group_bytes * uint64_t(bases.size());
  }
  *out = prog;
  return TS_OK;
}

extern "C" int ts_pool_reshard_program_info(const ts_pool_reshard_program* prog, int64_t* n_tasks,
                                            uint64_t* bytes) {
  tsb::clear_error();
  if (!prog) return set_error(TS_INVALID_ARGUMENT, "null program");
  if (n_tasks) *n_tasks = prog->n_tasks;
  if (bytes) *bytes = prog->bytes;
  return TS_OK;
}

extern "C" int ts_pool_reshard_program_launch(ts_pool_reshard_program* prog, void* stream,
                                              int max_ctas) {
  tsb::clear_error();
  if (!prog) return set_error(TS_INVALID_ARGUMENT, "null program");
  tsb::DeviceGuard g(prog->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int cap = tsb::sm_count(prog->device) * 3;
  if (max_ctas > 0) cap = std::min(cap, max_ctas);
  for (const auto& grp : prog->groups) {
    const int64_t n1 = grp.n_tasks - grp.n16 - grp.n4;
    const tsb::RelTask* part[3] = {grp.d_tasks, grp.d_tasks + grp.n16,
                                   grp.d_tasks + grp.n16 + grp.n4};
    const int64_t count[3] = {grp.n16, grp.n4, n1};
    for (int c = 0; c < 3; ++c) {
      const int64_t items = count[c] * grp.n_pools;
      if (items == 0) continue;
      const int64_t want = (items + (tsb::kThreads / 32) - 1) / (tsb::kThreads / 32);
      const int ctas = int(std::max<int64_t>(1, std::min<int64_t>(want, cap)));
      if (c == 0)
        tsb::pool_reshard_kernel<int4><<<ctas, tsb::kThreads, 0, s>>>(part[c], count[c],
                                                                       grp.d_pools, grp.n_pools);
      else if (c == 1)
        tsb::pool_reshard_kernel<uint32_t><<<ctas, tsb::kThreads, 0, s>>>(
            part[c], count[c], grp.d_pools, grp.n_pools);
      else
        tsb::pool_reshard_kernel<uint8_t><<<ctas, tsb::kThreads, 0, s>>>(
            part[c], count[c], grp.d_pools, grp.n_pools);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return tsb::cuda_error(e, "pool reshard launch");
    }
  }
  return TS_OK;
}

extern "C" void ts_pool_reshard_program_destroy(ts_pool_reshard_program* prog) {
  if (!prog) return;
  tsb::DeviceGuard g(prog->device);
  for (auto& grp : prog->groups) {
    if (grp.d_tasks) cudaFree(grp.d_tasks);
    if (grp.d_pools) cudaFree(grp.d_pools);
  }
  delete prog;
}

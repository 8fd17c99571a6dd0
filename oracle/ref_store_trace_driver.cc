// Replays a block-access trace through the REFERENCE's own LRUCache
// (tpu_sync/kv_cache/lru_cache.h) and LogicalBlockManager
// (tpu_sync/kv_cache/logical_block_manager.cc), composed the way
// KVCacheStore's local paths compose them.  Compiled from the reference
// checkout by oracle/build_ref.py into oracle/_ref/store_trace_ref.  TEST AND
// BASELINE INFRASTRUCTURE ONLY: it decides which blocks the C1 benchmark's
// CPU reference arm offloads and reloads, independently of the product, and
// tests compare the product store's decisions with its answers.
//
// The store operations are restated over the reference's index and allocator
// (the store, backend and controller classes need gRPC / PJRT and do not
// compile here):
//   Lookup        HostOffloadBackend::Lookup, local index, one sweep that
//                 pins each hit, answer cut at the first miss, later pins
//                 handed back (host_offload_backend.cc:154-288);
//   InsertAndLock all-or-nothing insert + pin (host_offload_backend.cc:370-470);
//   SaveLocal     lookup without pins, HBM / pinned checks, AllocateBlockIds,
//                 one pending save (kv_cache_store.cc:977-1058);
//   AllocateBlockIds  evict unpinned host-resident entries (candidates first,
//                 then the LRU end) to cover the shortfall, then
//                 Allocate(n, lock = true) (kv_cache_store.cc:1743-1781,
//                 :1553-1570, host_offload_backend.cc:656-688,
//                 core/controller/raiden_controller.cc:458-462);
//   Load          lookup without pins, pinned / on-host checks, one pending
//                 load (kv_cache_store.cc:1060-1137);
//   Poll*         a finished save sets host id + HOST_AND_HBM and releases
//                 its pin; a finished load sets device id + HOST_AND_HBM and
//                 releases (kv_cache_store.cc:2113-2254); Release unpins in
//                 reverse order (host_offload_backend.cc:529-536).
// Transfers complete at once (a host-only store); completions are processed
// at the explicit poll calls (the background poller is not modelled).
//
// Usage: store_trace_ref CAPACITY HOST_BLOCKS DEVICE_BLOCKS BATCH < trace
// where the trace is whitespace-separated int64 prefix ids.  A hash is the
// id's 8 little-endian bytes.  Output, per access batch:
//   "B <n_saves> <n_loads>" then one line "S dev host" per save and one line
//   "L host dev" per load; then "H <hits> <misses>" at the end.
#include <cstdint>
#include <cstring>
#include <iostream>
#include <string>
#include <unordered_set>
#include <vector>

#include "tpu_sync/kv_cache/logical_block_manager.h"
#include "tpu_sync/kv_cache/lru_cache.h"

namespace {

enum Status { kInit = 0, kHbm = 1, kHost = 2, kHostAndHbm = 3 };

struct Blk {
  int host_block_id = -1;
  int device_block_id = -1;
  int status = kInit;
};

struct Pending {
  std::vector<std::string> hashes;
  std::vector<int> ids;  // host ids (saves) / device ids (loads)
};

struct Store {
  tpu_raiden::kv_cache::LRUCache<std::string, Blk> lru;
  tpu_raiden::kv_cache::LogicalBlockManager bm;
  std::vector<Pending> saves, loads;
  std::unordered_set<std::string> saving, loading;

  Store(size_t capacity, int host_blocks) : lru(capacity), bm(host_blocks) {}

  std::vector<Blk> Lookup(const std::vector<std::string>& h, bool pin_found) {
    std::vector<bool> hit(h.size(), false);
    for (size_t i = 0; i < h.size(); ++i) {
      // interleaved lookup (the default): every hash is swept and pinned
      if (lru.Peek(h[i]) != nullptr) {
        if (pin_found) lru.Pin(h[i]);
        hit[i] = true;
      }
    }
    std::vector<Blk> out;
    for (size_t i = 0; i < h.size() && hit[i]; ++i) {
      const Blk* b = lru.Peek(h[i]);
      if (b == nullptr) break;
      out.push_back(*b);
    }
    if (pin_found)
      for (size_t i = out.size(); i < h.size(); ++i)
        if (hit[i]) lru.Unpin(h[i]);
    return out;
  }

  void Release(const std::vector<std::string>& h) {
    for (auto it = h.rbegin(); it != h.rend(); ++it) lru.Unpin(*it);
  }

  bool InsertAndLock(const std::vector<std::string>& h, const std::vector<Blk>& slices) {
    std::vector<size_t> existing, fresh;
    for (size_t i = 0; i < h.size(); ++i) (lru.Contains(h[i]) ? existing : fresh).push_back(i);
    for (size_t e = 0; e < existing.size(); ++e) {
      const size_t i = existing[e];
      if (!lru.Pin(h[i])) {
        for (size_t j = 0; j < e; ++j) lru.Unpin(h[existing[j]]);
        return false;
      }
      if (i < slices.size()) {
        Blk* b = lru.PeekMutable(h[i]);
        if (b != nullptr && b->status == kHbm) *b = slices[i];
      }
    }
    if (lru.available_space() < fresh.size()) {
      for (size_t i : existing) lru.Unpin(h[i]);
      return false;
    }
    for (auto it = fresh.rbegin(); it != fresh.rend(); ++it)
      lru.Put(h[*it], *it < slices.size() ? slices[*it] : Blk());
    for (size_t f = 0; f < fresh.size(); ++f) {
      if (!lru.Pin(h[fresh[f]])) {
        for (size_t j = 0; j < f; ++j) lru.Unpin(h[fresh[j]]);
        for (size_t j : existing) lru.Unpin(h[j]);
        for (size_t j : fresh) lru.Erase(h[j]);
        return false;
      }
    }
    return true;
  }

  size_t Evict(const std::vector<std::string>& keys) {
    std::vector<int> ids;
    for (const std::string& k : keys) {
      const Blk* b = lru.PeekIncludingCandidates(k);
      if (b != nullptr && lru.GetPinCount(k) == 0 &&
          (b->status == kHost || b->status == kHostAndHbm)) {
        ids.push_back(b->host_block_id);
        lru.Erase(k);
      }
    }
    if (!ids.empty()) (void)bm.Deallocate(absl::Span<const int>(ids.data(), ids.size()));
    return ids.size();
  }

  bool AllocateBlockIds(int needed, std::vector<int>* out) {
    const int to_free = needed - bm.num_free_blocks();
    if (to_free > 0) {
      std::vector<std::string> keys = lru.GetEvictableKeys(size_t(to_free));
      if (keys.size() < size_t(to_free)) return false;
      Evict(keys);
    }
    auto r = bm.Allocate(needed, /*lock=*/true);
    if (!r.ok()) return false;
    *out = *r;
    return true;
  }

  bool SaveLocal(const std::vector<std::string>& h) {
    const std::vector<Blk> found = Lookup(h, false);
    if (found.size() < h.size()) return false;
    for (size_t i = 0; i < h.size(); ++i) {
      if (found[i].status != kHbm || found[i].device_block_id == -1 ||
          lru.GetPinCount(h[i]) <= 0 || saving.count(h[i]))
        return false;
    }
    for (const std::string& x : h) saving.insert(x);
    std::vector<int> host_ids;
    if (!AllocateBlockIds(int(h.size()), &host_ids)) {
      for (const std::string& x : h) saving.erase(x);
      return false;
    }
    saves.push_back(Pending{h, host_ids});
    return true;
  }

  bool Load(const std::vector<std::string>& h, const std::vector<int>& dev) {
    if (h.size() != dev.size()) return false;
    if (h.empty()) return true;
    const std::vector<Blk> found = Lookup(h, false);
    if (found.size() < h.size()) return false;
    for (size_t i = 0; i < h.size(); ++i) {
      if (lru.GetPinCount(h[i]) <= 0 || loading.count(h[i])) return false;
      if (found[i].status != kHost && found[i].status != kHostAndHbm) return false;
      if (found[i].host_block_id == -1) return false;
    }
    for (const std::string& x : h) loading.insert(x);
    loads.push_back(Pending{h, dev});
    return true;
  }

  // PollSavesInternal / PollLoadsInternal for the (already finished)
  // transfers: the index update goes through Insert, which for a present
  // entry overwrites its value in place (host_offload_backend.cc:300-316).
  void Poll(bool save_side) {
    std::vector<Pending>& ops = save_side ? saves : loads;
    for (Pending& op : ops) {
      const std::vector<Blk> found = Lookup(op.hashes, false);
      std::vector<std::string> updated;
      for (size_t i = 0; i < op.hashes.size() && i < found.size(); ++i) {
        Blk* b = lru.PeekMutable(op.hashes[i]);
        if (b == nullptr) continue;
        if (save_side) b->host_block_id = op.ids[i];
        else b->device_block_id = op.ids[i];
        b->status = kHostAndHbm;
        updated.push_back(op.hashes[i]);
      }
      Release(updated);
      for (const std::string& x : op.hashes) (save_side ? saving : loading).erase(x);
    }
    ops.clear();
  }
};

std::string key_of(int64_t x) {
  std::string k(8, '\0');
  for (int i = 0; i < 8; ++i) k[size_t(i)] = char((uint64_t(x) >> (8 * i)) & 0xff);
  return k;
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 5) {
    std::cerr << "usage: store_trace_ref CAPACITY HOST_BLOCKS DEVICE_BLOCKS BATCH < trace\n";
    return 2;
  }
  const size_t capacity = std::stoul(argv[1]);
  const int host_blocks = std::stoi(argv[2]);
  const int64_t device_blocks = std::stoll(argv[3]);
  const size_t batch = std::stoul(argv[4]);
  std::vector<int64_t> trace;
  int64_t x;
  while (std::cin >> x) trace.push_back(x);

  Store store(capacity, host_blocks);
  int64_t ring = 0, hits = 0, misses = 0;
  std::ios::sync_with_stdio(false);
  for (size_t b0 = 0; b0 < trace.size(); b0 += batch) {
    std::unordered_set<std::string> seen;
    std::vector<std::string> hit_h, miss_h;
    std::vector<int> hit_dev;
    std::vector<Blk> miss_slices;
    std::vector<std::pair<int, int>> saves, loads;
    const size_t b1 = b0 + batch < trace.size() ? b0 + batch : trace.size();
    for (size_t i = b0; i < b1; ++i) {
      const std::string h = key_of(trace[i]);
      if (!seen.insert(h).second) continue;
      const int d = int(ring % device_blocks);
      ++ring;
      const std::vector<Blk> r = store.Lookup({h}, /*pin_found=*/true);
      if (!r.empty()) {
        hit_h.push_back(h);
        hit_dev.push_back(d);
        loads.emplace_back(r[0].host_block_id, d);
      } else {
        miss_h.push_back(h);
        Blk s;
        s.device_block_id = d;
        s.status = kHbm;
        miss_slices.push_back(s);
      }
    }
    hits += int64_t(hit_h.size());
    misses += int64_t(miss_h.size());
    if (!hit_h.empty()) store.Load(hit_h, hit_dev);
    if (!miss_h.empty() && store.InsertAndLock(miss_h, miss_slices)) {
      if (store.SaveLocal(miss_h)) {
        store.Poll(/*save_side=*/true);
        for (size_t i = 0; i < miss_h.size(); ++i) {
          const std::vector<Blk> r = store.Lookup({miss_h[i]}, false);
          saves.emplace_back(miss_slices[i].device_block_id, r.empty() ? -1 : r[0].host_block_id);
        }
      } else {
        store.Release(miss_h);
      }
    }
    store.Poll(/*save_side=*/false);
    store.Poll(/*save_side=*/true);
    std::cout << "B " << saves.size() << " " << loads.size() << "\n";
    for (auto& s : saves) std::cout << "S " << s.first << " " << s.second << "\n";
    for (auto& l : loads) std::cout << "L " << l.first << " " << l.second << "\n";
  }
  std::cout << "H " << hits << " " << misses << "\n";
  return 0;
}

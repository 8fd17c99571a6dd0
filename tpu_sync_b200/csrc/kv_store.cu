// Tier-2 prefix cache over the pinned host tier: LRU index, host block
// allocator and the local Lookup / Insert / Release / Save / Load / Poll state
// machine.
//
// Semantics follow the reference:
//  * LRUCache (tpu_sync/kv_cache/lru_cache.h:41-364): active list (MRU first),
//    pinned list, eviction-candidate list; Put demotes the LRU entry to a
//    candidate when full; Peek hides candidates; Pin / GetAndPin resurrect
//    them; Unpin returns an entry to MRU at pin count 0; GetEvictableKeys scans
//    candidates (oldest first) then the active list from its LRU end;
//  * LogicalBlockManager (tpu_sync/kv_cache/logical_block_manager.cc:32-224):
//    Allocate takes free ids in increasing order, then evictable (allocated,
//    unlocked) ids by (last access counter, id); one counter tick per call.
//    Same order here, but from ordered sets instead of a scan of every block
//    per call;
//  * HostOffloadBackend::Lookup / InsertAndLock / Release / Evict
//    (tpu_sync/kv_cache/host_offload_backend.cc:154-288, :370-470, :529, :656);
//  * KVCacheStore::SaveLocal / Load / AllocateBlockIds / PollSavesInternal /
//    PollLoadsInternal / PollSaveStatus / PollLoadStatus
//    (tpu_sync/kv_cache/kv_cache_store.cc:977-1140, :1743-1781, :2113-2254,
//    :1453-1521), local paths only (no registry, no remote peers).
// Save / Load move bytes with the manager (ts_d2h / ts_h2d); a store created
// without a manager completes transfers immediately (host-only state tests).

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <list>
#include <mutex>
#include <set>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "kv_metadata.h"
#include "ts_internal.h"

namespace tsb {
namespace {

struct BlockId {
  int32_t host_block_id = -1;
  int32_t device_block_id = -1;
  int32_t status = TS_BLOCK_INIT;
};

// ---------------------------------------------------------------------------
// LRU index with pins and eviction candidates.
// ---------------------------------------------------------------------------
class Lru {
 public:
  enum Loc { kLru, kPinned, kCand };
  struct Node {
    std::string key;
    BlockId value;
    int pins = 0;
    Loc loc = kLru;
  };
  using It = std::list<Node>::iterator;

  explicit Lru(size_t cap) : cap_(cap) {}

  size_t capacity() const { return cap_; }
  size_t size() const { return map_.size(); }
  size_t available_space() const { return cap_ > pinned_.size() ? cap_ - pinned_.size() : 0; }
  size_t active_size() const { return lru_.size() + pinned_.size(); }

  bool contains(const std::string& k) const {
    auto it = map_.find(k);
    return it != map_.end() && it->second->loc != kCand;
  }
  BlockId* peek(const std::string& k) {
    auto it = map_.find(k);
    if (it == map_.end() || it->second->loc == kCand) return nullptr;
    return &it->second->value;
  }
  BlockId* peek_any(const std::string& k) {
    auto it = map_.find(k);
    return it == map_.end() ? nullptr : &it->second->value;
  }
  int pin_count(const std::string& k) const {
    auto it = map_.find(k);
    return it == map_.end() ? 0 : it->second->pins;
  }

  // Put: returns true and the demoted key when an entry became a candidate.
  // Inserts nothing when every entry is pinned (reference caveat).
  bool put(const std::string& k, const BlockId& v, std::string* demoted) {
    auto it = map_.find(k);
    if (it != map_.end()) {
      it->second->value = v;
      promote(it->second);
      return false;
    }
    bool evicted = false;
    if (active_size() >= cap_) {
      if (!evict(demoted)) return false;
      evicted = true;
    }
    lru_.push_front(Node{k, v, 0, kLru});
    map_.emplace(k, lru_.begin());
    return evicted;
  }

  bool pin(const std::string& k) {
    auto it = map_.find(k);
    if (it == map_.end()) return false;
    It n = it->second;
    if (n->pins == 0) {
      if (n->loc == kLru) pinned_.splice(pinned_.begin(), lru_, n);
      else if (n->loc == kCand) pinned_.splice(pinned_.begin(), cand_, n);
      n->loc = kPinned;
    }
    n->pins++;
    return true;
  }

  bool unpin(const std::string& k) {
    auto it = map_.find(k);
    if (it == map_.end()) return false;
    It n = it->second;
    if (n->pins > 0 && --n->pins == 0) {
      lru_.splice(lru_.begin(), pinned_, n);
      n->loc = kLru;
    }
    return true;
  }

  std::vector<std::string> evictable_keys(size_t count) const {
    std::vector<std::string> keys;
    for (auto it = cand_.begin(); it != cand_.end() && keys.size() < count; ++it)
      keys.push_back(it->key);
    for (auto it = lru_.rbegin(); it != lru_.rend() && keys.size() < count; ++it)
      keys.push_back(it->key);
    return keys;
  }

  bool erase(const std::string& k) {
    auto it = map_.find(k);
    if (it == map_.end() || it->second->pins > 0) return false;
    if (it->second->loc == kLru) lru_.erase(it->second);
    else if (it->second->loc == kCand) cand_.erase(it->second);
    map_.erase(it);
    return true;
  }

  std::vector<std::string> candidate_keys() const {
    std::vector<std::string> keys;
    for (const Node& n : cand_) keys.push_back(n.key);
    return keys;
  }
  std::vector<std::string> active_keys() const {  // MRU first
    std::vector<std::string> keys;
    for (const Node& n : lru_) keys.push_back(n.key);
    return keys;
  }

 private:
  bool evict(std::string* demoted) {
    if (lru_.empty()) return false;
    It n = std::prev(lru_.end());
    n->loc = kCand;
    cand_.splice(cand_.end(), lru_, n);
    if (demoted) *demoted = n->key;
    return true;
  }
  void promote(It n) {
    if (n->pins > 0) {
      pinned_.splice(pinned_.begin(), pinned_, n);
      n->loc = kPinned;
    } else if (n->loc == kLru) {
      lru_.splice(lru_.begin(), lru_, n);
    } else if (n->loc == kCand) {
      lru_.splice(lru_.begin(), cand_, n);
      n->loc = kLru;
    }
  }

  size_t cap_;
  std::list<Node> lru_, pinned_, cand_;
  std::unordered_map<std::string, It> map_;
};

// ---------------------------------------------------------------------------
// Host block allocator (LogicalBlockManager order, ordered-set bookkeeping).
// ---------------------------------------------------------------------------
class BlockAllocator {
 public:
  explicit BlockAllocator(int total) : b_(size_t(total > 0 ? total : 0)) {
    for (int i = 0; i < total; ++i) free_.insert(i);
  }
  int total() const { return int(b_.size()); }
  int num_free() const { return int(free_.size()); }
  int num_allocated() const { return total() - num_free(); }
  int num_locked() const { return locked_; }

  int allocate(int n, bool lock, std::vector<int>* out) {
    if (n <= 0) return set_errorf(TS_INVALID_ARGUMENT, "Requested blocks must be > 0, got %d", n);
    if (n > total())
      return set_errorf(TS_INVALID_ARGUMENT, "Requested blocks (%d) exceed total blocks (%d)", n,
                        total());
    if (int(free_.size() + evictable_.size()) < n)
      return set_errorf(TS_RESOURCE_EXHAUSTED,
                        "Insufficient available blocks. Requested: %d, Free: %d, Evictable: %d",
                        n, int(free_.size()), int(evictable_.size()));
    out->clear();
    while (int(out->size()) < n && !free_.empty()) {
      out->push_back(*free_.begin());
      free_.erase(free_.begin());
    }
    while (int(out->size()) < n) {  // evictable blocks are never locked
      const int id = evictable_.begin()->second;
      evictable_.erase(evictable_.begin());
      out->push_back(id);
    }
    ++counter_;
    for (int id : *out) {
      Blk& x = b_[size_t(id)];
      x.allocated = true;
      x.locked = lock;
      x.counter = counter_;
      if (lock) ++locked_;
      else evictable_.insert({counter_, id});
    }
    return TS_OK;
  }

  int deallocate(const std::vector<int>& ids) {
    for (int id : ids) {
      if (id < 0 || id >= total()) return set_errorf(TS_INVALID_ARGUMENT, "Invalid block ID: %d", id);
      if (!b_[size_t(id)].allocated)
        return set_errorf(TS_INVALID_ARGUMENT, "Cannot deallocate unallocated block ID: %d", id);
    }
    for (int id : ids) {
      Blk& x = b_[size_t(id)];
      if (!x.allocated) continue;  // duplicate id in the list
      if (x.locked) --locked_;
      else evictable_.erase({x.counter, id});
      x.allocated = false;
      x.locked = false;
      free_.insert(id);
    }
    return TS_OK;
  }

  int allocate_target(const std::vector<int>& ids) {
    std::vector<bool> seen(b_.size(), false);
    for (int id : ids) {
      if (id < 0 || id >= total()) return set_errorf(TS_INVALID_ARGUMENT, "Invalid block ID: %d", id);
      if (b_[size_t(id)].allocated)
        return set_errorf(TS_FAILED_PRECONDITION, "Already allocated block ID: %d", id);
      if (seen[size_t(id)]) return set_errorf(TS_INVALID_ARGUMENT, "Duplicate block ID: %d", id);
      seen[size_t(id)] = true;
    }
    ++counter_;
    for (int id : ids) {
      Blk& x = b_[size_t(id)];
      free_.erase(id);
      x.allocated = true;
      x.locked = true;
      x.counter = counter_;
      ++locked_;
    }
    return TS_OK;
  }

  int unlock(const std::vector<int>& ids) {
    for (int id : ids) {
      if (id < 0 || id >= total()) return set_errorf(TS_INVALID_ARGUMENT, "Invalid block ID: %d", id);
      if (!b_[size_t(id)].allocated)
        return set_errorf(TS_INVALID_ARGUMENT, "Cannot unlock unallocated block ID: %d", id);
    }
    for (int id : ids) {
      Blk& x = b_[size_t(id)];
      if (x.locked) {
        x.locked = false;
        --locked_;
        evictable_.insert({x.counter, id});
      }
    }
    return TS_OK;
  }

  int access(int id) {
    if (id < 0 || id >= total()) return set_errorf(TS_INVALID_ARGUMENT, "Invalid block ID: %d", id);
    Blk& x = b_[size_t(id)];
    if (!x.allocated)
      return set_errorf(TS_INVALID_ARGUMENT, "Cannot access unallocated block ID: %d", id);
    ++counter_;
    if (!x.locked) {
      evictable_.erase({x.counter, id});
      evictable_.insert({counter_, id});
    }
    x.counter = counter_;
    return TS_OK;
  }

 private:
  struct Blk {
    bool allocated = false;
    bool locked = false;
    uint64_t counter = 0;
  };
  std::vector<Blk> b_;
  std::set<int> free_;
  std::set<std::pair<uint64_t, int>> evictable_;
  uint64_t counter_ = 0;
  int locked_ = 0;
};

std::vector<std::string> unpack_keys(const uint8_t* keys, const int64_t* offs, int64_t n) {
  std::vector<std::string> out;
  out.reserve(size_t(n > 0 ? n : 0));
  for (int64_t i = 0; i < n; ++i)
    out.emplace_back(reinterpret_cast<const char*>(keys) + offs[i], size_t(offs[i + 1] - offs[i]));
  return out;
}

std::string hex(const std::string& s) {
  static const char* d = "0123456789abcdef";
  std::string o;
  for (unsigned char c : s) {
    o.push_back(d[c >> 4]);
    o.push_back(d[c & 15]);
  }
  return o;
}

}  // namespace
}  // namespace tsb

struct ts_store {
  explicit ts_store(size_t cap, int host_blocks) : lru(cap), alloc(host_blocks) {}
  ts_manager* mgr = nullptr;
  tsb::Lru lru;
  tsb::BlockAllocator alloc;
  std::mutex mu;
  std::unordered_set<std::string> saving, loading;
  struct Op {
    ts_event* ev = nullptr;  // null: completed at issue (no manager)
    std::vector<std::string> hashes;
    std::vector<int> host_ids;
    std::vector<int> dev_ids;
  };
  std::vector<Op> saves, loads;
  std::vector<std::string> done_saves, failed_saves, done_loads, failed_loads;
  // optional crash-persistent record of host-resident blocks
  ts_kv_metadata* meta = nullptr;
  uint64_t next_seq = 0;
};

namespace tsb {
namespace {

bool host_resident(const BlockId& b) {
  return b.status == TS_BLOCK_HOST || b.status == TS_BLOCK_HOST_AND_HBM;
}

// SetMetadataEntry / ClearMetadataEntry
// (tpu_sync/kv_cache/host_offload_backend.cc:1224-1256): only entries that
// hold host bytes are recorded; a failed record is not fatal there either.
void meta_set(ts_store* s, const std::string& hash, const BlockId& b) {
  if (s->meta == nullptr || !host_resident(b)) return;
  ts_kv_metadata_table(s->meta)->set(b.host_block_id, hash.data(), hash.size(), s->next_seq++);
}

void meta_clear(ts_store* s, const BlockId& b) {
  if (s->meta == nullptr || !host_resident(b)) return;
  ts_kv_metadata_table(s->meta)->clear(b.host_block_id);
}

// HostOffloadBackend::Lookup, local index only: every hit is found (and
// pinned when asked) in one sweep; the answer ends at the first miss and the
// pins taken past it are handed back (which, as in the reference, moves those
// entries to the MRU end).
int64_t lookup_locked(ts_store* s, const std::vector<std::string>& h, bool pin,
                      std::vector<BlockId>* out) {
  std::vector<bool> hit(h.size(), false);
  for (size_t i = 0; i < h.size(); ++i) {
    if (s->lru.peek(h[i]) != nullptr) {
      if (pin) s->lru.pin(h[i]);
      hit[i] = true;
    }
  }
  out->clear();
  size_t n = 0;
  while (n < h.size() && hit[n]) {
    out->push_back(*s->lru.peek(h[n]));
    ++n;
  }
  if (pin)
    for (size_t i = n; i < h.size(); ++i)
      if (hit[i]) s->lru.unpin(h[i]);
  return int64_t(n);
}

void release_locked(ts_store* s, const std::vector<std::string>& h) {
  for (auto it = h.rbegin(); it != h.rend(); ++it) s->lru.unpin(*it);
}

// KVCacheStore::AllocateBlockIds: evict enough unpinned host-resident entries
// (candidates first, then the LRU end) to cover the shortfall, then allocate
// locked host ids.
int allocate_host_ids(ts_store* s, int needed, std::vector<int>* ids) {
  const int to_free = needed - s->alloc.num_free();
  if (to_free > 0) {
    std::vector<std::string> keys = s->lru.evictable_keys(size_t(to_free));
    if (int(keys.size()) < to_free)
      return set_errorf(TS_RESOURCE_EXHAUSTED,
                        "Insufficient free blocks and not enough evictable blocks. Needed: %d, "
                        "Free: %d, Evictable: %d",
                        needed, s->alloc.num_free(), int(keys.size()));
    std::vector<int> host_ids;
    for (const std::string& k : keys) {
      BlockId* b = s->lru.peek_any(k);
      if (b != nullptr && s->lru.pin_count(k) == 0 &&
          (b->status == TS_BLOCK_HOST || b->status == TS_BLOCK_HOST_AND_HBM)) {
        host_ids.push_back(b->host_block_id);
        meta_clear(s, *b);
        s->lru.erase(k);
      }
    }
    if (!host_ids.empty()) s->alloc.deallocate(host_ids);
  }
  return s->alloc.allocate(needed, /*lock=*/true, ids);
}

bool op_ready(const ts_store::Op& op, int* status, std::string* msg) {
  if (op.ev == nullptr) {
    *status = TS_OK;
    return true;
  }
  const int rc = ts_event_query(op.ev);
  if (rc == TS_PENDING) return false;
  *status = rc;
  if (rc != TS_OK) *msg = ts_last_error();
  return true;
}

// PollSavesInternal / PollLoadsInternal for the operations that finished.
void poll_locked(ts_store* s) {
  for (size_t i = 0; i < s->saves.size();) {
    ts_store::Op& op = s->saves[i];
    int st;
    std::string msg;
    if (!op_ready(op, &st, &msg)) {
      ++i;
      continue;
    }
    if (st == TS_OK) {
      std::vector<std::string> updated;
      for (size_t k = 0; k < op.hashes.size(); ++k) {
        BlockId* b = s->lru.peek(op.hashes[k]);
        if (b != nullptr) {
          b->host_block_id = op.host_ids[k];
          b->status = TS_BLOCK_HOST_AND_HBM;
          meta_set(s, op.hashes[k], *b);
          updated.push_back(op.hashes[k]);
        }
        s->done_saves.push_back(op.hashes[k]);
      }
      release_locked(s, updated);
    } else {
      s->alloc.deallocate(op.host_ids);
      for (const std::string& h : op.hashes) s->failed_saves.push_back(h);
    }
    for (const std::string& h : op.hashes) s->saving.erase(h);
    if (op.ev) ts_event_release(op.ev);
    s->saves.erase(s->saves.begin() + long(i));
  }
  for (size_t i = 0; i < s->loads.size();) {
    ts_store::Op& op = s->loads[i];
    int st;
    std::string msg;
    if (!op_ready(op, &st, &msg)) {
      ++i;
      continue;
    }
    if (st == TS_OK) {
      std::vector<std::string> updated;
      for (size_t k = 0; k < op.hashes.size(); ++k) {
        BlockId* b = s->lru.peek(op.hashes[k]);
        if (b != nullptr) {
          b->device_block_id = op.dev_ids[k];
          b->status = TS_BLOCK_HOST_AND_HBM;
          meta_set(s, op.hashes[k], *b);
          updated.push_back(op.hashes[k]);
        }
        s->done_loads.push_back(op.hashes[k]);
      }
      release_locked(s, updated);
    } else {
      for (const std::string& h : op.hashes) s->failed_loads.push_back(h);
    }
    for (const std::string& h : op.hashes) s->loading.erase(h);
    if (op.ev) ts_event_release(op.ev);
    s->loads.erase(s->loads.begin() + long(i));
  }
}

int pack(const std::vector<std::vector<std::string>*>& lists, int64_t* counts, uint8_t* buf,
         int64_t buf_len, int64_t* offs, int64_t offs_len, int64_t* need_bytes,
         int64_t* need_keys) {
  int64_t nb = 0, nk = 0;
  for (auto* l : lists)
    for (const std::string& k : *l) {
      nb += int64_t(k.size());
      ++nk;
    }
  *need_bytes = nb;
  *need_keys = nk;
  for (size_t c = 0; c < lists.size(); ++c) counts[c] = int64_t(lists[c]->size());
  if (nb > buf_len || nk + 1 > offs_len || (nb > 0 && buf == nullptr) || offs == nullptr)
    return TS_RESOURCE_EXHAUSTED;
  int64_t pos = 0, i = 0;
  offs[0] = 0;
  for (auto* l : lists)
    for (const std::string& k : *l) {
      std::memcpy(buf + pos, k.data(), k.size());
      pos += int64_t(k.size());
      offs[++i] = pos;
    }
  return TS_OK;
}

}  // namespace
}  // namespace tsb

using tsb::set_error;
using tsb::set_errorf;

extern "C" int ts_store_create(ts_manager* mgr, int64_t capacity, int64_t host_blocks,
                               ts_store** out) {
  tsb::clear_error();
  if (!out) return set_error(TS_INVALID_ARGUMENT, "out must not be null");
  if (capacity < 0 || host_blocks < 0 || host_blocks > INT32_MAX)
    return set_error(TS_INVALID_ARGUMENT, "capacity and host_blocks must be non-negative");
  auto* s = new ts_store(size_t(capacity), int(host_blocks));
  s->mgr = mgr;
  *out = s;
  return TS_OK;
}

extern "C" int ts_store_destroy(ts_store* s) {
  tsb::clear_error();
  if (!s) return TS_OK;
  for (auto* ops : {&s->saves, &s->loads})
    for (auto& op : *ops)
      if (op.ev) ts_event_release(op.ev);  // waits for in-flight transfers
  delete s;
  return TS_OK;
}

extern "C" int ts_store_lookup(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n,
                               int pin_found, ts_block_info* out, int64_t* n_found) {
  tsb::clear_error();
  if (!s || !n_found || (n > 0 && (!keys || !offs || !out)))
    return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::vector<std::string> h = tsb::unpack_keys(keys, offs, n);
  std::lock_guard<std::mutex> lock(s->mu);
  std::vector<tsb::BlockId> ids;
  *n_found = tsb::lookup_locked(s, h, pin_found != 0, &ids);
  for (size_t i = 0; i < ids.size(); ++i)
    out[i] = ts_block_info{ids[i].host_block_id, ids[i].device_block_id, ids[i].status, 0};
  return TS_OK;
}

extern "C" int ts_store_insert(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n,
                               const ts_block_info* slices, int64_t n_slices, int on_host) {
  tsb::clear_error();
  (void)on_host;
  if (!s || (n > 0 && (!keys || !offs)) || (n_slices > 0 && !slices))
    return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::vector<std::string> h = tsb::unpack_keys(keys, offs, n);
  for (int64_t i = 0; i < n_slices; ++i)
    if (slices[i].status == TS_BLOCK_REMOTE)
      return set_errorf(TS_INVALID_ARGUMENT,
                        "Insert only takes LOCAL entries; slice %lld (hash %s) has status REMOTE",
                        (long long)i, i < n ? tsb::hex(h[size_t(i)]).c_str() : "<none>");
  auto slice = [&](size_t i) {
    tsb::BlockId b;
    b.host_block_id = slices[i].host_block_id;
    b.device_block_id = slices[i].device_block_id;
    b.status = slices[i].status;
    return b;
  };
  std::lock_guard<std::mutex> lock(s->mu);
  // HostOffloadBackend::InsertAndLock: all-or-nothing.
  std::vector<size_t> existing, fresh;
  for (size_t i = 0; i < h.size(); ++i) (s->lru.contains(h[i]) ? existing : fresh).push_back(i);
  const char* refused =
      "Insert refused: not enough unpinned space, or a hash could not be pinned";
  for (size_t e = 0; e < existing.size(); ++e) {
    const size_t i = existing[e];
    if (!s->lru.pin(h[i])) {
      for (size_t j = 0; j < e; ++j) s->lru.unpin(h[existing[j]]);
      return set_error(TS_RESOURCE_EXHAUSTED, refused);
    }
    if (int64_t(i) < n_slices) {
      tsb::BlockId* b = s->lru.peek(h[i]);
      if (b != nullptr && b->status == TS_BLOCK_HBM) {
        tsb::meta_clear(s, *b);
        *b = slice(i);
        tsb::meta_set(s, h[i], *b);
      }
    }
  }
  if (s->lru.available_space() < fresh.size()) {
    for (size_t i : existing) s->lru.unpin(h[i]);
    return set_error(TS_RESOURCE_EXHAUSTED, refused);
  }
  for (auto it = fresh.rbegin(); it != fresh.rend(); ++it) {
    const size_t i = *it;
    if (const tsb::BlockId* stale = s->lru.peek_any(h[i])) tsb::meta_clear(s, *stale);
    std::string demoted;
    s->lru.put(h[i], int64_t(i) < n_slices ? slice(i) : tsb::BlockId(), &demoted);
    if (int64_t(i) < n_slices) tsb::meta_set(s, h[i], slice(i));
  }
  for (size_t f = 0; f < fresh.size(); ++f) {
    if (!s->lru.pin(h[fresh[f]])) {
      for (size_t j = 0; j < f; ++j) s->lru.unpin(h[fresh[j]]);
      for (size_t j : existing) s->lru.unpin(h[j]);
      for (size_t j : fresh) {
        if (const tsb::BlockId* v = s->lru.peek_any(h[j])) tsb::meta_clear(s, *v);
        s->lru.erase(h[j]);
      }
      return set_error(TS_RESOURCE_EXHAUSTED, refused);
    }
  }
  return TS_OK;
}

extern "C" int ts_store_release(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n) {
  tsb::clear_error();
  if (!s || (n > 0 && (!keys || !offs))) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::vector<std::string> h = tsb::unpack_keys(keys, offs, n);
  std::lock_guard<std::mutex> lock(s->mu);
  tsb::release_locked(s, h);
  return TS_OK;
}

extern "C" int ts_store_pin_count(ts_store* s, const uint8_t* key, int64_t len, int* out) {
  tsb::clear_error();
  if (!s || !out || (len > 0 && !key)) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::lock_guard<std::mutex> lock(s->mu);
  *out = s->lru.pin_count(std::string(reinterpret_cast<const char*>(key), size_t(len)));
  return TS_OK;
}

extern "C" int ts_store_save(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n,
                             void* stream) {
  tsb::clear_error();
  if (!s || (n > 0 && (!keys || !offs))) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::vector<std::string> h = tsb::unpack_keys(keys, offs, n);
  // SaveLocal processes no completions: finished transfers update the index
  // only when polled (kv_cache_store.cc:977-1058), so a load finished but
  // not yet polled still holds its pin here.
  std::lock_guard<std::mutex> lock(s->mu);
  std::vector<tsb::BlockId> found;
  const int64_t nf = tsb::lookup_locked(s, h, false, &found);
  if (nf < n) return set_errorf(TS_NOT_FOUND, "Block hash not found: %s", tsb::hex(h[size_t(nf)]).c_str());
  std::vector<int64_t> src;
  for (size_t i = 0; i < h.size(); ++i) {
    const tsb::BlockId& b = found[i];
    if (b.status != TS_BLOCK_HBM)
      return set_errorf(TS_FAILED_PRECONDITION, "Block is not in HBM status: %s", tsb::hex(h[i]).c_str());
    if (b.device_block_id == -1)
      return set_errorf(TS_FAILED_PRECONDITION, "Block device_block_id is -1: %s", tsb::hex(h[i]).c_str());
    if (s->lru.pin_count(h[i]) <= 0)
      return set_errorf(TS_FAILED_PRECONDITION, "Block is not pinned: %s", tsb::hex(h[i]).c_str());
    if (s->saving.count(h[i]))
      return set_errorf(TS_FAILED_PRECONDITION, "Block is already saving: %s", tsb::hex(h[i]).c_str());
    src.push_back(b.device_block_id);
  }
  if (h.empty()) return TS_OK;
  std::vector<int> host_ids;
  int rc = tsb::allocate_host_ids(s, int(h.size()), &host_ids);
  if (rc != TS_OK) return rc;
  ts_store::Op op;
  op.hashes = h;
  op.host_ids = host_ids;
  if (s->mgr != nullptr) {
    std::vector<int64_t> dst(host_ids.begin(), host_ids.end());
    rc = ts_d2h(s->mgr, src.data(), dst.data(), nullptr, int64_t(src.size()), int64_t(dst.size()),
                0, -1, -1, stream, &op.ev);
    if (rc != TS_OK) {
      const std::string msg = ts_last_error();
      s->alloc.deallocate(host_ids);
      return set_error(rc, msg);
    }
  }
  for (const std::string& x : h) s->saving.insert(x);
  s->saves.push_back(std::move(op));
  return TS_OK;
}

extern "C" int ts_store_load(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n,
                             const int32_t* device_block_ids, int64_t n_ids, void* stream) {
  tsb::clear_error();
  if (!s || (n > 0 && (!keys || !offs || !device_block_ids)))
    return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  if (n != n_ids)
    return set_error(TS_INVALID_ARGUMENT, "block_hashes and device_block_ids size mismatch");
  if (n == 0) return TS_OK;
  std::vector<std::string> h = tsb::unpack_keys(keys, offs, n);
  std::lock_guard<std::mutex> lock(s->mu);  // no completions processed (as Load)
  std::vector<tsb::BlockId> found;
  const int64_t nf = tsb::lookup_locked(s, h, false, &found);
  if (nf < n) return set_errorf(TS_NOT_FOUND, "Block hash not found: %s", tsb::hex(h[size_t(nf)]).c_str());
  std::vector<int64_t> src, dst;
  for (size_t i = 0; i < h.size(); ++i) {
    const tsb::BlockId& b = found[i];
    const std::string x = tsb::hex(h[i]);
    if (b.status == TS_BLOCK_REMOTE)
      return set_errorf(TS_INVALID_ARGUMENT,
                        "Load without slices is local-only, but block is REMOTE: %s", x.c_str());
    if (s->lru.pin_count(h[i]) <= 0)
      return set_errorf(TS_FAILED_PRECONDITION, "Block is not pinned: %s", x.c_str());
    if (s->loading.count(h[i]))
      return set_errorf(TS_FAILED_PRECONDITION, "Block is already loading: %s", x.c_str());
    if (b.status != TS_BLOCK_HOST && b.status != TS_BLOCK_HOST_AND_HBM)
      return set_errorf(TS_FAILED_PRECONDITION, "Block is not on host: %s", x.c_str());
    if (b.host_block_id == -1)
      return set_errorf(TS_FAILED_PRECONDITION, "Block host_block_id is -1: %s", x.c_str());
    src.push_back(b.host_block_id);
    dst.push_back(device_block_ids[i]);
  }
  ts_store::Op op;
  op.hashes = h;
  op.dev_ids.assign(device_block_ids, device_block_ids + n);
  if (s->mgr != nullptr) {
    const int rc = ts_h2d(s->mgr, src.data(), dst.data(), nullptr, int64_t(src.size()),
                          int64_t(dst.size()), 0, -1, -1, stream, &op.ev);
    if (rc != TS_OK) return rc;
  }
  for (const std::string& x : h) s->loading.insert(x);
  s->loads.push_back(std::move(op));
  return TS_OK;
}

extern "C" int ts_store_poll(ts_store* s, int which, int64_t* counts, uint8_t* buf,
                             int64_t buf_len, int64_t* offs, int64_t offs_len,
                             int64_t* need_bytes, int64_t* need_keys) {
  tsb::clear_error();
  if (!s || !counts || !need_bytes || !need_keys || (which != 0 && which != 1))
    return set_error(TS_INVALID_ARGUMENT, "bad arguments");
  std::lock_guard<std::mutex> lock(s->mu);
  tsb::poll_locked(s);
  std::vector<std::string> pending, empty1, empty2;
  for (const auto& op : which == 0 ? s->saves : s->loads)
    pending.insert(pending.end(), op.hashes.begin(), op.hashes.end());
  std::vector<std::string>& done = which == 0 ? s->done_saves : s->done_loads;
  std::vector<std::string>& failed = which == 0 ? s->failed_saves : s->failed_loads;
  std::vector<std::vector<std::string>*> lists{&done, &failed, &pending};
  if (which == 0) {  // existing / unregistered: verdicts of remote saves only
    lists.push_back(&empty1);
    lists.push_back(&empty2);
  }
  const int rc = tsb::pack(lists, counts, buf, buf_len, offs, offs_len, need_bytes, need_keys);
  if (rc != TS_OK) return set_error(rc, "poll buffers too small");
  done.clear();
  failed.clear();
  return TS_OK;
}

extern "C" int ts_store_stats(ts_store* s, int64_t* stats) {
  tsb::clear_error();
  if (!s || !stats) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::lock_guard<std::mutex> lock(s->mu);
  stats[0] = int64_t(s->lru.capacity());
  stats[1] = int64_t(s->lru.size());
  stats[2] = int64_t(s->lru.available_space());
  stats[3] = s->alloc.total();
  stats[4] = s->alloc.num_free();
  stats[5] = s->alloc.num_locked();
  return TS_OK;
}

// Test hooks for the index and allocator orders (host only).
extern "C" int ts_store_lru_order(ts_store* s, int which, uint8_t* buf, int64_t buf_len,
                                  int64_t* offs, int64_t offs_len, int64_t* need_bytes,
                                  int64_t* need_keys) {
  tsb::clear_error();
  if (!s || !need_bytes || !need_keys) return set_error(TS_INVALID_ARGUMENT, "bad arguments");
  std::lock_guard<std::mutex> lock(s->mu);
  std::vector<std::string> keys =
      which == 0 ? s->lru.active_keys() : (which == 1 ? s->lru.candidate_keys()
                                                      : s->lru.evictable_keys(SIZE_MAX));
  int64_t c = 0;
  const int rc = tsb::pack({&keys}, &c, buf, buf_len, offs, offs_len, need_bytes, need_keys);
  if (rc != TS_OK) return set_error(rc, "buffers too small");
  return TS_OK;
}

extern "C" int ts_store_allocate_host_blocks(ts_store* s, int n, int lock, int32_t* out) {
  tsb::clear_error();
  if (!s || !out) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::lock_guard<std::mutex> guard(s->mu);
  std::vector<int> ids;
  const int rc = s->alloc.allocate(n, lock != 0, &ids);
  if (rc != TS_OK) return rc;
  for (size_t i = 0; i < ids.size(); ++i) out[i] = ids[i];
  return TS_OK;
}

extern "C" int ts_store_host_block_op(ts_store* s, int op, const int32_t* ids, int64_t n) {
  tsb::clear_error();
  if (!s || (n > 0 && !ids)) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::lock_guard<std::mutex> guard(s->mu);
  std::vector<int> v(ids, ids + n);
  switch (op) {
    case 0: return s->alloc.deallocate(v);
    case 1: return s->alloc.allocate_target(v);
    case 2: return s->alloc.unlock(v);
    case 3: return n == 1 ? s->alloc.access(v[0]) : set_error(TS_INVALID_ARGUMENT, "one id");
    default: return set_error(TS_INVALID_ARGUMENT, "unknown host block op");
  }
}

// Test hook: one raw operation on the store's LRU index, so its behaviour can
// be replayed against the reference LRUCache.  op: 0 put (in), 1 pin, 2 unpin,
// 3 peek, 4 peek including candidates, 5 pin count, 6 erase, 7 contains,
// 8 available space, 9 size.  *out_val gets the boolean / count / found flag;
// put returns the demoted key (if any) in out_key.
extern "C" int ts_store_lru_op(ts_store* s, int op, const uint8_t* key, int64_t len,
                               const ts_block_info* in, ts_block_info* out_info,
                               int64_t* out_val, uint8_t* out_key, int64_t out_key_cap,
                               int64_t* out_key_len) {
  tsb::clear_error();
  if (!s || !out_val) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  std::lock_guard<std::mutex> lock(s->mu);
  const std::string k(reinterpret_cast<const char*>(key ? key : (const uint8_t*)""), size_t(len));
  *out_val = 0;
  if (out_key_len) *out_key_len = -1;
  switch (op) {
    case 0: {
      if (!in) return set_error(TS_INVALID_ARGUMENT, "put needs a value");
      tsb::BlockId v;
      v.host_block_id = in->host_block_id;
      v.device_block_id = in->device_block_id;
      v.status = in->status;
      std::string demoted;
      if (s->lru.put(k, v, &demoted)) {
        *out_val = 1;
        if (out_key && out_key_len && int64_t(demoted.size()) <= out_key_cap) {
          std::memcpy(out_key, demoted.data(), demoted.size());
          *out_key_len = int64_t(demoted.size());
        }
      }
      return TS_OK;
    }
    case 1: *out_val = s->lru.pin(k); return TS_OK;
    case 2: *out_val = s->lru.unpin(k); return TS_OK;
    case 3:
    case 4: {
      tsb::BlockId* b = op == 3 ? s->lru.peek(k) : s->lru.peek_any(k);
      if (b) {
        *out_val = 1;
        if (out_info) *out_info = ts_block_info{b->host_block_id, b->device_block_id, b->status, 0};
      }
      return TS_OK;
    }
    case 5: *out_val = s->lru.pin_count(k); return TS_OK;
    case 6: *out_val = s->lru.erase(k); return TS_OK;
    case 7: *out_val = s->lru.contains(k); return TS_OK;
    case 8: *out_val = int64_t(s->lru.available_space()); return TS_OK;
    case 9: *out_val = int64_t(s->lru.size()); return TS_OK;
    default: return set_error(TS_INVALID_ARGUMENT, "unknown lru op");
  }
}

// KVCacheStore::Evict / HostOffloadBackend::Evict (kv_cache_store.cc:1553-1570,
// host_offload_backend.cc:656-686): unpinned host-resident entries among the
// keys leave the index and their host blocks return to the allocator.
extern "C" int ts_store_evict(ts_store* s, const uint8_t* keys, const int64_t* offs, int64_t n,
                              int64_t* evicted) {
  tsb::clear_error();
  if (!s || !evicted || n < 0 || (n > 0 && (!keys || !offs)))
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(s->mu);
  std::vector<int> host_ids;
  for (int64_t i = 0; i < n; ++i) {
    const std::string k(reinterpret_cast<const char*>(keys) + offs[i], size_t(offs[i + 1] - offs[i]));
    const tsb::BlockId* b = s->lru.peek_any(k);
    if (b != nullptr && s->lru.pin_count(k) == 0 && tsb::host_resident(*b)) {
      host_ids.push_back(b->host_block_id);
      tsb::meta_clear(s, *b);
      s->lru.erase(k);
    }
  }
  if (!host_ids.empty()) s->alloc.deallocate(host_ids);
  *evicted = int64_t(host_ids.size());
  return TS_OK;
}

extern "C" int ts_store_attach_metadata(ts_store* s, ts_kv_metadata* meta) {
  tsb::clear_error();
  if (!s) return set_error(TS_INVALID_ARGUMENT, "null store");
  std::lock_guard<std::mutex> lock(s->mu);
  // Host block ids index the table; one the table cannot hold goes
  // unrecorded, as a failed Set is only logged by the reference.
  s->meta = meta;
  return TS_OK;
}

// KVCacheStore::RecoverFromLocalManifest / HostOffloadBackend's
// (tpu_sync/kv_cache/kv_cache_store.cc:1541-1551,
// host_offload_backend.cc:559-617): the newest entry per hash, in recency
// order, becomes a HOST entry of the LRU over its (now allocated) host block;
// older duplicates are cleared from the table.
extern "C" int ts_store_recover(ts_store* s, int64_t* recovered) {
  tsb::clear_error();
  if (!s || !recovered) return set_error(TS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lock(s->mu);
  *recovered = 0;
  if (s->lru.size() != 0)
    return set_error(TS_FAILED_PRECONDITION,
                     "RecoverFromLocalManifest can only be called on an empty cache store");
  if (s->meta == nullptr)
    return set_error(TS_FAILED_PRECONDITION, "KVCacheMetadata is required for crash recovery");
  tsb::meta::Table* t = ts_kv_metadata_table(s->meta);
  const std::vector<tsb::meta::Record> entries = t->valid_entries();
  if (entries.empty()) return TS_OK;
  std::unordered_map<std::string, const tsb::meta::Record*> newest;
  for (const auto& e : entries) {
    auto it = newest.find(e.hash);
    if (it == newest.end())
      newest.emplace(e.hash, &e);
    else if (e.seq > it->second->seq)
      it->second = &e;
  }
  std::vector<const tsb::meta::Record*> keep;
  for (const auto& [hash, e] : newest) keep.push_back(e);
  std::sort(keep.begin(), keep.end(),
            [](const tsb::meta::Record* a, const tsb::meta::Record* b) { return a->seq < b->seq; });
  std::vector<int> ids;
  for (const auto* e : keep) ids.push_back(e->block_id);
  int rc = s->alloc.allocate_target(ids);
  if (rc != TS_OK) return rc;
  uint64_t max_seq = 0;
  for (const auto* e : keep) {
    tsb::BlockId b;
    b.host_block_id = e->block_id;
    b.device_block_id = -1;
    b.status = TS_BLOCK_HOST;
    std::string demoted;
    s->lru.put(e->hash, b, &demoted);
    max_seq = std::max(max_seq, e->seq);
  }
  s->next_seq = max_seq + 1;
  for (const auto& e : entries)
    if (newest.at(e.hash)->block_id != e.block_id) t->clear(e.block_id);
  *recovered = int64_t(keep.size());
  return TS_OK;
}

// Crash-persistent KV block metadata: which host block holds which prefix
// hash, kept in a /dev/shm segment next to the shared-memory host tier so a
// restarted process can rebuild its tier-2 index over the surviving blocks.
//
// Restates KVCacheMetadata (tpu_sync/kv_cache/kv_cache_metadata.h:19-106,
// kv_cache_metadata.cc:27-173) and KVCacheMetadataShmRegion
// (kv_cache_metadata_shm.cc:29-160).  The on-memory format is the
// reference's byte for byte (a table written by either side attaches on the
// other): a 128-byte header {u64 magic "RAIDENKM", u32 version 1, u32
// num_blocks, u32 entry_size 128, char model_uid[64] at offset 20} followed
// by num_blocks 128-byte entries {u64 seq, u16 hash_len, u8 valid at offset
// 10 (committed last, with release ordering), 5 reserved bytes, 112 hash
// bytes at offset 16}.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <cstring>
#include <string>
#include <vector>

#include "kv_metadata.h"
#include "ts_internal.h"

namespace tsb {
namespace meta {

namespace {

constexpr uint64_t kMagic = 0x52414944454E4B4Dull;  // "RAIDENKM"
constexpr uint32_t kVersion = 1;
constexpr size_t kHeaderBytes = 128;
constexpr size_t kEntryBytes = 128;
constexpr size_t kUidBytes = 64;
constexpr size_t kMaxHash = 112;

struct alignas(64) Header {
  uint64_t magic;
  uint32_t version;
  uint32_t num_blocks;
  uint32_t entry_size;
  char model_uid[kUidBytes];
};
static_assert(sizeof(Header) == kHeaderBytes, "header layout");
static_assert(offsetof(Header, model_uid) == 20, "header layout");

struct alignas(64) Entry {
  uint64_t seq;
  uint16_t hash_len;
  std::atomic<uint8_t> valid;
  uint8_t reserved[5];
  char hash[kMaxHash];
};
static_assert(sizeof(Entry) == kEntryBytes, "entry layout");
static_assert(offsetof(Entry, hash) == 16, "entry layout");
static_assert(std::atomic<uint8_t>::is_always_lock_free, "lock-free valid byte");

std::string S(int64_t v) { return std::to_string(v); }

int validate_region(const void* region, uint64_t size, int num_blocks, const std::string& uid) {
  if (num_blocks <= 0)
    return set_error(TS_INVALID_ARGUMENT, "num_blocks must be positive, got " + S(num_blocks));
  if (uid.size() >= kUidBytes)
    return set_error(TS_INVALID_ARGUMENT, "model_uid length " + S(int64_t(uid.size())) +
                                              " exceeds the maximum of " + S(kUidBytes - 1));
  if (region == nullptr) return set_error(TS_INVALID_ARGUMENT, "Metadata region is null");
  if (reinterpret_cast<uintptr_t>(region) % 64 != 0)
    return set_error(TS_INVALID_ARGUMENT, "Metadata region must be 64-byte aligned");
  const uint64_t need = required_bytes(num_blocks);
  if (size < need)
    return set_error(TS_INVALID_ARGUMENT, "Metadata region too small: " + S(int64_t(size)) +
                                              " bytes, need " + S(int64_t(need)));
  return TS_OK;
}

Entry* entries_of(void* region) {
  return reinterpret_cast<Entry*>(static_cast<uint8_t*>(region) + kHeaderBytes);
}

}  // namespace

uint64_t required_bytes(int num_blocks) {
  return kHeaderBytes + uint64_t(num_blocks) * kEntryBytes;
}

int Table::format(void* region, uint64_t size, int num_blocks, const std::string& uid) {
  int rc = validate_region(region, size, num_blocks, uid);
  if (rc != TS_OK) return rc;
  // fields written in place over the zeroed table: the header's padding
  // bytes [84, 128) stay zero
  std::memset(region, 0, required_bytes(num_blocks));
  Header* h = static_cast<Header*>(region);
  h->magic = kMagic;
  h->version = kVersion;
  h->num_blocks = uint32_t(num_blocks);
  h->entry_size = uint32_t(kEntryBytes);
  std::memcpy(h->model_uid, uid.data(), uid.size());
  base = region;
  blocks = num_blocks;
  return TS_OK;
}

int Table::attach(void* region, uint64_t size, int num_blocks, const std::string& uid) {
  int rc = validate_region(region, size, num_blocks, uid);
  if (rc != TS_OK) return rc;
  const Header* h = static_cast<const Header*>(region);
  if (h->magic != kMagic) return set_error(TS_FAILED_PRECONDITION, "Metadata region magic mismatch");
  if (h->version != kVersion)
    return set_error(TS_FAILED_PRECONDITION, "Metadata region version mismatch: " +
                                                 S(h->version) + " vs " + S(kVersion));
  if (h->entry_size != kEntryBytes)
    return set_error(TS_FAILED_PRECONDITION, "Metadata entry size mismatch: " +
                                                 S(h->entry_size) + " vs " + S(kEntryBytes));
  if (h->num_blocks != uint32_t(num_blocks))
    return set_error(TS_FAILED_PRECONDITION, "Metadata num_blocks mismatch: " +
                                                 S(h->num_blocks) + " vs " + S(num_blocks));
  const std::string recorded(h->model_uid, strnlen(h->model_uid, kUidBytes));
  if (recorded != uid)
    return set_error(TS_FAILED_PRECONDITION,
                     "Metadata model_uid mismatch: \"" + recorded + "\" vs \"" + uid + "\"");
  base = region;
  blocks = num_blocks;
  return TS_OK;
}

int Table::set(int block_id, const void* hash, size_t len, uint64_t seq) {
  if (block_id < 0 || block_id >= blocks)
    return set_error(TS_INVALID_ARGUMENT, "Block ID out of range: " + S(block_id));
  if (len == 0) return set_error(TS_INVALID_ARGUMENT, "Hash must not be empty");
  if (len > kMaxHash)
    return set_error(TS_INVALID_ARGUMENT, "Hash length " + S(int64_t(len)) +
                                              " exceeds the maximum of " + S(kMaxHash));
  Entry& e = entries_of(base)[block_id];
  // invalidate first, commit last: a crash in between leaves the slot empty
  e.valid.store(0, std::memory_order_release);
  e.seq = seq;
  e.hash_len = uint16_t(len);
  std::memcpy(e.hash, hash, len);
  e.valid.store(1, std::memory_order_release);
  return TS_OK;
}

int Table::clear(int block_id) {
  if (block_id < 0 || block_id >= blocks)
    return set_error(TS_INVALID_ARGUMENT, "Block ID out of range: " + S(block_id));
  entries_of(base)[block_id].valid.store(0, std::memory_order_release);
  return TS_OK;
}

std::vector<Record> Table::valid_entries() const {
  std::vector<Record> out;
  const Entry* es = entries_of(base);
  for (int i = 0; i < blocks; ++i) {
    const Entry& e = es[i];
    if (e.valid.load(std::memory_order_acquire) == 0) continue;
    if (e.hash_len == 0 || e.hash_len > kMaxHash) continue;
    out.push_back({i, std::string(e.hash, e.hash_len), e.seq});
  }
  return out;
}

}  // namespace meta
}  // namespace tsb

// A table on a /dev/shm segment (AttachOrFormat) or on caller memory.
struct ts_kv_metadata {
  tsb::meta::Table table;
  std::string key;  // "" for caller memory
  void* mapped = nullptr;
  size_t mapped_size = 0;
  int fd = -1;
  bool warm = false;
  std::string uid;
};

using tsb::set_error;

tsb::meta::Table* ts_kv_metadata_table(ts_kv_metadata* m) { return &m->table; }

namespace {

std::string shm_key(const char* k) {
  std::string key(k ? k : "");
  if (key.empty() || key[0] != '/') key.insert(0, "/");
  return key;
}

size_t page_aligned(int num_blocks) {
  return size_t((tsb::meta::required_bytes(num_blocks) + 4095) & ~uint64_t(4095));
}

}  // namespace

extern "C" uint64_t ts_kv_metadata_required_bytes(int num_blocks) {
  return num_blocks > 0 ? tsb::meta::required_bytes(num_blocks) : 0;
}

extern "C" int ts_kv_metadata_open(const char* key_c, int num_blocks, const char* model_uid,
                                   ts_kv_metadata** out, int* warm) {
  tsb::clear_error();
  if (!out) return set_error(TS_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  if (num_blocks <= 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "num_blocks must be positive, got " + std::to_string(num_blocks));
  const std::string key = shm_key(key_c);
  const std::string uid = model_uid ? model_uid : "";
  const size_t size = page_aligned(num_blocks);
  // warm path: a surviving segment whose table validates
  int fd = shm_open(key.c_str(), O_RDWR, 0666);
  if (fd >= 0) {
    struct stat st;
    void* mapped = MAP_FAILED;
    if (fstat(fd, &st) == 0 && size_t(st.st_size) >= size)
      mapped = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (mapped != MAP_FAILED) {
      auto* m = new ts_kv_metadata();
      if (m->table.attach(mapped, size, num_blocks, uid) == TS_OK) {
        m->key = key;
        m->mapped = mapped;
        m->mapped_size = size;
        m->fd = fd;
        m->warm = true;
        m->uid = uid;
        *out = m;
        if (warm) *warm = 1;
        tsb::clear_error();
        return TS_OK;
      }
      delete m;
      munmap(mapped, size);
    }
    close(fd);
    shm_unlink(key.c_str());
  }
  // cold path: a fresh segment with an empty table
  fd = shm_open(key.c_str(), O_CREAT | O_RDWR | O_EXCL, 0666);
  if (fd < 0) fd = shm_open(key.c_str(), O_CREAT | O_RDWR, 0666);
  if (fd < 0)
    return set_error(TS_INTERNAL, "shm_open failed to create KV metadata segment " + key + ": " +
                                      std::strerror(errno));
  if (ftruncate(fd, off_t(size)) != 0) {
    const int e = errno;
    close(fd);
    shm_unlink(key.c_str());
    return set_error(TS_INTERNAL,
                     "ftruncate failed on KV metadata segment " + key + ": " + std::strerror(e));
  }
  void* mapped = mmap(nullptr, size, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  if (mapped == MAP_FAILED) {
    const int e = errno;
    close(fd);
    shm_unlink(key.c_str());
    return set_error(TS_RESOURCE_EXHAUSTED,
                     "mmap failed on KV metadata segment " + key + ": " + std::strerror(e));
  }
  auto* m = new ts_kv_metadata();
  int rc = m->table.format(mapped, size, num_blocks, uid);
  if (rc != TS_OK) {
    delete m;
    munmap(mapped, size);
    close(fd);
    shm_unlink(key.c_str());
    return rc;
  }
  m->key = key;
  m->mapped = mapped;
  m->mapped_size = size;
  m->fd = fd;
  m->warm = false;
  m->uid = uid;
  *out = m;
  if (warm) *warm = 0;
  return TS_OK;
}

extern "C" int ts_kv_metadata_on_region(void* region, uint64_t size, int num_blocks,
                                        const char* model_uid, int attach, ts_kv_metadata** out) {
  tsb::clear_error();
  if (!out) return set_error(TS_INVALID_ARGUMENT, "null output");
  *out = nullptr;
  auto* m = new ts_kv_metadata();
  m->uid = model_uid ? model_uid : "";
  const int rc = attach ? m->table.attach(region, size, num_blocks, m->uid)
                        : m->table.format(region, size, num_blocks, m->uid);
  if (rc != TS_OK) {
    delete m;
    return rc;
  }
  m->warm = attach != 0;
  *out = m;
  return TS_OK;
}

extern "C" int ts_kv_metadata_set(ts_kv_metadata* m, int block_id, const uint8_t* hash,
                                  int64_t len, uint64_t seq) {
  tsb::clear_error();
  if (!m) return set_error(TS_INVALID_ARGUMENT, "null metadata");
  if (len < 0 || (len > 0 && !hash)) return set_error(TS_INVALID_ARGUMENT, "invalid hash");
  return m->table.set(block_id, hash, size_t(len), seq);
}

extern "C" int ts_kv_metadata_clear(ts_kv_metadata* m, int block_id) {
  tsb::clear_error();
  if (!m) return set_error(TS_INVALID_ARGUMENT, "null metadata");
  return m->table.clear(block_id);
}

extern "C" int ts_kv_metadata_entries(ts_kv_metadata* m, int32_t* block_ids, uint64_t* seqs,
                                      uint8_t* buf, int64_t buf_len, int64_t* offs,
                                      int64_t cap, int64_t* n_out, int64_t* need_bytes) {
  tsb::clear_error();
  if (!m || !n_out || !need_bytes) return set_error(TS_INVALID_ARGUMENT, "null argument");
  const std::vector<tsb::meta::Record> es = m->table.valid_entries();
  int64_t bytes = 0;
  for (const auto& e : es) bytes += int64_t(e.hash.size());
  *n_out = int64_t(es.size());
  *need_bytes = bytes;
  if (int64_t(es.size()) > cap || bytes > buf_len || !block_ids || !seqs || !offs ||
      (bytes > 0 && !buf))
    return es.empty() ? TS_OK : set_error(TS_RESOURCE_EXHAUSTED, "entry capacity too small");
  int64_t pos = 0;
  for (size_t i = 0; i < es.size(); ++i) {
    block_ids[i] = es[i].block_id;
    seqs[i] = es[i].seq;
    offs[i] = pos;
    std::memcpy(buf + pos, es[i].hash.data(), es[i].hash.size());
    pos += int64_t(es[i].hash.size());
  }
  offs[es.size()] = pos;
  return TS_OK;
}

extern "C" int ts_kv_metadata_reformat(ts_kv_metadata* m) {
  tsb::clear_error();
  if (!m || !m->table.base) return set_error(TS_INVALID_ARGUMENT, "null metadata");
  const uint64_t size = m->mapped ? m->mapped_size : tsb::meta::required_bytes(m->table.blocks);
  int rc = m->table.format(m->table.base, size, m->table.blocks, m->uid);
  if (rc == TS_OK) m->warm = false;
  return rc;
}

extern "C" int ts_kv_metadata_info(ts_kv_metadata* m, int* num_blocks, int* warm) {
  tsb::clear_error();
  if (!m) return set_error(TS_INVALID_ARGUMENT, "null metadata");
  if (num_blocks) *num_blocks = m->table.blocks;
  if (warm) *warm = m->warm ? 1 : 0;
  return TS_OK;
}

extern "C" int ts_kv_metadata_close(ts_kv_metadata* m, int unlink_shm) {
  if (!m) return TS_OK;
  if (m->mapped) munmap(m->mapped, m->mapped_size);
  if (m->fd >= 0) close(m->fd);
  if (unlink_shm && !m->key.empty()) shm_unlink(m->key.c_str());
  delete m;
  return TS_OK;
}

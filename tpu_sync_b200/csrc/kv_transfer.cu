// Same-node KV block hand-off between managers: the reference's pull protocol
// (producer NotifyForRead, consumer StartRead, both CompleteRead;
// tpu_sync/core/kv_cache_manager_with_transfer.cc:624-665, :1478-1760) with
// the TCP control and data planes replaced by a /dev/shm mailbox, CUDA IPC
// and one copy kernel over NVLink.
//
// Producer (ts_xfer_endpoint): publishes a mailbox named by its endpoint
// string.  The header lists the manager's storages (IPC handle of each
// allocation, offset, geometry); every registered read is an entry {uuid,
// req_id, block ids}.  Registration records an event on the producer's
// stream; a watcher thread of the endpoint marks the entry READY once that
// event has completed, i.e. once the blocks are written.
//
// Consumer (ts_xfer_reader): maps the producer's storages once per process
// and device, claims the READY entry of a uuid, copies every storage's bytes
// of each (remote block, local block) pair with one kernel that loads the
// peer's memory over NVLink, and records its own completion.  Its poll
// reports the read done (or failed) and marks the entry consumed; the
// producer's poll then reports the send done and recycles the entry.
//
// No event crosses a process or a device: a stream of one GPU waiting on an
// interprocess event recorded on another GPU crashed the process in the
// CUDA runtime on this platform, so readiness travels through the mailbox.
//
// Entry state words carry a generation (upper 24 bits) that changes every
// time the entry is recycled, so a late consumer cannot touch an entry that
// was timed out and reused.  A producer times out entries nobody claimed
// (reported as done sending, as the reference does); a claimed entry waits
// for its consumer unless that process has exited.  Producer and consumer
// in one process use raw pointers and events (CUDA IPC handles cannot be
// opened by the process that exported them).

#include <fcntl.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <cerrno>
#include <chrono>
#include <condition_variable>
#include <thread>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <unordered_set>
#include <vector>

#include <cuda_runtime.h>

#include "ts_internal.h"

using tsb::set_error;
using tsb::set_errorf;

namespace tsb {
namespace xfer {
namespace {

constexpr uint64_t kMagic = 0x3152454658425354ull;  // "TSBXFER1" little-endian
constexpr uint32_t kVersion = 1;
constexpr int kReqIdBytes = 128;
constexpr size_t kHeaderBytes = 4096;

enum : uint32_t { kFree = 0, kWriting = 1, kRegistered = 2, kReady = 3, kReading = 4,
                  kConsumed = 5, kFailed = 6 };

struct alignas(64) Header {
  uint64_t magic;
  uint32_t version;
  int32_t n_storages;
  int32_t max_entries;
  int32_t max_blocks;
  int32_t device;  // the producer's device ordinal in its process
  int32_t pid;     // the producer process
  uint64_t nonce;  // new on every create: readers remap when it changes
  uint64_t storages_off, entries_off, blocks_off, total_bytes;
};

struct StorageRec {
  uint8_t handle[64];  // cudaIpcMemHandle_t of the allocation holding the storage
  uint64_t offset;     // the storage's byte offset in that allocation
  uint64_t dev_ptr;    // its address in the producer process
  uint64_t nbytes;
  int64_t dim0;
  uint64_t block_bytes;
  uint64_t pad[3];
};
static_assert(sizeof(StorageRec) == 128, "storage record layout");

struct alignas(64) Entry {
  std::atomic<uint32_t> word;  // generation << 8 | state
  int32_t consumer_pid;
  int64_t n_blocks;
  uint64_t uuid;
  int64_t deadline_ns;         // CLOCK_MONOTONIC, the same clock in every process
  uint64_t reserved[9];
  char req_id[kReqIdBytes];
};
static_assert(std::atomic<uint32_t>::is_always_lock_free, "lock-free state word");

uint32_t state_of(uint32_t w) { return w & 0xffu; }
uint32_t gen_of(uint32_t w) { return w >> 8; }
uint32_t make_word(uint32_t gen, uint32_t st) { return ((gen & 0xffffffu) << 8) | st; }

int64_t now_ns() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return int64_t(ts.tv_sec) * 1000000000 + ts.tv_nsec;
}

std::string shm_name(const std::string& endpoint) {
  std::string n = endpoint;
  if (n.rfind("ipc:", 0) == 0) n = n.substr(4);
  if (n.empty() || n[0] != '/') n.insert(0, "/");
  return n;
}

// pid 0: the consumer claimed the entry and has not written its pid yet.
// Step trace of the consumer path on stderr when TSB_XFER_TRACE is set.
void trace(const char* what) {
  static const bool on = std::getenv("TSB_XFER_TRACE") != nullptr;
  if (on) {
    std::fprintf(stderr, "xfer: %s\n", what);
    std::fflush(stderr);
  }
}

bool process_alive(int pid) { return pid <= 0 || kill(pid, 0) == 0 || errno != ESRCH; }

// Blocks a storage holds at its block size: the bound every block id of a
// copy is checked against (the kernel addresses id x block bytes).
int64_t blocks_of(uint64_t nbytes, uint64_t bb) { return bb == 0 ? INT64_MAX : int64_t(nbytes / bb); }

struct Mailbox {
  std::string name;
  int fd = -1;
  void* map = nullptr;
  size_t bytes = 0;
  Header* h = nullptr;
  StorageRec* st = nullptr;
  Entry* e = nullptr;
  int64_t* blocks = nullptr;

  void bind() {
    h = static_cast<Header*>(map);
    st = reinterpret_cast<StorageRec*>(static_cast<uint8_t*>(map) + h->storages_off);
    e = reinterpret_cast<Entry*>(static_cast<uint8_t*>(map) + h->entries_off);
    blocks = reinterpret_cast<int64_t*>(static_cast<uint8_t*>(map) + h->blocks_off);
  }
  void release() {
    if (map) munmap(map, bytes);
    if (fd >= 0) close(fd);
    map = nullptr;
    fd = -1;
  }
};

// Storages of a manager: (device pointer, bytes, dim0, block bytes).
struct Geo {
  uint64_t ptr, nbytes, bb;
  int64_t dim0;
};

int manager_geometry(ts_manager* mgr, int* device, std::vector<Geo>* out) {
  int n = 0;
  int rc = ts_mgr_num_storages(mgr, &n);
  if (rc != TS_OK) return rc;
  out->resize(size_t(n));
  for (int i = 0; i < n; ++i) {
    Geo& g = (*out)[size_t(i)];
    rc = ts_mgr_storage(mgr, i, device, &g.ptr, &g.nbytes, &g.dim0, &g.bb);
    if (rc != TS_OK) return rc;
  }
  return TS_OK;
}

// Packs strings into (buf, offs) under the capacity protocol of the C ABI.
int pack_strings(std::vector<std::string>* items, uint8_t* buf, int64_t buf_len, int64_t* offs,
                 int64_t offs_len, int64_t* n_out, int64_t* need_bytes) {
  int64_t bytes = 0;
  for (const auto& s : *items) bytes += int64_t(s.size());
  *n_out = int64_t(items->size());
  *need_bytes = bytes;
  if (items->empty()) return TS_OK;
  if (bytes > buf_len || offs_len < int64_t(items->size()) + 1 || !offs || (bytes > 0 && !buf))
    return set_error(TS_RESOURCE_EXHAUSTED, "result buffer too small");
  int64_t pos = 0;
  for (size_t i = 0; i < items->size(); ++i) {
    offs[i] = pos;
    std::memcpy(buf + pos, (*items)[i].data(), (*items)[i].size());
    pos += int64_t((*items)[i].size());
  }
  offs[items->size()] = pos;
  items->clear();
  return TS_OK;
}

// ---------------------------------------------------------------------------
// The copy kernel: every storage's block bytes of each (remote, local) pair.
// ---------------------------------------------------------------------------

struct PeerStorage {
  uint64_t src;  // the producer's storage base as this device addresses it
  uint64_t dst;  // the local storage base
  uint64_t bb;
};

constexpr int kThreads = 256;
constexpr int kVec = 8;
constexpr uint64_t kPiece = uint64_t(kThreads) * kVec * 16;  // 32 KiB

template <bool kVector>
__global__ void __launch_bounds__(kThreads)
    peer_block_copy_kernel(const PeerStorage* __restrict__ st, int n_st,
                           const int64_t* __restrict__ pairs, int64_t n_pairs, uint32_t ppu) {
  const int64_t per_pair = int64_t(n_st) * ppu;
  const int64_t units = n_pairs * per_pair;
  for (int64_t w = blockIdx.x; w < units; w += gridDim.x) {
    const int64_t k = w / per_pair;
    const int64_t r = w - k * per_pair;
    const int s = int(r / ppu);
    const uint64_t off = uint64_t(r - int64_t(s) * ppu) * kPiece;
    const uint64_t bb = st[s].bb;
    if (off >= bb) continue;
    const uint64_t nbytes = bb - off < kPiece ? bb - off : kPiece;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(st[s].src) + uint64_t(pairs[2 * k]) * bb + off;
    uint8_t* dst = reinterpret_cast<uint8_t*>(st[s].dst) + uint64_t(pairs[2 * k + 1]) * bb + off;
    if (kVector) {
      const uint32_t nvec = uint32_t(nbytes >> 4);
      int4 v[kVec];
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const uint32_t idx = threadIdx.x + uint32_t(i) * kThreads;
        if (idx < nvec) v[i] = reinterpret_cast<const int4*>(src)[idx];
      }
#pragma unroll
      for (int i = 0; i < kVec; ++i) {
        const uint32_t idx = threadIdx.x + uint32_t(i) * kThreads;
        if (idx < nvec) reinterpret_cast<int4*>(dst)[idx] = v[i];
      }
    } else {
      for (uint64_t b = threadIdx.x; b < nbytes; b += kThreads) dst[b] = src[b];
    }
  }
}

}  // namespace
}  // namespace xfer
}  // namespace tsb

using namespace tsb::xfer;

// ===========================================================================
// Producer
// ===========================================================================

struct ts_xfer_endpoint {
  Mailbox mb;
  int device = 0;
  int64_t timeout_ns = 0;
  std::vector<cudaEvent_t> events;  // per entry: the "blocks written" event
  std::vector<std::string> done_sending;
  std::mutex mu;
  std::condition_variable cv;
  bool stop = false;
  int pending = 0;  // entries registered whose event has not completed
  std::thread watcher;
};

namespace {

void recycle(ts_xfer_endpoint* ep, int i, uint32_t gen) {
  if (ep->events[size_t(i)] != nullptr) {
    cudaEventDestroy(ep->events[size_t(i)]);
    ep->events[size_t(i)] = nullptr;
  }
  ep->mb.e[i].word.store(make_word(gen + 1, kFree), std::memory_order_release);
}

// Marks registered entries READY once their event completed (FAILED if the
// event reports an error).  Runs on the watcher thread, under ep->mu.
void mark_ready_locked(ts_xfer_endpoint* ep) {
  int pending = 0;
  for (int i = 0; i < ep->mb.h->max_entries; ++i) {
    Entry& e = ep->mb.e[i];
    uint32_t w = e.word.load(std::memory_order_acquire);
    if (state_of(w) != kRegistered) continue;
    const cudaError_t q = cudaEventQuery(ep->events[size_t(i)]);
    if (q == cudaErrorNotReady) {
      ++pending;
      continue;
    }
    e.word.compare_exchange_strong(w, make_word(gen_of(w), q == cudaSuccess ? kReady : kFailed),
                                   std::memory_order_acq_rel);
  }
  ep->pending = pending;
}

void watch(ts_xfer_endpoint* ep) {
  cudaSetDevice(ep->device);
  std::unique_lock<std::mutex> lock(ep->mu);
  while (!ep->stop) {
    if (ep->pending > 0)
      ep->cv.wait_for(lock, std::chrono::microseconds(50));
    else
      ep->cv.wait_for(lock, std::chrono::milliseconds(100));
    if (ep->stop) break;
    mark_ready_locked(ep);
  }
}

// CompleteRead's producer half: consumed (or failed) entries are sends done;
// registered entries nobody claimed before their deadline time out (done
// too, as the reference's send entries do); a claimed entry whose consumer
// exited is released.
void poll_sends_locked(ts_xfer_endpoint* ep) {
  const int64_t now = now_ns();
  for (int i = 0; i < ep->mb.h->max_entries; ++i) {
    Entry& e = ep->mb.e[i];
    uint32_t w = e.word.load(std::memory_order_acquire);
    const uint32_t st = state_of(w), gen = gen_of(w);
    bool done = false;
    if (st == kConsumed || st == kFailed) {
      done = true;
    } else if ((st == kRegistered || st == kReady) && now > e.deadline_ns) {
      done = e.word.compare_exchange_strong(w, make_word(gen, kFailed), std::memory_order_acq_rel);
    } else if (st == kReading && !process_alive(e.consumer_pid)) {
      done = e.word.compare_exchange_strong(w, make_word(gen, kFailed), std::memory_order_acq_rel);
    }
    if (done) {
      ep->done_sending.emplace_back(e.req_id, strnlen(e.req_id, kReqIdBytes));
      recycle(ep, i, gen);
    }
  }
}

}  // namespace

extern "C" int ts_xfer_endpoint_create(ts_manager* mgr, const char* name, int max_entries,
                                       int max_blocks, int64_t timeout_ms,
                                       ts_xfer_endpoint** out) {
  tsb::clear_error();
  if (!mgr || !name || !out) return set_error(TS_INVALID_ARGUMENT, "null argument");
  *out = nullptr;
  if (max_entries <= 0 || max_blocks <= 0 || timeout_ms <= 0)
    return set_error(TS_INVALID_ARGUMENT, "max_entries, max_blocks and timeout must be positive");
  int device = 0;
  std::vector<Geo> geo;
  int rc = manager_geometry(mgr, &device, &geo);
  if (rc != TS_OK) return rc;
  std::vector<StorageRec> recs(geo.size());
  for (size_t i = 0; i < geo.size(); ++i) {
    std::memset(&recs[i], 0, sizeof(StorageRec));
    rc = ts_ipc_export(reinterpret_cast<const void*>(geo[i].ptr), recs[i].handle, &recs[i].offset);
    if (rc != TS_OK) return rc;
    recs[i].dev_ptr = geo[i].ptr;
    recs[i].nbytes = geo[i].nbytes;
    recs[i].dim0 = geo[i].dim0;
    recs[i].block_bytes = geo[i].bb;
  }
  const uint64_t storages_off = kHeaderBytes;
  const uint64_t entries_off = storages_off + sizeof(StorageRec) * geo.size();
  const uint64_t blocks_off = entries_off + sizeof(Entry) * uint64_t(max_entries);
  const uint64_t total = (blocks_off + 8ull * uint64_t(max_entries) * uint64_t(max_blocks) + 4095) &
                         ~uint64_t(4095);
  auto* ep = new ts_xfer_endpoint();
  ep->mb.name = shm_name(name);
  shm_unlink(ep->mb.name.c_str());  // a mailbox left by an earlier producer of this name
  ep->mb.fd = shm_open(ep->mb.name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (ep->mb.fd < 0) {
    delete ep;
    return set_errorf(TS_INTERNAL, "shm_open of the transfer mailbox failed: %s", std::strerror(errno));
  }
  if (ftruncate(ep->mb.fd, off_t(total)) != 0) {
    const int e = errno;
    ep->mb.release();
    shm_unlink(ep->mb.name.c_str());
    delete ep;
    return set_errorf(TS_INTERNAL, "ftruncate of the transfer mailbox failed: %s", std::strerror(e));
  }
  ep->mb.bytes = size_t(total);
  ep->mb.map = mmap(nullptr, ep->mb.bytes, PROT_READ | PROT_WRITE, MAP_SHARED, ep->mb.fd, 0);
  if (ep->mb.map == MAP_FAILED) {
    const int e = errno;
    ep->mb.map = nullptr;
    ep->mb.release();
    shm_unlink(ep->mb.name.c_str());
    delete ep;
    return set_errorf(TS_RESOURCE_EXHAUSTED, "mmap of the transfer mailbox failed: %s",
                      std::strerror(e));
  }
  Header* h = static_cast<Header*>(ep->mb.map);
  std::memset(h, 0, kHeaderBytes);
  h->version = kVersion;
  h->n_storages = int32_t(geo.size());
  h->max_entries = max_entries;
  h->max_blocks = max_blocks;
  h->device = device;
  h->pid = int32_t(getpid());
  h->nonce = uint64_t(now_ns()) ^ (uint64_t(getpid()) << 32);
  h->storages_off = storages_off;
  h->entries_off = entries_off;
  h->blocks_off = blocks_off;
  h->total_bytes = total;
  ep->mb.bind();
  std::memcpy(ep->mb.st, recs.data(), sizeof(StorageRec) * recs.size());
  for (int i = 0; i < max_entries; ++i) new (&ep->mb.e[i]) Entry();
  std::atomic_thread_fence(std::memory_order_release);
  h->magic = kMagic;  // published last: readers check it
  ep->device = device;
  ep->timeout_ns = timeout_ms * 1000000;
  ep->events.assign(size_t(max_entries), nullptr);
  ep->watcher = std::thread(watch, ep);
  *out = ep;
  return TS_OK;
}

extern "C" int ts_xfer_endpoint_destroy(ts_xfer_endpoint* ep) {
  if (!ep) return TS_OK;
  {
    std::lock_guard<std::mutex> lock(ep->mu);
    ep->stop = true;
  }
  ep->cv.notify_all();
  if (ep->watcher.joinable()) ep->watcher.join();
  tsb::DeviceGuard g(ep->device);
  for (cudaEvent_t e : ep->events)
    if (e) cudaEventDestroy(e);
  ep->mb.release();
  shm_unlink(ep->mb.name.c_str());
  delete ep;
  return TS_OK;
}

extern "C" int ts_xfer_register_read(ts_xfer_endpoint* ep, const char* req_id, uint64_t uuid,
                                     const int64_t* block_ids, int64_t n, void* stream,
                                     int* registered) {
  tsb::clear_error();
  if (!ep || !req_id || !registered || n < 0 || (n > 0 && !block_ids))
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  *registered = 0;
  if (n == 0) return TS_OK;  // nothing to transfer
  const size_t rl = std::strlen(req_id);
  if (rl >= size_t(kReqIdBytes))
    return set_errorf(TS_INVALID_ARGUMENT, "req_id longer than %d bytes", kReqIdBytes - 1);
  Header* h = ep->mb.h;
  if (n > h->max_blocks)
    return set_errorf(TS_INVALID_ARGUMENT, "%lld blocks exceed the endpoint's %d per read",
                      (long long)n, h->max_blocks);
  int64_t dim0 = INT64_MAX;
  for (int s = 0; s < h->n_storages; ++s)
    dim0 = std::min(dim0, blocks_of(ep->mb.st[s].nbytes, ep->mb.st[s].block_bytes));
  for (int64_t i = 0; i < n; ++i)
    if (block_ids[i] < 0 || block_ids[i] >= dim0)
      return set_errorf(TS_OUT_OF_RANGE, "block id %lld out of range [0, %lld)",
                        (long long)block_ids[i], (long long)dim0);
  std::lock_guard<std::mutex> lock(ep->mu);
  poll_sends_locked(ep);
  for (int i = 0; i < h->max_entries; ++i) {
    const uint32_t st = state_of(ep->mb.e[i].word.load(std::memory_order_acquire));
    if ((st == kRegistered || st == kReady || st == kReading) && ep->mb.e[i].uuid == uuid)
      return set_errorf(TS_ALREADY_EXISTS, "uuid %llu is already registered for read",
                        (unsigned long long)uuid);
  }
  int slot = -1;
  uint32_t gen = 0;
  for (int i = 0; i < h->max_entries && slot < 0; ++i) {
    uint32_t w = ep->mb.e[i].word.load(std::memory_order_acquire);
    if (state_of(w) == kFree &&
        ep->mb.e[i].word.compare_exchange_strong(w, make_word(gen_of(w), kWriting),
                                                 std::memory_order_acq_rel)) {
      slot = i;
      gen = gen_of(w);
    }
  }
  if (slot < 0)
    return set_errorf(TS_RESOURCE_EXHAUSTED, "all %d read entries of the endpoint are in use",
                      h->max_entries);
  Entry& e = ep->mb.e[slot];
  tsb::DeviceGuard g(ep->device);
  cudaEvent_t ev = nullptr;
  cudaError_t ce = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventRecord(ev, reinterpret_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    if (ev) cudaEventDestroy(ev);
    e.word.store(make_word(gen, kFree), std::memory_order_release);
    return tsb::cuda_error(ce, "read registration event");
  }
  ep->events[size_t(slot)] = ev;
  e.uuid = uuid;
  e.n_blocks = n;
  e.consumer_pid = 0;
  e.deadline_ns = now_ns() + ep->timeout_ns;
  std::memset(e.req_id, 0, kReqIdBytes);
  std::memcpy(e.req_id, req_id, rl);
  std::memcpy(ep->mb.blocks + int64_t(slot) * h->max_blocks, block_ids, sizeof(int64_t) * size_t(n));
  e.word.store(make_word(gen, kRegistered), std::memory_order_release);
  ep->pending += 1;
  ep->cv.notify_all();
  *registered = 1;
  return TS_OK;
}

extern "C" int ts_xfer_poll_sends(ts_xfer_endpoint* ep, uint8_t* buf, int64_t buf_len,
                                  int64_t* offs, int64_t offs_len, int64_t* n_out,
                                  int64_t* need_bytes) {
  tsb::clear_error();
  if (!ep || !n_out || !need_bytes) return set_error(TS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lock(ep->mu);
  poll_sends_locked(ep);
  return pack_strings(&ep->done_sending, buf, buf_len, offs, offs_len, n_out, need_bytes);
}

extern "C" int ts_xfer_read_state(ts_xfer_endpoint* ep, uint64_t uuid, int* state) {
  tsb::clear_error();
  if (!ep || !state) return set_error(TS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lock(ep->mu);
  mark_ready_locked(ep);
  *state = 0;
  for (int i = 0; i < ep->mb.h->max_entries; ++i) {
    const uint32_t st = state_of(ep->mb.e[i].word.load(std::memory_order_acquire));
    if (st != kFree && st != kWriting && ep->mb.e[i].uuid == uuid) *state = int(st);
  }
  return TS_OK;
}

extern "C" int ts_xfer_endpoint_name(ts_xfer_endpoint* ep, char* buf, int64_t cap) {
  tsb::clear_error();
  if (!ep || !buf || cap <= int64_t(ep->mb.name.size()))
    return set_error(TS_INVALID_ARGUMENT, "name buffer too small");
  std::memcpy(buf, ep->mb.name.c_str(), ep->mb.name.size() + 1);
  return TS_OK;
}

// ===========================================================================
// Consumer
// ===========================================================================

namespace {

struct Remote {
  Mailbox mb;
  uint64_t nonce = 0;
  bool same_process = false;
  std::vector<void*> opened;        // IPC mappings taken (ts_ipc_open), released on close
  PeerStorage* d_table = nullptr;   // device table of (src, dst, bb) per storage
  bool vec = true;
  uint32_t ppu = 1;
  int64_t dim0 = 0;
};

struct Read {
  std::string req_id;
  uint64_t uuid = 0;
  Remote* rem = nullptr;
  std::vector<int64_t> pairs;  // remote, local interleaved
  cudaStream_t stream = nullptr;
  int64_t deadline_ns = 0;
  bool launched = false;
  int entry = -1;
  uint32_t gen = 0;
  cudaEvent_t done = nullptr;
};

}  // namespace

struct ts_xfer_reader {
  int device = 0;
  std::vector<Geo> local;
  int64_t timeout_ns = 0;
  std::map<std::string, Remote*> remotes;
  std::vector<Read> reads;
  std::vector<std::string> done_recving, failed_recving;
  std::mutex mu;
};

namespace {

void close_remote(ts_xfer_reader* r, Remote* rem) {
  if (rem->d_table) {
    tsb::DeviceGuard g(r->device);
    cudaFree(rem->d_table);
  }
  for (void* base : rem->opened) ts_ipc_close(r->device, base);
  rem->mb.release();
  delete rem;
}

bool reads_use(ts_xfer_reader* r, Remote* rem) {
  for (const Read& x : r->reads)
    if (x.rem == rem) return true;
  return false;
}

int open_remote(ts_xfer_reader* r, const std::string& name, Remote** out) {
  auto it = r->remotes.find(name);
  if (it != r->remotes.end()) {
    Remote* rem = it->second;
    if (rem->mb.h->magic == kMagic && rem->mb.h->nonce == rem->nonce) {
      *out = rem;
      return TS_OK;
    }
    if (reads_use(r, rem))
      return set_error(TS_FAILED_PRECONDITION,
                       "the producer endpoint was re-created while reads from it are in flight");
    close_remote(r, rem);
    r->remotes.erase(it);
  }
  trace("open_remote: map");
  auto* rem = new Remote();
  rem->mb.name = name;
  rem->mb.fd = shm_open(name.c_str(), O_RDWR, 0600);
  if (rem->mb.fd < 0) {
    delete rem;
    return set_errorf(TS_NOT_FOUND, "no transfer endpoint %s: %s", name.c_str(), std::strerror(errno));
  }
  struct stat sb;
  if (fstat(rem->mb.fd, &sb) != 0 || uint64_t(sb.st_size) < kHeaderBytes) {
    rem->mb.release();
    delete rem;
    return set_errorf(TS_FAILED_PRECONDITION, "transfer endpoint %s is not initialised", name.c_str());
  }
  rem->mb.bytes = size_t(sb.st_size);
  rem->mb.map = mmap(nullptr, rem->mb.bytes, PROT_READ | PROT_WRITE, MAP_SHARED, rem->mb.fd, 0);
  if (rem->mb.map == MAP_FAILED) {
    rem->mb.map = nullptr;
    rem->mb.release();
    delete rem;
    return set_errorf(TS_RESOURCE_EXHAUSTED, "mmap of endpoint %s failed", name.c_str());
  }
  Header* h = static_cast<Header*>(rem->mb.map);
  if (h->magic != kMagic || h->version != kVersion || h->total_bytes > rem->mb.bytes) {
    rem->mb.release();
    delete rem;
    return set_errorf(TS_FAILED_PRECONDITION, "%s is not a transfer endpoint of this version",
                      name.c_str());
  }
  std::atomic_thread_fence(std::memory_order_acquire);
  rem->mb.bind();
  rem->nonce = h->nonce;
  // the producer's geometry must be the consumer's (storage for storage)
  if (size_t(h->n_storages) != r->local.size()) {
    const int ns = h->n_storages;
    rem->mb.release();
    delete rem;
    return set_errorf(TS_INVALID_ARGUMENT, "remote endpoint has %d storages, the local manager %d",
                      ns, int(r->local.size()));
  }
  rem->dim0 = INT64_MAX;
  for (int s = 0; s < h->n_storages; ++s) {
    if (rem->mb.st[s].block_bytes != r->local[size_t(s)].bb) {
      const unsigned long long a = rem->mb.st[s].block_bytes, b = r->local[size_t(s)].bb;
      rem->mb.release();
      delete rem;
      return set_errorf(TS_INVALID_ARGUMENT,
                        "storage %d: remote block bytes %llu differ from the local %llu", s, a, b);
    }
    rem->dim0 = std::min(rem->dim0, blocks_of(rem->mb.st[s].nbytes, rem->mb.st[s].block_bytes));
  }
  rem->same_process = h->pid == int32_t(getpid());
  trace(rem->same_process ? "open_remote: same process" : "open_remote: other process");
  std::vector<PeerStorage> table(size_t(h->n_storages));
  uint64_t max_bb = 0;
  int rc = TS_OK;
  if (rem->same_process && h->device != r->device) {
    trace("open_remote: enable peer access");
    rc = ts_enable_peer_access(r->device, h->device);
  }
  for (int s = 0; s < h->n_storages && rc == TS_OK; ++s) {
    uint64_t base = 0;
    if (rem->same_process) {
      base = rem->mb.st[s].dev_ptr;
    } else {
      void* b = nullptr;
      rc = ts_ipc_open(r->device, rem->mb.st[s].handle, &b);
      if (rc != TS_OK) break;
      rem->opened.push_back(b);
      base = uint64_t(reinterpret_cast<uintptr_t>(b)) + rem->mb.st[s].offset;
    }
    table[size_t(s)] = {base, r->local[size_t(s)].ptr, r->local[size_t(s)].bb};
    rem->vec = rem->vec && (base % 16 == 0) && (table[size_t(s)].dst % 16 == 0) &&
               (table[size_t(s)].bb % 16 == 0);
    max_bb = std::max(max_bb, table[size_t(s)].bb);
  }
  trace("open_remote: storage table");
  if (rc == TS_OK) {
    tsb::DeviceGuard g(r->device);
    cudaError_t ce = cudaMalloc(&rem->d_table, sizeof(PeerStorage) * table.size());
    if (ce == cudaSuccess)
      ce = cudaMemcpy(rem->d_table, table.data(), sizeof(PeerStorage) * table.size(),
                      cudaMemcpyHostToDevice);
    if (ce != cudaSuccess) rc = tsb::cuda_error(ce, "peer storage table");
  }
  if (rc != TS_OK) {
    close_remote(r, rem);
    return rc;
  }
  rem->ppu = uint32_t((max_bb + kPiece - 1) / kPiece);
  if (rem->ppu == 0) rem->ppu = 1;
  r->remotes[name] = rem;
  *out = rem;
  return TS_OK;
}

// Claims the producer's entry for `x` and queues the copy; *launched = 0
// when the producer has not registered the uuid yet.
int try_launch(ts_xfer_reader* r, Read* x, bool* launched) {
  *launched = false;
  Remote* rem = x->rem;
  Header* h = rem->mb.h;
  int slot = -1;
  uint32_t gen = 0;
  for (int i = 0; i < h->max_entries && slot < 0; ++i) {
    Entry& e = rem->mb.e[i];
    uint32_t w = e.word.load(std::memory_order_acquire);
    if (state_of(w) != kReady || e.uuid != x->uuid) continue;
    if (e.word.compare_exchange_strong(w, make_word(gen_of(w), kReading),
                                       std::memory_order_acq_rel)) {
      slot = i;
      gen = gen_of(w);
    }
  }
  if (slot < 0) return TS_OK;
  trace("try_launch: claimed");
  Entry& e = rem->mb.e[slot];
  e.consumer_pid = int32_t(getpid());
  x->entry = slot;
  x->gen = gen;
  auto fail_entry = [&]() {
    uint32_t w = make_word(gen, kReading);
    e.word.compare_exchange_strong(w, make_word(gen, kFailed), std::memory_order_acq_rel);
  };
  // only registered blocks may be read (the producer serves those)
  std::unordered_set<int64_t> reg(rem->mb.blocks + int64_t(slot) * h->max_blocks,
                                  rem->mb.blocks + int64_t(slot) * h->max_blocks + e.n_blocks);
  for (size_t k = 0; k < x->pairs.size(); k += 2) {
    if (!reg.count(x->pairs[k])) {
      fail_entry();
      return set_errorf(TS_INVALID_ARGUMENT, "block %lld was not registered for read by uuid %llu",
                        (long long)x->pairs[k], (unsigned long long)x->uuid);
    }
  }
  trace("try_launch: blocks checked");
  // READY: the producer's writes of these blocks completed before it set
  // the state, so the copy needs no wait on the producer's stream
  tsb::DeviceGuard g(r->device);
  cudaError_t ce = cudaSuccess;
  void* d_pairs = nullptr;
  const size_t pbytes = sizeof(int64_t) * x->pairs.size();
  if (ce == cudaSuccess) ce = cudaMallocAsync(&d_pairs, pbytes, x->stream);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(d_pairs, x->pairs.data(), pbytes, cudaMemcpyHostToDevice, x->stream);
  trace("try_launch: kernel");
  if (ce == cudaSuccess) {
    const int64_t n_pairs = int64_t(x->pairs.size() / 2);
    const int64_t units = n_pairs * h->n_storages * int64_t(rem->ppu);
    const int64_t cap = int64_t(tsb::sm_count(r->device)) * 8;
    const int grid = int(units < cap ? units : cap);
    if (rem->vec)
      peer_block_copy_kernel<true><<<grid, kThreads, 0, x->stream>>>(
          rem->d_table, h->n_storages, static_cast<const int64_t*>(d_pairs), n_pairs, rem->ppu);
    else
      peer_block_copy_kernel<false><<<grid, kThreads, 0, x->stream>>>(
          rem->d_table, h->n_storages, static_cast<const int64_t*>(d_pairs), n_pairs, rem->ppu);
    ce = cudaGetLastError();
  }
  if (d_pairs) {
    const cudaError_t fe = cudaFreeAsync(d_pairs, x->stream);
    if (ce == cudaSuccess) ce = fe;
  }
  trace("try_launch: done event");
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&x->done, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventRecord(x->done, x->stream);
  if (ce != cudaSuccess) {
    if (x->done) cudaEventDestroy(x->done);
    x->done = nullptr;
    fail_entry();
    return tsb::cuda_error(ce, "peer block read");
  }
  *launched = true;
  x->launched = true;
  return TS_OK;
}

void finish(ts_xfer_reader* r, Read* x, bool ok) {
  if (x->entry >= 0) {
    Entry& e = x->rem->mb.e[x->entry];
    uint32_t w = make_word(x->gen, kReading);
    e.word.compare_exchange_strong(w, make_word(x->gen, ok ? kConsumed : kFailed),
                                   std::memory_order_acq_rel);
  }
  tsb::DeviceGuard g(r->device);
  if (x->done) cudaEventDestroy(x->done);
  (ok ? r->done_recving : r->failed_recving).push_back(x->req_id);
}

void poll_reads_locked(ts_xfer_reader* r) {
  const int64_t now = now_ns();
  for (size_t i = 0; i < r->reads.size();) {
    Read& x = r->reads[i];
    bool finished = false, ok = false;
    if (!x.launched) {
      bool launched = false;
      const int rc = try_launch(r, &x, &launched);
      if (rc != TS_OK) {
        finished = true;
      } else if (!launched && now > x.deadline_ns) {
        finished = true;  // the producer never registered the uuid in time
      }
    } else {
      tsb::DeviceGuard g(r->device);
      const cudaError_t q = cudaEventQuery(x.done);
      if (q == cudaSuccess) {
        finished = ok = true;
      } else if (q != cudaErrorNotReady) {
        finished = true;
      }
    }
    if (finished) {
      finish(r, &x, ok);
      r->reads.erase(r->reads.begin() + int64_t(i));
    } else {
      ++i;
    }
  }
}

}  // namespace

extern "C" int ts_xfer_reader_create(ts_manager* mgr, int64_t timeout_ms, ts_xfer_reader** out) {
  tsb::clear_error();
  if (!mgr || !out) return set_error(TS_INVALID_ARGUMENT, "null argument");
  if (timeout_ms <= 0) return set_error(TS_INVALID_ARGUMENT, "timeout must be positive");
  *out = nullptr;
  auto* r = new ts_xfer_reader();
  int rc = manager_geometry(mgr, &r->device, &r->local);
  if (rc != TS_OK) {
    delete r;
    return rc;
  }
  r->timeout_ns = timeout_ms * 1000000;
  *out = r;
  return TS_OK;
}

extern "C" int ts_xfer_reader_destroy(ts_xfer_reader* r) {
  if (!r) return TS_OK;
  {
    std::lock_guard<std::mutex> lock(r->mu);
    tsb::DeviceGuard g(r->device);
    for (Read& x : r->reads) {
      if (x.launched && x.done) cudaEventSynchronize(x.done);
      finish(r, &x, x.launched);
    }
    r->reads.clear();
    for (auto& kv : r->remotes) close_remote(r, kv.second);
    r->remotes.clear();
  }
  delete r;
  return TS_OK;
}

extern "C" int ts_xfer_start_read(ts_xfer_reader* r, const char* req_id, uint64_t uuid,
                                  const char* endpoint, const int64_t* remote_ids,
                                  const int64_t* local_ids, int64_t n, void* stream) {
  tsb::clear_error();
  if (!r || !req_id || !endpoint || n < 0 || (n > 0 && (!remote_ids || !local_ids)))
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  int64_t local_dim0 = INT64_MAX;
  for (const Geo& g : r->local) local_dim0 = std::min(local_dim0, blocks_of(g.nbytes, g.bb));
  for (int64_t i = 0; i < n; ++i)
    if (local_ids[i] < 0 || local_ids[i] >= local_dim0)
      return set_errorf(TS_OUT_OF_RANGE, "local block id %lld out of range [0, %lld)",
                        (long long)local_ids[i], (long long)local_dim0);
  std::lock_guard<std::mutex> lock(r->mu);
  if (n == 0) {  // nothing to move
    r->done_recving.emplace_back(req_id);
    return TS_OK;
  }
  Remote* rem = nullptr;
  int rc = open_remote(r, shm_name(endpoint), &rem);
  if (rc != TS_OK) return rc;
  for (int64_t i = 0; i < n; ++i)
    if (remote_ids[i] < 0 || remote_ids[i] >= rem->dim0)
      return set_errorf(TS_OUT_OF_RANGE, "remote block id %lld out of range [0, %lld)",
                        (long long)remote_ids[i], (long long)rem->dim0);
  // A registration of this uuid that does not cover the requested blocks
  // fails the read now (and is released to its producer as failed).
  for (int i = 0; i < rem->mb.h->max_entries; ++i) {
    Entry& e = rem->mb.e[i];
    uint32_t w = e.word.load(std::memory_order_acquire);
    const uint32_t st = state_of(w);
    if ((st != kRegistered && st != kReady) || e.uuid != uuid) continue;
    const int64_t* reg = rem->mb.blocks + int64_t(i) * rem->mb.h->max_blocks;
    std::unordered_set<int64_t> have(reg, reg + e.n_blocks);
    for (int64_t k = 0; k < n; ++k) {
      if (!have.count(remote_ids[k])) {
        e.word.compare_exchange_strong(w, make_word(gen_of(w), kFailed), std::memory_order_acq_rel);
        return set_errorf(TS_INVALID_ARGUMENT,
                          "block %lld was not registered for read by uuid %llu",
                          (long long)remote_ids[k], (unsigned long long)uuid);
      }
    }
    break;
  }
  Read x;
  x.req_id = req_id;
  x.uuid = uuid;
  x.rem = rem;
  x.stream = reinterpret_cast<cudaStream_t>(stream);
  x.deadline_ns = now_ns() + r->timeout_ns;
  x.pairs.resize(size_t(2 * n));
  for (int64_t i = 0; i < n; ++i) {
    x.pairs[size_t(2 * i)] = remote_ids[i];
    x.pairs[size_t(2 * i + 1)] = local_ids[i];
  }
  bool launched = false;
  rc = try_launch(r, &x, &launched);
  if (rc != TS_OK) return rc;
  r->reads.push_back(std::move(x));  // launched, or pending the producer's registration
  return TS_OK;
}

extern "C" int ts_xfer_poll_reads(ts_xfer_reader* r, int which, uint8_t* buf, int64_t buf_len,
                                  int64_t* offs, int64_t offs_len, int64_t* n_out,
                                  int64_t* need_bytes) {
  tsb::clear_error();
  if (!r || !n_out || !need_bytes || (which != 0 && which != 1))
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  std::lock_guard<std::mutex> lock(r->mu);
  if (which == 0) poll_reads_locked(r);
  return pack_strings(which == 0 ? &r->done_recving : &r->failed_recving, buf, buf_len, offs,
                      offs_len, n_out, need_bytes);
}

extern "C" int ts_xfer_reader_pending(ts_xfer_reader* r, int64_t* n) {
  tsb::clear_error();
  if (!r || !n) return set_error(TS_INVALID_ARGUMENT, "null argument");
  std::lock_guard<std::mutex> lock(r->mu);
  *n = int64_t(r->reads.size());
  return TS_OK;
}

// Weight-sync reshard pulled by the receivers ("staged pull").
//
// Measured on this platform: a kernel loading a peer GPU's memory over
// NVLink reaches the peer-copy rate (1.00-1.01 of it), a kernel or the copy
// engines storing into a peer's memory stop near 0.92.  The push paths
// (ts_reshard_copy into a peer, ts_reshard_ce_*) cast on the sender and
// store; this path makes the receiver read:
//
//   sender    fp32 shard --cast kernel, group by group--> local bf16 staging
//             (same element layout), each group published in a /dev/shm
//             mailbox by a watcher thread once its cast event completed;
//   receiver  maps each sender's staging (CUDA IPC), and launches, in group
//             order, the strided copies of its chunks (the reshard kernel,
//             bf16 -> bf16, peer loads + local stores) as soon as every
//             sender they read from has published the groups they need;
//             when its copies have finished it acknowledges the generation
//             in each sender's mailbox, and a sender waits for every
//             attached receiver's acknowledgement before it overwrites the
//             staging with the next generation.
//
// No kernel waits on another GPU or process: all readiness goes through
// host memory, and every host wait is bounded by the caller's timeout.
//
// Reference: WeightSynchronizerBase::PushWeightsResharded
// (tpu_sync/weight_sync/weight_synchronizer_base.cc:558-760) pushes each
// entry's bytes from the sender's host mirror over TCP into the receiver's
// host buffer, then H2D; the chunks here are the same (src_off, dst_off,
// size, strides, count) rows, read by the receiver instead.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "ts_internal.h"

using tsb::set_error;
using tsb::set_errorf;

namespace tsb {
namespace wpull {
namespace {

constexpr uint64_t kMagic = 0x314c4c5550575354ull;  // "TSWPULL1" little-endian
constexpr uint32_t kVersion = 2;
constexpr int kMaxGroups = 64;   // groups per staging (n_groups + 3 at most)
constexpr int kMaxGroupArg = kMaxGroups - 3;
constexpr int kMaxReceivers = 16;
constexpr uint64_t kDetached = ~uint64_t(0);  // a receiver slot nobody waits for
constexpr size_t kBoxBytes = 4096;

struct alignas(64) Box {
  uint64_t magic;
  uint32_t version;
  int32_t device;      // the sender's device ordinal in its process
  int32_t pid;         // the sender process
  int32_t n_groups;
  uint64_t n_elems;      // bf16 elements of the staging
  uint64_t group_elems;  // the full group size (elements)
  uint64_t dev_ptr;      // the staging's address in the sender's process
  uint8_t handle[64];    // cudaIpcMemHandle_t of the staging allocation
  uint64_t offset;       // the staging's byte offset in that allocation
  std::atomic<uint64_t> gen;          // generation staged last (0: none yet)
  std::atomic<int32_t> n_receivers;   // receiver slots claimed
  alignas(64) std::atomic<uint64_t> ready[kMaxGroups];     // generation published per group
  alignas(64) std::atomic<uint64_t> done[kMaxReceivers];   // generation pulled per receiver
  uint64_t bounds[kMaxGroups + 1];  // group g = staging elements [bounds[g], bounds[g + 1])
};
static_assert(sizeof(Box) <= kBoxBytes, "mailbox layout");
static_assert(std::atomic<uint64_t>::is_always_lock_free, "lock-free mailbox words");

std::string shm_path(const char* name) {
  std::string n = name ? name : "";
  if (n.rfind("ipc:", 0) == 0) n = n.substr(4);
  if (n.empty() || n[0] != '/') n.insert(0, "/");
  return n;
}

using Clock = std::chrono::steady_clock;

// Spins (yielding) until pred() holds or the deadline passes.
template <typename Pred>
bool wait_until(Pred pred, Clock::time_point deadline) {
  for (uint32_t i = 0;; ++i) {
    if (pred()) return true;
    if ((i & 255u) == 255u && Clock::now() > deadline) return pred();
    if (i < 4096) {
      std::this_thread::yield();
    } else {
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
}

Clock::time_point deadline_in(int64_t timeout_ms) {
  if (timeout_ms < 0) timeout_ms = int64_t(1) << 40;  // effectively none
  return Clock::now() + std::chrono::milliseconds(timeout_ms);
}

// One launch of the reshard kernel: a device chunk table with its prefix.
struct Launch {
  ts_reshard_chunk* d_chunks = nullptr;
  int64_t* d_prefix = nullptr;
  int64_t n_chunks = 0, n_items = 0;
  uint64_t bytes = 0;
};

int upload(int device, const std::vector<ts_reshard_chunk>& chunks, int src_dtype,
           int dst_dtype, Launch* out) {
  out->n_chunks = int64_t(chunks.size());
  std::vector<int64_t> prefix(chunks.size() + 1, 0);
  int rc = ts_reshard_work_items(chunks.data(), out->n_chunks, src_dtype, dst_dtype,
                                 prefix.data());
  if (rc != TS_OK) return rc;
  out->n_items = prefix.back();
  DeviceGuard g(device);
  TS_CUDA_RET(cudaMalloc(&out->d_chunks, sizeof(ts_reshard_chunk) * chunks.size()),
              "pull chunk table");
  TS_CUDA_RET(cudaMalloc(&out->d_prefix, sizeof(int64_t) * prefix.size()), "pull chunk table");
  TS_CUDA_RET(cudaMemcpy(out->d_chunks, chunks.data(), sizeof(ts_reshard_chunk) * chunks.size(),
                         cudaMemcpyHostToDevice),
              "pull chunk table");
  TS_CUDA_RET(cudaMemcpy(out->d_prefix, prefix.data(), sizeof(int64_t) * prefix.size(),
                         cudaMemcpyHostToDevice),
              "pull chunk table");
  return TS_OK;
}

void free_launch(Launch* l) {
  if (l->d_chunks) cudaFree(l->d_chunks);
  if (l->d_prefix) cudaFree(l->d_prefix);
  l->d_chunks = nullptr;
  l->d_prefix = nullptr;
}

}  // namespace
}  // namespace wpull
}  // namespace tsb

// ---------------------------------------------------------------------------
// Sender
// ---------------------------------------------------------------------------

struct ts_wpull_src {
  int device = 0;
  std::string path;
  tsb::wpull::Box* box = nullptr;
  uint8_t* staging = nullptr;
  uint64_t n_elems = 0;
  std::vector<tsb::wpull::Launch> casts;  // one per group
  std::vector<cudaEvent_t> cast_done;     // one per group
  cudaStream_t stream = nullptr;
  cudaEvent_t start = nullptr;
  std::thread watcher;                    // publishes the last stage()'s groups
  std::atomic<int> published{0};          // groups of the last stage() published
  std::atomic<int> watch_error{0};
  uint64_t gen = 0;
};

namespace {

void src_join(ts_wpull_src* p) {
  if (p->watcher.joinable()) p->watcher.join();
}

void src_release(ts_wpull_src* p) {
  src_join(p);
  if (p->box) {
    // Receivers in other processes map the staging: give them a moment to
    // detach (ts_wpull_dst_destroy) before it is freed.
    tsb::wpull::Box* box = p->box;
    tsb::wpull::wait_until(
        [&] {
          const int n = std::min(box->n_receivers.load(std::memory_order_acquire),
                                 tsb::wpull::kMaxReceivers);
          for (int r = 0; r < n; ++r)
            if (box->done[r].load(std::memory_order_acquire) != tsb::wpull::kDetached)
              return false;
          return true;
        },
        tsb::wpull::deadline_in(2000));
  }
  {
    tsb::DeviceGuard g(p->device);
    if (p->stream) cudaStreamSynchronize(p->stream);
    for (auto& l : p->casts) tsb::wpull::free_launch(&l);
    for (cudaEvent_t e : p->cast_done)
      if (e) cudaEventDestroy(e);
    if (p->start) cudaEventDestroy(p->start);
    if (p->stream) cudaStreamDestroy(p->stream);
    if (p->staging) cudaFree(p->staging);
  }
  if (p->box) {
    munmap(p->box, tsb::wpull::kBoxBytes);
    shm_unlink(p->path.c_str());
  }
  delete p;
}

}  // namespace

extern "C" int ts_wpull_src_create(int device, const char* name, const void* src_f32,
                                   int64_t n_elems, int n_groups, ts_wpull_src** out) {
  using namespace tsb::wpull;
  tsb::clear_error();
  if (!out || !name || !src_f32 || n_elems <= 0)
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  *out = nullptr;
  if (n_groups < 1 || n_groups > kMaxGroupArg)
    return set_errorf(TS_INVALID_ARGUMENT, "n_groups must be in [1, %d]", kMaxGroupArg);
  if (reinterpret_cast<uintptr_t>(src_f32) % 16 != 0)
    return set_error(TS_INVALID_ARGUMENT, "the fp32 source must be 16-byte aligned");
  auto* p = new ts_wpull_src();
  p->device = device;
  p->path = shm_path(name);
  p->n_elems = uint64_t(n_elems);
  // Group size ge = n_elems / n_groups, a multiple of 8 elements (whole
  // 16-byte bf16 vectors).  The first three groups are ge/8, ge/4 and ge/2:
  // receivers can start after a short first cast, and the cast of each next
  // group still finishes before the receivers have read the previous one
  // (the cast moves 6 bytes of HBM per element, a receiver 2 of NVLink).
  uint64_t ge = (uint64_t(n_elems) + uint64_t(n_groups) - 1) / uint64_t(n_groups);
  ge = (ge + 7) / 8 * 8;
  std::vector<uint64_t> bounds{0};
  while (bounds.back() < uint64_t(n_elems)) {
    const int k = int(bounds.size()) - 1;
    uint64_t sz = k < 3 ? (ge >> (3 - k)) : ge;
    sz = std::max<uint64_t>(8, (sz + 7) / 8 * 8);
    bounds.push_back(std::min<uint64_t>(bounds.back() + sz, uint64_t(n_elems)));
  }
  const int groups = int(bounds.size()) - 1;
  tsb::DeviceGuard g(device);
  cudaError_t ce = cudaMalloc(&p->staging, uint64_t(n_elems) * 2);
  if (ce != cudaSuccess) {
    src_release(p);
    return tsb::cuda_error(ce, "pull staging");
  }
  for (int k = 0; k < groups; ++k) {
    const uint64_t a = bounds[size_t(k)], b = bounds[size_t(k) + 1];
    ts_reshard_chunk c{};
    c.src_ptr = reinterpret_cast<uint64_t>(src_f32);
    c.dst_ptr = reinterpret_cast<uint64_t>(p->staging);
    c.src_off = c.dst_off = int64_t(a);
    c.size = c.src_stride = c.dst_stride = int64_t(b - a);
    c.count = 1;
    Launch l;
    int rc = upload(device, {c}, TS_DTYPE_F32, TS_DTYPE_BF16, &l);
    l.bytes = (b - a) * 2;
    p->casts.push_back(l);
    if (rc != TS_OK) {
      src_release(p);
      return rc;
    }
    cudaEvent_t e = nullptr;
    ce = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    p->cast_done.push_back(e);
    if (ce != cudaSuccess) {
      src_release(p);
      return tsb::cuda_error(ce, "pull events");
    }
  }
  ce = cudaStreamCreateWithFlags(&p->stream, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming);
  if (ce != cudaSuccess) {
    src_release(p);
    return tsb::cuda_error(ce, "pull stream");
  }
  uint8_t handle[64];
  uint64_t offset = 0;
  int rc = ts_ipc_export(p->staging, handle, &offset);
  if (rc != TS_OK) {
    src_release(p);
    return rc;
  }
  const int fd = shm_open(p->path.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
  if (fd < 0) {
    const int err = errno;
    p->path.clear();  // not ours: do not unlink
    src_release(p);
    return set_errorf(err == EEXIST ? TS_ALREADY_EXISTS : TS_INTERNAL,
                      "pull mailbox %s: %s", name, strerror(err));
  }
  if (ftruncate(fd, off_t(kBoxBytes)) != 0) {
    const int err = errno;
    close(fd);
    src_release(p);
    return set_errorf(TS_INTERNAL, "pull mailbox size: %s", strerror(err));
  }
  void* m = mmap(nullptr, kBoxBytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    const int err = errno;
    src_release(p);
    return set_errorf(TS_INTERNAL, "pull mailbox map: %s", strerror(err));
  }
  std::memset(m, 0, kBoxBytes);
  auto* box = static_cast<Box*>(m);
  p->box = box;
  box->version = kVersion;
  box->device = device;
  box->pid = int32_t(getpid());
  box->n_groups = groups;
  box->n_elems = uint64_t(n_elems);
  box->group_elems = ge;
  for (int k = 0; k <= groups; ++k) box->bounds[k] = bounds[size_t(k)];
  box->dev_ptr = reinterpret_cast<uint64_t>(p->staging);
  std::memcpy(box->handle, handle, 64);
  box->offset = offset;
  for (int r = 0; r < kMaxReceivers; ++r) box->done[r].store(kDetached);
  std::atomic_thread_fence(std::memory_order_release);
  reinterpret_cast<std::atomic<uint64_t>*>(&box->magic)->store(kMagic, std::memory_order_release);
  *out = p;
  return TS_OK;
}

extern "C" int ts_wpull_src_stage(ts_wpull_src* p, void* stream, int64_t timeout_ms) {
  using namespace tsb::wpull;
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null sender");
  src_join(p);  // the previous generation's groups are all published
  const auto deadline = deadline_in(timeout_ms);
  Box* box = p->box;
  // Every attached receiver has pulled the previous generation before its
  // staging is overwritten.
  const uint64_t prev = p->gen;
  const bool pulled = wait_until(
      [&] {
        const int n = std::min(box->n_receivers.load(std::memory_order_acquire), kMaxReceivers);
        for (int r = 0; r < n; ++r) {
          const uint64_t d = box->done[r].load(std::memory_order_acquire);
          if (d != kDetached && d < prev) return false;
        }
        return true;
      },
      deadline);
  if (!pulled)
    return set_errorf(TS_DEADLINE_EXCEEDED,
                      "a receiver has not finished pulling generation %llu",
                      (unsigned long long)prev);
  tsb::DeviceGuard g(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TS_CUDA_RET(cudaEventRecord(p->start, s), "event record");
  TS_CUDA_RET(cudaStreamWaitEvent(p->stream, p->start, 0), "stream wait");
  for (size_t k = 0; k < p->casts.size(); ++k) {
    const Launch& l = p->casts[k];
    int rc = ts_reshard_copy(p->device, l.d_chunks, l.d_prefix, l.n_chunks, l.n_items,
                             TS_DTYPE_F32, TS_DTYPE_BF16, p->stream);
    if (rc != TS_OK) return rc;
    TS_CUDA_RET(cudaEventRecord(p->cast_done[k], p->stream), "event record");
  }
  TS_CUDA_RET(cudaStreamWaitEvent(s, p->cast_done.back(), 0), "stream wait");
  const uint64_t gen = ++p->gen;
  box->gen.store(gen, std::memory_order_release);
  p->published.store(0);
  p->watch_error.store(0);
  p->watcher = std::thread([p, gen] {
    cudaSetDevice(p->device);
    for (size_t k = 0; k < p->cast_done.size(); ++k) {
      const cudaError_t e = cudaEventSynchronize(p->cast_done[k]);
      if (e != cudaSuccess) {
        p->watch_error.store(int(e));
        return;  // receivers time out on the unpublished groups
      }
      p->box->ready[k].store(gen, std::memory_order_release);
      p->published.fetch_add(1, std::memory_order_release);
    }
  });
  return TS_OK;
}

extern "C" int ts_wpull_src_wait(ts_wpull_src* p, int64_t timeout_ms) {
  using namespace tsb::wpull;
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null sender");
  if (!p->watcher.joinable()) return TS_OK;
  const int n = int(p->cast_done.size());
  const bool ok = wait_until(
      [&] { return p->published.load(std::memory_order_acquire) >= n || p->watch_error.load(); },
      deadline_in(timeout_ms));
  if (!ok) return set_error(TS_DEADLINE_EXCEEDED, "staging not finished within the timeout");
  src_join(p);
  if (const int e = p->watch_error.load())
    return tsb::cuda_error(cudaError_t(e), "pull staging cast");
  return TS_OK;
}

extern "C" int ts_wpull_src_info(ts_wpull_src* p, int64_t* generation, int64_t* groups,
                                 uint64_t* staging_bytes, int64_t* receivers) {
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null sender");
  if (generation) *generation = int64_t(p->gen);
  if (groups) *groups = int64_t(p->casts.size());
  if (staging_bytes) *staging_bytes = p->n_elems * 2;
  if (receivers) *receivers = p->box->n_receivers.load();
  return TS_OK;
}

extern "C" int ts_wpull_src_destroy(ts_wpull_src* p) {
  if (!p) return TS_OK;
  src_release(p);
  return TS_OK;
}

// ---------------------------------------------------------------------------
// Receiver
// ---------------------------------------------------------------------------

struct ts_wpull_dst {
  struct Sender {
    tsb::wpull::Box* box = nullptr;
    void* ipc_base = nullptr;  // mapping to close (other process), or null
    uint64_t staging = 0;      // the staging's address for this device's kernels
    int slot = -1;             // this receiver's slot in the sender's mailbox
    uint64_t base_gen = 0;     // the sender's generation when this receiver attached
  };
  struct Batch {
    int group = 0;
    std::vector<int> senders;  // whose group `group` the batch reads
    tsb::wpull::Launch launch;
  };
  int device = 0;
  std::vector<Sender> senders;
  std::vector<Batch> batches;  // in group order
  cudaStream_t side = nullptr;  // every other batch: a batch's drain overlaps the next
  cudaEvent_t start = nullptr, side_done = nullptr;
  cudaEvent_t done = nullptr;
  std::thread acker;           // acknowledges the last pull once it finished
  uint64_t pulls = 0;
  int64_t launches = 0;
  uint64_t bytes = 0;
};

namespace {

void dst_release(ts_wpull_dst* p) {
  using namespace tsb::wpull;
  if (p->acker.joinable()) p->acker.join();
  tsb::DeviceGuard g(p->device);
  if (p->done) cudaEventSynchronize(p->done);
  if (p->side) cudaStreamSynchronize(p->side);
  for (auto& b : p->batches) free_launch(&b.launch);
  if (p->done) cudaEventDestroy(p->done);
  if (p->start) cudaEventDestroy(p->start);
  if (p->side_done) cudaEventDestroy(p->side_done);
  if (p->side) cudaStreamDestroy(p->side);
  for (auto& s : p->senders) {
    if (s.box && s.slot >= 0) s.box->done[s.slot].store(kDetached, std::memory_order_release);
    if (s.ipc_base) ts_ipc_close(p->device, s.ipc_base);
    if (s.box) munmap(s.box, kBoxBytes);
  }
  delete p;
}

}  // namespace

extern "C" int ts_wpull_dst_create(int device, const char* const* names, int n_src,
                                   const ts_reshard_chunk* chunks, int64_t n_chunks,
                                   ts_wpull_dst** out) {
  using namespace tsb::wpull;
  tsb::clear_error();
  if (!out || !names || n_src <= 0 || n_chunks < 0 || (n_chunks > 0 && !chunks))
    return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  *out = nullptr;
  auto* p = new ts_wpull_dst();
  p->device = device;
  p->senders.resize(size_t(n_src));
  for (int t = 0; t < n_src; ++t) {
    ts_wpull_dst::Sender& s = p->senders[size_t(t)];
    const std::string path = shm_path(names[t]);
    const int fd = shm_open(path.c_str(), O_RDWR, 0);
    if (fd < 0) {
      const int err = errno;
      dst_release(p);
      return set_errorf(TS_NOT_FOUND, "pull mailbox %s: %s", names[t], strerror(err));
    }
    void* m = mmap(nullptr, kBoxBytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (m == MAP_FAILED) {
      const int err = errno;
      dst_release(p);
      return set_errorf(TS_INTERNAL, "pull mailbox map: %s", strerror(err));
    }
    s.box = static_cast<Box*>(m);
    if (reinterpret_cast<std::atomic<uint64_t>*>(&s.box->magic)->load(std::memory_order_acquire) !=
            kMagic ||
        s.box->version != kVersion) {
      dst_release(p);
      return set_errorf(TS_FAILED_PRECONDITION, "%s is not a pull mailbox of this version",
                        names[t]);
    }
    if (s.box->pid == int32_t(getpid())) {
      // a sender in this process: its pointer, with peer access if needed
      if (s.box->device != device) {
        int rc = ts_enable_peer_access(device, s.box->device);
        if (rc != TS_OK) {
          dst_release(p);
          return rc;
        }
      }
      s.staging = s.box->dev_ptr;
    } else {
      int rc = ts_ipc_open(device, s.box->handle, &s.ipc_base);
      if (rc != TS_OK) {
        dst_release(p);
        return rc;
      }
      s.staging = reinterpret_cast<uint64_t>(s.ipc_base) + s.box->offset;
    }
    const int slot = s.box->n_receivers.fetch_add(1, std::memory_order_acq_rel);
    if (slot >= kMaxReceivers) {
      dst_release(p);
      return set_errorf(TS_RESOURCE_EXHAUSTED, "%s has %d receivers already", names[t],
                        kMaxReceivers);
    }
    s.slot = slot;
    s.base_gen = s.box->gen.load(std::memory_order_acquire);
    s.box->done[slot].store(s.base_gen, std::memory_order_release);
  }
  // Every chunk checked against its sender's staging; batched by the last
  // group it reads.
  std::vector<std::vector<ts_reshard_chunk>> by_group(kMaxGroups);
  std::vector<std::vector<int>> need(kMaxGroups);
  for (int64_t i = 0; i < n_chunks; ++i) {
    ts_reshard_chunk c = chunks[i];
    const int64_t t = int64_t(c.src_ptr);
    if (t < 0 || t >= n_src) {
      dst_release(p);
      return set_errorf(TS_INVALID_ARGUMENT, "chunk %lld: sender index %lld out of range",
                        (long long)i, (long long)t);
    }
    if (c.size < 0 || c.count < 0 || c.src_off < 0 || c.dst_off < 0 || c.src_stride < 0 ||
        c.dst_stride < 0) {
      dst_release(p);
      return set_errorf(TS_INVALID_ARGUMENT, "chunk %lld: negative fields", (long long)i);
    }
    if (c.size == 0 || c.count == 0) continue;
    const Box* box = p->senders[size_t(t)].box;
    // one past the last element read, overflow-safe
    const uint64_t rows = uint64_t(c.count - 1);
    const uint64_t n = box->n_elems;
    if (uint64_t(c.size) > n || uint64_t(c.src_off) > n - uint64_t(c.size) ||
        (rows > 0 && uint64_t(c.src_stride) > (n - uint64_t(c.src_off) - uint64_t(c.size)) / rows)) {
      dst_release(p);
      return set_errorf(TS_OUT_OF_RANGE,
                        "chunk %lld reads past the %llu elements of sender %lld's staging",
                        (long long)i, (unsigned long long)n, (long long)t);
    }
    const uint64_t end = uint64_t(c.src_off) + rows * uint64_t(c.src_stride) + uint64_t(c.size);
    // the group holding the last element read
    const uint64_t* gb = box->bounds;
    const int group =
        int(std::upper_bound(gb + 1, gb + box->n_groups + 1, end - 1) - (gb + 1));
    c.src_ptr = p->senders[size_t(t)].staging;
    by_group[size_t(group)].push_back(c);
    auto& nd = need[size_t(group)];
    if (std::find(nd.begin(), nd.end(), int(t)) == nd.end()) nd.push_back(int(t));
    p->bytes += uint64_t(c.size) * uint64_t(c.count) * 2;
  }
  for (int k = 0; k < kMaxGroups; ++k) {
    if (by_group[size_t(k)].empty()) continue;
    ts_wpull_dst::Batch b;
    b.group = k;
    b.senders = need[size_t(k)];
    int rc = upload(device, by_group[size_t(k)], TS_DTYPE_BF16, TS_DTYPE_BF16, &b.launch);
    p->batches.push_back(b);
    if (rc != TS_OK) {
      dst_release(p);
      return rc;
    }
  }
  tsb::DeviceGuard g(device);
  cudaError_t ce = cudaEventCreateWithFlags(&p->done, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->side_done, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&p->side, cudaStreamNonBlocking);
  if (ce != cudaSuccess) {
    dst_release(p);
    return tsb::cuda_error(ce, "pull events");
  }
  *out = p;
  return TS_OK;
}

extern "C" int ts_wpull_dst_pull(ts_wpull_dst* p, void* stream, int64_t timeout_ms) {
  using namespace tsb::wpull;
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null receiver");
  if (p->acker.joinable()) p->acker.join();  // the previous pull is acknowledged
  const auto deadline = deadline_in(timeout_ms);
  const uint64_t k = ++p->pulls;
  tsb::DeviceGuard g(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // Batches alternate between the caller's stream and a side stream ordered
  // after it (their destinations are disjoint): one batch's last CTAs drain
  // while the next batch's start.
  TS_CUDA_RET(cudaEventRecord(p->start, s), "event record");
  TS_CUDA_RET(cudaStreamWaitEvent(p->side, p->start, 0), "stream wait");
  size_t nb = 0;
  for (const auto& b : p->batches) {
    const bool ready = wait_until(
        [&] {
          for (int t : b.senders) {
            const auto& snd = p->senders[size_t(t)];
            if (snd.box->ready[b.group].load(std::memory_order_acquire) < snd.base_gen + k)
              return false;
          }
          return true;
        },
        deadline);
    if (!ready)
      return set_errorf(TS_DEADLINE_EXCEEDED,
                        "group %d of generation %llu not published within the timeout",
                        b.group, (unsigned long long)k);
    int rc = ts_reshard_copy(p->device, b.launch.d_chunks, b.launch.d_prefix, b.launch.n_chunks,
                             b.launch.n_items, TS_DTYPE_BF16, TS_DTYPE_BF16,
                             (nb++ & 1) ? p->side : s);
    if (rc != TS_OK) return rc;
    ++p->launches;
  }
  TS_CUDA_RET(cudaEventRecord(p->side_done, p->side), "event record");
  TS_CUDA_RET(cudaStreamWaitEvent(s, p->side_done, 0), "stream wait");
  TS_CUDA_RET(cudaEventRecord(p->done, s), "event record");
  p->acker = std::thread([p, k] {
    cudaSetDevice(p->device);
    if (cudaEventSynchronize(p->done) != cudaSuccess) return;  // senders time out
    for (auto& snd : p->senders)
      snd.box->done[snd.slot].store(snd.base_gen + k, std::memory_order_release);
  });
  return TS_OK;
}

extern "C" int ts_wpull_dst_info(ts_wpull_dst* p, int64_t* generation, int64_t* launches,
                                 uint64_t* bytes) {
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null receiver");
  if (generation) *generation = int64_t(p->pulls);
  if (launches) *launches = int64_t(p->batches.size());
  if (bytes) *bytes = p->bytes;
  return TS_OK;
}

extern "C" int ts_wpull_dst_destroy(ts_wpull_dst* p) {
  if (!p) return TS_OK;
  dst_release(p);
  return TS_OK;
}

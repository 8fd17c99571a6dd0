// KV cache manager: the device path of KVCacheManagerBase on one B200.
//
// Reference behaviour kept (tpu_sync/kv_cache/kv_cache_manager_base.cc):
//  * storages are a [layer][shard] grid of device buffers whose dim-0 slices
//    are blocks; block bytes of layer l = physical_size(l) / dim0(layer 0)
//    (layer_block_byte_size, kv_cache_manager_base.h:434-439);
//  * D2h/H2d take block-unit (src, dst, size) lists, validated
//    (ValidateOffsetsAndSizes :72-102), coalesced (:121-141), bounds-checked
//    per storage and run in (layer, shard, run) order with the reference's
//    codes and messages (:1994-2012, :2089-2103), and an empty list means
//    "whole storage" (:1984-1993, :2078-2088);
//  * optional layer / shard restriction (:540-545);
//  * a future per call (PjRtCopyFuture -> ts_event).
//
// B200 design:
//  * the host tier is block-major: host block h holds block h of every
//    storage contiguously (pitch = sum of block bytes), so a KV block of all
//    layers is one contiguous host range and one DMA;
//  * offload = extract kernel (HBM pages -> HBM staging slot, block-major)
//    on a kernel stream, then copy-engine D2H DMAs of whole host blocks on a
//    copy stream; reload = H2D DMAs into a staging slot, then the insert
//    kernel.  Two staging slots per direction double-buffer chunks of up to
//    kMaxParamIds blocks, so the next chunk's gather overlaps the current
//    chunk's DMA, and offload and reload use separate slots and streams so
//    both PCIe directions run at once;
//  * block-level hazard tracking orders a reload after an in-flight offload
//    of the same host/device blocks (and vice versa) without serialising
//    independent calls.

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <deque>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "pool_layout.h"
#include "ts_internal.h"

struct ts_host_tier;

namespace tsb {
namespace {

constexpr int kMaxCopyStreams = 4;
constexpr int kEventRing = 256;
constexpr int kErrWords = 4096;

struct Storage {
  uint64_t dev_ptr = 0;
  uint64_t nbytes = 0;
  int64_t dim0 = 0;
  uint64_t bb = 0;        // layer_block_byte_size
  uint64_t host_off = 0;  // offset inside a host block (and a staging block)
  uint64_t host_bytes = 0;  // bytes of this storage in one host block
};

struct Slot {
  uint8_t* buf = nullptr;
  cudaEvent_t ready = nullptr;
  cudaEvent_t free = nullptr;
};

// Completion record of one call, kept so later calls can wait on it: the
// whole call, and each pipelined chunk of a whole-block call (chunk_ev[c]
// completes once chunk c's blocks have been read and written).
struct CallRec {
  uint64_t seq = 0;
  cudaEvent_t done = nullptr;
  std::vector<cudaEvent_t> chunk_ev;
};

}  // namespace
}  // namespace tsb

struct ts_manager;

struct ts_event {
  ts_manager* mgr = nullptr;
  int device = 0;
  cudaEvent_t start = nullptr;
  cudaEvent_t done = nullptr;
  int* err_word = nullptr;  // mapped pinned int (host view)
  int err_index = -1;
  bool finished = false;
  int status = TS_PENDING;
  std::string message;
};

struct ts_manager {
  int device = 0;
  int num_layers = 0;
  int num_shards = 0;
  int64_t major_dim = 0;
  uint64_t bytes_per_block = 0;  // slice byte size of layer 0 (reference bytes_per_block)
  std::vector<tsb::Storage> st;
  int64_t host_blocks = 0;
  uint64_t host_pitch = 0;
  uint64_t scale_off = 0;  // fp8: offset of the per-storage scales in a block
  bool fp8 = false;
  ts_host_tier* tier = nullptr;
  uint8_t* host = nullptr;

  ts_block_storage* d_table = nullptr;
  bool vec_ok = true;
  bool wide_ok = false;  // every storage, slot and the host tier 32-byte aligned
  int numa_node = -1;    // assigned NUMA node (-1: none known)
  bool numa_placed = false;
  uint64_t max_bb = 0;
  int64_t chunk_blocks = 64;

  int mode = 0;       // bit 0: offload direct, bit 1: reload direct (else staged)
  int ncs = 2;        // copy streams per direction (staged)
  int max_ctas = 0;   // grid cap of the kernels
  int reload_staged_every = 0;  // direct reloads: every n-th chunk staged (0 = none)
  int sched = 0;                // TS_SCHED_* flags
  uint8_t* host_dev = nullptr;  // device address of the mapped host tier

  cudaStream_t s_out_kernel = nullptr, s_in_kernel = nullptr;
  cudaStream_t s_in_kernel2 = nullptr;  // second reload kernel stream (overlap)
  cudaEvent_t in_join = nullptr;
  cudaStream_t out_cs[tsb::kMaxCopyStreams] = {};
  cudaStream_t in_cs[tsb::kMaxCopyStreams] = {};
  cudaEvent_t out_join[tsb::kMaxCopyStreams] = {};
  cudaEvent_t ev_user = nullptr;
  std::vector<tsb::Slot> out_slots, in_slots;
  int next_out = 0, next_in = 0;

  // hazard tracking: sequence numbers of the last offload (d2h) / reload
  // (h2d) call touching each host block and device block.
  std::vector<uint64_t> host_d2h_seq, host_h2d_seq, dev_d2h_seq, dev_h2d_seq;
  // ... and the chunk of that call which moved the block (-1: not chunked)
  std::vector<int32_t> host_d2h_chunk, host_h2d_chunk, dev_d2h_chunk, dev_h2d_chunk;
  uint64_t d2h_seq = 0, h2d_seq = 0;
  tsb::CallRec d2h_ring[tsb::kEventRing];
  tsb::CallRec h2d_ring[tsb::kEventRing];

  // optional per-launch timing of the extract (0) / insert (1) kernels
  bool profiling = false;
  std::vector<cudaEvent_t> prof_ev[2];  // start/stop pairs, in launch order
  std::vector<uint64_t> prof_bytes[2];
  std::vector<cudaEvent_t> prof_free;

  // mapped pinned error words, one per outstanding event
  int* err_host = nullptr;
  std::vector<int> err_free;

  // explicit pools (RegisterPools); empty / false = implicit pools
  std::vector<tsb::pool::Pool> pools;
  bool explicit_pools = false;

  std::mutex mu;
  // 1 for the owner + 1 per live event; the struct (its mutex and error
  // words) is freed when the last reference goes, so events released after
  // ts_mgr_destroy stay valid.
  std::atomic<int> refs{1};
  bool closed = false;
};

namespace tsb {
namespace {

// Returns the index of a free error word, or -1 (error recorded).
int alloc_err_word(ts_manager* m, int** word) {
  if (m->err_free.empty()) {
    set_error(TS_RESOURCE_EXHAUSTED, "too many outstanding transfer events");
    return -1;
  }
  const int i = m->err_free.back();
  m->err_free.pop_back();
  m->err_host[i] = 0;
  *word = m->err_host + i;
  return i;
}

uint64_t round16(uint64_t v) { return (v + 15) & ~uint64_t(15); }

// Waits (on `stream`) for the call `seq` of the ring if it may still run.
int wait_for_call(CallRec* ring, uint64_t seq, cudaStream_t stream) {
  if (seq == 0) return TS_OK;
  CallRec& r = ring[seq % kEventRing];
  if (r.seq != seq || r.done == nullptr) return TS_OK;  // recycled => long done
  TS_CUDA_RET(cudaStreamWaitEvent(stream, r.done, 0), "cross-direction ordering");
  return TS_OK;
}

int record_call(CallRec* ring, uint64_t seq, cudaStream_t stream) {
  CallRec& r = ring[seq % kEventRing];
  if (r.done == nullptr) {
    TS_CUDA_RET(cudaEventCreateWithFlags(&r.done, cudaEventDisableTiming), "event create");
  } else if (r.seq != 0) {
    // The slot's previous call is kEventRing calls old; make sure it is done
    // before its record is dropped (later calls may no longer wait on it).
    TS_CUDA_RET(cudaEventSynchronize(r.done), "event ring recycle");
  }
  r.seq = seq;
  TS_CUDA_RET(cudaEventRecord(r.done, stream), "event record");
  return TS_OK;
}

// One strided DMA between a device storage and its host mirror.
struct DmaRun {
  uint64_t dev, host;  // host: pinned host address
  uint64_t width, dev_pitch, host_pitch, rows;
};

struct Plan {
  std::vector<int> storages;  // storage indices touched
  std::vector<int64_t> src, dst;  // per-block ids (hazard tracking for pool copies)
  bool whole = false;             // all storages of the grid
  // pool copies: the byte work itself, already oriented for the direction
  bool pool = false;
  std::vector<DmaRun> dma;
  std::vector<SegTask> seg;
};

// Validation, coalescing and bounds checks in the reference's order.
// `to_host` = D2H direction.
int build_plan(ts_manager* m, bool to_host, const int64_t* src, const int64_t* dst,
               const int64_t* sizes, int64_t n_src, int64_t n_dst, int64_t n_sizes,
               int64_t layer_idx, int64_t shard_idx, Plan* plan) {
  int rc = ts_validate_copy_spec(src, n_src, dst, n_dst, sizes, n_sizes);
  if (rc != TS_OK) return rc;
  if (n_src > 0 && n_dst == 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "src_offsets, dst_offsets, and sizes must have the same length");
  if (layer_idx >= m->num_layers || shard_idx >= m->num_shards)
    return set_error(TS_OUT_OF_RANGE, "layer or shard index out of range");
  std::vector<int64_t> ones;
  if (n_src > 0 && n_sizes == 0) {
    ones.assign(size_t(n_src), 1);
    sizes = ones.data();
  }
  std::vector<int64_t> cs(n_src), cd(n_src), cn(n_src);
  int64_t runs = 0;
  ts_coalesce_runs(src, dst, sizes, n_src, cs.data(), cd.data(), cn.data(), &runs);
  const bool partial = runs > 0;

  plan->storages.clear();
  for (int l = 0; l < m->num_layers; ++l) {
    if (layer_idx >= 0 && l != layer_idx) continue;
    for (int s = 0; s < m->num_shards; ++s) {
      if (shard_idx >= 0 && s != shard_idx) continue;
      plan->storages.push_back(l * m->num_shards + s);
    }
  }
  plan->whole = int(plan->storages.size()) == int(m->st.size());
  if (!plan->whole && m->fp8)
    return set_error(TS_UNIMPLEMENTED,
                     "layer / shard restricted copies are not supported on an fp8 host tier");

  // Reference host mirror size per storage: host_blocks * bytes_per_block().
  const int64_t ref_host_size = m->host_blocks * int64_t(m->bytes_per_block);
  for (int si : plan->storages) {
    const Storage& sd = m->st[si];
    const int64_t bb = int64_t(sd.bb);
    if (!partial) {
      // whole-storage copy: physical size against the host mirror
      if (int64_t(sd.nbytes) > ref_host_size ||
          (bb > 0 && int64_t(sd.nbytes) / bb > m->host_blocks)) {
        if (to_host)
          return set_error(TS_OUT_OF_RANGE, "Copy range exceeds destination host buffer size");
        return set_error(TS_INVALID_ARGUMENT, "Source host buffer is too small");
      }
      continue;
    }
    for (int64_t r = 0; r < runs; ++r) {
      const int64_t so = cs[r] * bb, dof = cd[r] * bb, n = cn[r] * bb;
      const int64_t host_id_end = (to_host ? cd[r] : cs[r]) + cn[r];
      if (to_host) {
        if (so + n > int64_t(sd.nbytes))
          return set_error(TS_INVALID_ARGUMENT, "Copy range exceeds source device buffer size");
        if (dof + n > ref_host_size || host_id_end > m->host_blocks)
          return set_error(TS_INVALID_ARGUMENT, "Copy range exceeds destination host buffer size");
      } else {
        if (so + n > ref_host_size || host_id_end > m->host_blocks)
          return set_error(TS_INVALID_ARGUMENT, "Copy range exceeds source host buffer size");
        if (dof + n > int64_t(sd.nbytes))
          return set_error(TS_INVALID_ARGUMENT, "Copy range exceeds destination device buffer size");
      }
    }
  }

  plan->src.clear();
  plan->dst.clear();
  if (!partial) {
    // Whole storages: every block of the largest storage (the kernels skip
    // ids past a smaller storage's end only when they are out of its bounds,
    // so restrict to the common block count).
    int64_t nb = INT64_MAX;
    for (int si : plan->storages) {
      const Storage& sd = m->st[si];
      nb = std::min<int64_t>(nb, sd.bb ? int64_t(sd.nbytes / sd.bb) : 0);
    }
    if (nb == INT64_MAX) nb = 0;
    for (int64_t b = 0; b < nb; ++b) {
      plan->src.push_back(b);
      plan->dst.push_back(b);
    }
  } else {
    for (int64_t r = 0; r < runs; ++r)
      for (int64_t j = 0; j < cn[r]; ++j) {
        plan->src.push_back(cs[r] + j);
        plan->dst.push_back(cd[r] + j);
      }
    // A destination block named more than once ends with the last copy's
    // bytes: the reference copies run by run, in order
    // (kv_cache_manager_base.cc:1945-2124), and nothing reads a destination
    // within one call.  The earlier copies to such a block are dropped, so no
    // kernel launch or DMA ever has two writers of one block (the pieces of
    // one chunk run concurrently).
    std::unordered_set<int64_t> seen;
    bool repeats = false;
    for (int64_t d : plan->dst)
      if (!seen.insert(d).second) { repeats = true; break; }
    if (repeats) {
      seen.clear();
      std::vector<int64_t> ks, kd;
      for (size_t i = plan->dst.size(); i-- > 0;)
        if (seen.insert(plan->dst[i]).second) {
          ks.push_back(plan->src[i]);
          kd.push_back(plan->dst[i]);
        }
      std::reverse(ks.begin(), ks.end());
      std::reverse(kd.begin(), kd.end());
      plan->src.swap(ks);
      plan->dst.swap(kd);
    }
  }
  return TS_OK;
}

void unref_manager(ts_manager* m) {
  if (m->refs.fetch_sub(1) == 1) {
    if (m->err_host) cudaFreeHost(m->err_host);
    delete m;
  }
}

// Frees an event whose work has drained, with the manager lock held (the
// owner's reference is still held, so this never frees the manager).
void drop_event_locked(ts_event* ev) {
  if (ev->err_index >= 0) ev->mgr->err_free.push_back(ev->err_index);
  cudaEventDestroy(ev->start);
  cudaEventDestroy(ev->done);
  ev->mgr->refs.fetch_sub(1);
  delete ev;
}

int make_event(ts_manager* m, ts_event** out) {
  auto* ev = new ts_event();
  ev->mgr = m;
  ev->device = m->device;
  cudaError_t e = cudaEventCreate(&ev->start);
  if (e == cudaSuccess) e = cudaEventCreate(&ev->done);
  if (e != cudaSuccess) {
    delete ev;
    return cuda_error(e, "event create");
  }
  const int idx = alloc_err_word(m, &ev->err_word);
  if (idx < 0) {
    cudaEventDestroy(ev->start);
    cudaEventDestroy(ev->done);
    delete ev;
    return TS_RESOURCE_EXHAUSTED;
  }
  ev->err_index = idx;
  m->refs.fetch_add(1);
  *out = ev;
  return TS_OK;
}

// Storage-subset copies (layer / shard restricted): one strided 2-D DMA per
// run between the device storage and that storage's slot in the host blocks.
int enqueue_subset(ts_manager* m, bool to_host, const Plan& p, cudaStream_t s) {
  for (int si : p.storages) {
    const Storage& sd = m->st[si];
    size_t i = 0;
    while (i < p.src.size()) {
      size_t j = i + 1;
      while (j < p.src.size() && p.src[j] == p.src[j - 1] + 1 && p.dst[j] == p.dst[j - 1] + 1) ++j;
      const int64_t n = int64_t(j - i);
      const int64_t dev_id = to_host ? p.src[i] : p.dst[i];
      const int64_t host_id = to_host ? p.dst[i] : p.src[i];
      uint8_t* dev = reinterpret_cast<uint8_t*>(sd.dev_ptr) + uint64_t(dev_id) * sd.bb;
      uint8_t* host = m->host + uint64_t(host_id) * m->host_pitch + sd.host_off;
      if (to_host) {
        TS_CUDA_RET(cudaMemcpy2DAsync(host, m->host_pitch, dev, sd.bb, sd.bb, size_t(n),
                                      cudaMemcpyDeviceToHost, s),
                    "D2H storage copy");
      } else {
        TS_CUDA_RET(cudaMemcpy2DAsync(dev, sd.bb, host, m->host_pitch, sd.bb, size_t(n),
                                      cudaMemcpyHostToDevice, s),
                    "H2D storage copy");
      }
      i = j;
    }
  }
  return TS_OK;
}

// Pool copies: whole aligned blocks as strided DMAs, partial live regions
// with one segment-copy kernel reading / writing the mapped host tier.
int enqueue_pool(ts_manager* m, bool to_host, const Plan& p, cudaStream_t s) {
  for (const DmaRun& r : p.dma) {
    void* dev = reinterpret_cast<void*>(r.dev);
    void* host = reinterpret_cast<void*>(r.host);
    if (to_host) {
      TS_CUDA_RET(cudaMemcpy2DAsync(host, r.host_pitch, dev, r.dev_pitch, r.width, r.rows,
                                    cudaMemcpyDeviceToHost, s),
                  "D2H pool block copy");
    } else {
      TS_CUDA_RET(cudaMemcpy2DAsync(dev, r.dev_pitch, host, r.host_pitch, r.width, r.rows,
                                    cudaMemcpyHostToDevice, s),
                  "H2D pool block copy");
    }
  }
  return seg_copy(m->device, p.seg.data(), int64_t(p.seg.size()), s, m->max_ctas);
}

cudaEvent_t prof_event(ts_manager* m) {
  if (!m->prof_free.empty()) {
    cudaEvent_t e = m->prof_free.back();
    m->prof_free.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Algorithmic HBM bytes of one kernel launch over `cn` blocks.
uint64_t kernel_bytes(const ts_manager* m, int64_t cn, bool extract) {
  uint64_t dev = 0, stage = 0;
  for (const Storage& s : m->st) {
    dev += s.bb;
    stage += s.host_bytes;
  }
  if (m->fp8) stage += 4 * m->st.size();
  (void)extract;
  return uint64_t(cn) * (dev + stage);
}

bool is_direct(const ts_manager* m, bool to_host) {
  return (m->mode & (to_host ? 1 : 2)) != 0;
}

// The stream on which every call of a direction completes.
cudaStream_t last_stream(const ts_manager* m, bool to_host) {
  if (!to_host) return m->s_in_kernel;
  return is_direct(m, true) ? m->s_out_kernel : m->out_cs[0];
}

int launch_chunk(ts_manager* m, bool to_host, const ParamIds& ids, int64_t cn,
                 void* staging, int* err_dev, cudaStream_t ks) {
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (m->profiling) {
    e0 = prof_event(m);
    e1 = prof_event(m);
    TS_CUDA_RET(cudaEventRecord(e0, ks), "event record");
  }
  // A direct reload waits on PCIe for its whole chunk; launched one CTA per
  // piece its CTAs retire as pieces land, so other kernels get SM slots.
  const int ctas = !to_host && ids.direct && (m->sched & TS_SCHED_RELOAD_PER_PIECE) != 0
                       ? -1 : m->max_ctas;
  // bulk copies only between device buffers (staged chunks)
  const int variant = !ids.direct && (m->sched & TS_SCHED_BULK_COPY) != 0 ? kCopyBulk
                      : ids.direct && m->wide_ok && (m->sched & TS_SCHED_WIDE_LOADS) != 0
                          ? kCopyWide : kCopyVec;
  int rc = to_host
               ? mgr_extract(m->device, m->d_table, int(m->st.size()), ids, cn, staging,
                             m->host_pitch, err_dev, ks, m->vec_ok, m->max_bb, m->fp8,
                             m->scale_off, m->max_ctas, variant)
               : mgr_insert(m->device, m->d_table, int(m->st.size()), ids, cn, staging,
                            m->host_pitch, err_dev, ks, m->vec_ok, m->max_bb, m->fp8,
                            m->scale_off, ctas, variant);
  if (rc != TS_OK) return rc;
  if (m->profiling) {
    TS_CUDA_RET(cudaEventRecord(e1, ks), "event record");
    const int w = to_host ? 0 : 1;
    m->prof_ev[w].push_back(e0);
    m->prof_ev[w].push_back(e1);
    m->prof_bytes[w].push_back(kernel_bytes(m, cn, to_host));
  }
  return TS_OK;
}

// `seq` is the sequence number this call will get; chunk_of[i] receives the
// pipelined chunk that moves block i of the plan (-1 when not chunked).
int enqueue_transfer(ts_manager* m, bool to_host, const Plan& p, void* user_stream,
                     ts_event* ev, uint64_t seq, std::vector<int32_t>* chunk_of) {
  cudaStream_t user = reinterpret_cast<cudaStream_t>(user_stream);
  cudaStream_t ks = to_host ? m->s_out_kernel : m->s_in_kernel;
  cudaStream_t* cs = to_host ? m->out_cs : m->in_cs;
  const bool direct = is_direct(m, to_host) && p.whole;
  // direct reloads may route every n-th chunk through the copy engines
  const int staged_every = to_host ? 0 : m->reload_staged_every;
  const cudaStream_t last = last_stream(m, to_host);
  std::vector<cudaStream_t> streams{ks};
  if (!is_direct(m, to_host) || staged_every > 0)
    for (int i = 0; i < m->ncs; ++i) streams.push_back(cs[i]);
  cudaStream_t ks2 = !to_host && direct ? m->s_in_kernel2 : nullptr;
  if (ks2 != nullptr) streams.push_back(ks2);
  int* err_dev = nullptr;
  TS_CUDA_RET(cudaHostGetDevicePointer(reinterpret_cast<void**>(&err_dev), ev->err_word, 0),
              "error word mapping");

  // Order after the producer's queued work.
  TS_CUDA_RET(cudaEventRecord(m->ev_user, user), "event record");
  for (cudaStream_t s : streams)
    TS_CUDA_RET(cudaStreamWaitEvent(s, m->ev_user, 0), "stream wait");

  // Cross-direction hazards, per block: the latest in-flight call of the
  // other direction that wrote what this call reads (or reads what it
  // writes).  Independent blocks go first; dependent ones follow in order of
  // the call they wait for, and each chunk waits only for what its own
  // blocks need, so a few conflicting blocks do not hold back the rest.
  CallRec* ring = to_host ? m->h2d_ring : m->d2h_ring;
  const size_t nb = p.src.size();
  chunk_of->assign(nb, -1);
  // This call's own record: its previous user (kEventRing calls ago) is
  // drained first, and until this call is recorded nothing may name it.
  CallRec& own = (to_host ? m->d2h_ring : m->h2d_ring)[seq % kEventRing];
  if (own.seq != 0 && own.done != nullptr)
    TS_CUDA_RET(cudaEventSynchronize(own.done), "event ring recycle");
  own.seq = 0;
  std::vector<uint64_t> need(nb, 0);
  // the (call, chunk) pairs each block waits for (seq 0 = none)
  struct Dep {
    uint64_t seq = 0;
    int32_t chunk = -1;
  };
  std::vector<Dep> dep_a(nb), dep_b(nb);
  std::unordered_map<uint64_t, bool> finished;
  auto still_running = [&](uint64_t seq) {
    if (seq == 0) return false;
    auto it = finished.find(seq);
    if (it != finished.end()) return !it->second;
    const CallRec& r = ring[seq % kEventRing];
    const bool done = r.seq != seq || r.done == nullptr || cudaEventQuery(r.done) == cudaSuccess;
    finished.emplace(seq, done);
    return !done;
  };
  for (size_t i = 0; i < nb; ++i) {
    const size_t si = size_t(p.src[i]), di = size_t(p.dst[i]);
    const uint64_t a = to_host ? m->dev_h2d_seq[si] : m->host_d2h_seq[si];
    const uint64_t b = to_host ? m->host_h2d_seq[di] : m->dev_d2h_seq[di];
    if (still_running(a)) dep_a[i] = {a, to_host ? m->dev_h2d_chunk[si] : m->host_d2h_chunk[si]};
    if (still_running(b)) dep_b[i] = {b, to_host ? m->host_h2d_chunk[di] : m->dev_d2h_chunk[di]};
    need[i] = std::max(dep_a[i].seq, dep_b[i].seq);
  }
  cudaGetLastError();  // cudaEventQuery's "not ready" is not an error
  std::vector<size_t> order(nb);
  for (size_t i = 0; i < nb; ++i) order[i] = i;
  bool dup_dst = false;
  {
    std::unordered_set<int64_t> seen;
    for (int64_t d : p.dst)
      if (!seen.insert(d).second) { dup_dst = true; break; }
  }
  if (!dup_dst)  // reordering is only safe when no destination repeats
    std::stable_sort(order.begin(), order.end(),
                     [&](size_t a, size_t b) { return need[a] < need[b]; });
  uint64_t waited = 0;
  auto wait_upto = [&](uint64_t seq) -> int {
    if (seq <= waited) return TS_OK;
    for (cudaStream_t s : streams) {
      int rc = wait_for_call(ring, seq, s);
      if (rc != TS_OK) return rc;
    }
    waited = seq;
    return TS_OK;
  };
  if (dup_dst || !p.whole) {
    uint64_t all = 0;
    for (uint64_t x : need) all = std::max(all, x);
    int rc = wait_upto(all);
    if (rc != TS_OK) return rc;
  }
  TS_CUDA_RET(cudaEventRecord(ev->start, ks), "event record");

  if (!p.whole) {
    int rc = p.pool ? enqueue_pool(m, to_host, p, last) : enqueue_subset(m, to_host, p, last);
    if (rc != TS_OK) return rc;
    TS_CUDA_RET(cudaEventRecord(ev->done, last), "event record");
    return TS_OK;
  }

  const int64_t nblk = int64_t(nb);
  std::vector<int64_t> dev_ids(nb), host_ids(nb);
  for (size_t k = 0; k < nb; ++k) {
    const size_t i = order[k];
    dev_ids[k] = to_host ? p.src[i] : p.dst[i];
    host_ids[k] = to_host ? p.dst[i] : p.src[i];
    (*chunk_of)[i] = int32_t(int64_t(k) / m->chunk_blocks);
  }
  // A chunk waits for the chunks of other calls that moved its blocks (or
  // for a whole call when that call was not chunked).
  std::set<std::pair<uint64_t, int32_t>> waited_chunks;
  auto wait_chunk_deps = [&](int64_t c0, int64_t cn) -> int {
    for (int64_t k = c0; k < c0 + cn; ++k) {
      for (const Dep& d : {dep_a[order[size_t(k)]], dep_b[order[size_t(k)]]}) {
        if (d.seq == 0 || d.seq <= waited) continue;
        const CallRec& r = ring[d.seq % kEventRing];
        if (r.seq != d.seq) continue;  // recycled => long done
        if (d.chunk < 0 || size_t(d.chunk) >= r.chunk_ev.size()) {
          int rc = wait_upto(d.seq);
          if (rc != TS_OK) return rc;
          continue;
        }
        if (!waited_chunks.insert({d.seq, d.chunk}).second) continue;
        for (cudaStream_t s : streams)
          TS_CUDA_RET(cudaStreamWaitEvent(s, r.chunk_ev[size_t(d.chunk)], 0),
                      "cross-direction ordering");
      }
    }
    return TS_OK;
  };
  auto record_chunk = [&](int64_t ci, cudaStream_t s) -> int {
    while (own.chunk_ev.size() <= size_t(ci)) {
      cudaEvent_t e = nullptr;
      TS_CUDA_RET(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event create");
      own.chunk_ev.push_back(e);
    }
    TS_CUDA_RET(cudaEventRecord(own.chunk_ev[size_t(ci)], s), "event record");
    return TS_OK;
  };
  std::vector<Slot>& slots = to_host ? m->out_slots : m->in_slots;
  int& next = to_host ? m->next_out : m->next_in;
  int chunk = 0;  // staged chunks issued (copy stream rotation)
  int64_t ci = 0;
  // Direct reload chunks alternate between two kernel streams (their
  // destinations are distinct, so they may run concurrently).
  const bool overlap = ks2 != nullptr && !dup_dst;
  int n_direct = 0;
  bool used_ks2 = false;
  for (int64_t c0 = 0; c0 < nblk; c0 += m->chunk_blocks, ++ci) {
    const int64_t cn = std::min<int64_t>(m->chunk_blocks, nblk - c0);
    int rc0 = wait_chunk_deps(c0, cn);
    if (rc0 != TS_OK) return rc0;
    if (direct && !(staged_every > 0 && ci % staged_every == staged_every - 1)) {
      // the kernel moves the chunk over PCIe itself (mapped host tier)
      ParamIds ids;
      ids.direct = 1;
      for (int64_t k = 0; k < cn; ++k) {
        ids.v[k] = dev_ids[size_t(c0 + k)];
        ids.s[k] = host_ids[size_t(c0 + k)];
      }
      cudaStream_t kc = overlap && (n_direct++ & 1) ? ks2 : ks;
      used_ks2 = used_ks2 || kc == ks2;
      int rc = launch_chunk(m, to_host, ids, cn, m->host_dev, err_dev, kc);
      if (rc == TS_OK) rc = record_chunk(ci, kc);
      if (rc != TS_OK) return rc;
      continue;
    }
    ++chunk;
    Slot& slot = slots[size_t(next)];
    next = (next + 1) % int(slots.size());
    // a repeated destination keeps every DMA on one copy stream, so the
    // later copy lands last
    cudaStream_t cc = dup_dst ? cs[0] : cs[(chunk - 1) % m->ncs];
    ParamIds ids;
    ids.direct = 0;
    for (int64_t k = 0; k < cn; ++k) ids.v[k] = dev_ids[size_t(c0 + k)];
    if (to_host) {
      TS_CUDA_RET(cudaStreamWaitEvent(ks, slot.free, 0), "stream wait");
      int rc = launch_chunk(m, true, ids, cn, slot.buf, err_dev, ks);
      if (rc != TS_OK) return rc;
      TS_CUDA_RET(cudaEventRecord(slot.ready, ks), "event record");
      TS_CUDA_RET(cudaStreamWaitEvent(cc, slot.ready, 0), "stream wait");
    } else {
      TS_CUDA_RET(cudaStreamWaitEvent(cc, slot.free, 0), "stream wait");
    }
    // one DMA per maximal run of consecutive host block ids
    int64_t k = 0;
    while (k < cn) {
      int64_t e = k + 1;
      while (e < cn && host_ids[size_t(c0 + e)] == host_ids[size_t(c0 + e - 1)] + 1) ++e;
      uint8_t* h = m->host + uint64_t(host_ids[size_t(c0 + k)]) * m->host_pitch;
      uint8_t* d = slot.buf + uint64_t(k) * m->host_pitch;
      const size_t bytes = size_t(e - k) * m->host_pitch;
      if (to_host) {
        TS_CUDA_RET(cudaMemcpyAsync(h, d, bytes, cudaMemcpyDeviceToHost, cc), "D2H DMA");
      } else {
        TS_CUDA_RET(cudaMemcpyAsync(d, h, bytes, cudaMemcpyHostToDevice, cc), "H2D DMA");
      }
      k = e;
    }
    if (to_host) {
      TS_CUDA_RET(cudaEventRecord(slot.free, cc), "event record");
      int rc = record_chunk(ci, cc);
      if (rc != TS_OK) return rc;
    } else {
      TS_CUDA_RET(cudaEventRecord(slot.ready, cc), "event record");
      TS_CUDA_RET(cudaStreamWaitEvent(ks, slot.ready, 0), "stream wait");
      int rc = launch_chunk(m, false, ids, cn, slot.buf, err_dev, ks);
      if (rc != TS_OK) return rc;
      TS_CUDA_RET(cudaEventRecord(slot.free, ks), "event record");
      rc = record_chunk(ci, ks);
      if (rc != TS_OK) return rc;
    }
  }
  if (to_host) {  // join the other copy streams into the completing one
    for (int i = 1; i < m->ncs && i < chunk; ++i) {
      TS_CUDA_RET(cudaEventRecord(m->out_join[i], cs[i]), "event record");
      TS_CUDA_RET(cudaStreamWaitEvent(last, m->out_join[i], 0), "stream wait");
    }
  }
  if (used_ks2) {
    TS_CUDA_RET(cudaEventRecord(m->in_join, ks2), "event record");
    TS_CUDA_RET(cudaStreamWaitEvent(last, m->in_join, 0), "stream wait");
  }
  TS_CUDA_RET(cudaEventRecord(ev->done, last), "event record");
  return TS_OK;
}

void sync_all(ts_manager* m) {
  for (cudaStream_t s : {m->s_out_kernel, m->s_in_kernel, m->s_in_kernel2})
    if (s) cudaStreamSynchronize(s);
  for (int i = 0; i < kMaxCopyStreams; ++i) {
    if (m->out_cs[i]) cudaStreamSynchronize(m->out_cs[i]);
    if (m->in_cs[i]) cudaStreamSynchronize(m->in_cs[i]);
  }
}

int submit_locked(ts_manager* m, bool to_host, const Plan& p, void* stream, ts_event** out);

int transfer(ts_manager* m, bool to_host, const int64_t* src, const int64_t* dst,
             const int64_t* sizes, int64_t n_src, int64_t n_dst, int64_t n_sizes,
             int64_t layer_idx, int64_t shard_idx, void* stream, ts_event** out) {
  clear_error();
  if (!m || !out) return set_error(TS_INVALID_ARGUMENT, "null manager or output");
  *out = nullptr;
  Plan p;
  int rc = build_plan(m, to_host, src, dst, sizes, n_src, n_dst, n_sizes, layer_idx,
                      shard_idx, &p);
  if (rc != TS_OK) return rc;
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->closed) return set_error(TS_FAILED_PRECONDITION, "manager already destroyed");
  return submit_locked(m, to_host, p, stream, out);
}

// Queues a planned transfer (manager lock held): event, hazard waits, the
// copies, and the per-block hazard bookkeeping.
int submit_locked(ts_manager* m, bool to_host, const Plan& p, void* stream, ts_event** out) {
  DeviceGuard g(m->device);
  ts_event* ev = nullptr;
  int rc = make_event(m, &ev);
  if (rc != TS_OK) return rc;
  const uint64_t seq = (to_host ? m->d2h_seq : m->h2d_seq) + 1;
  std::vector<int32_t> chunk_of;
  rc = enqueue_transfer(m, to_host, p, stream, ev, seq, &chunk_of);
  if (rc != TS_OK) {
    // Work already queued stays ordered on the manager's streams; drain it so
    // the error word can be recycled safely.
    sync_all(m);
    std::string msg = ts_last_error();
    drop_event_locked(ev);
    return set_error(rc, msg);
  }
  cudaStream_t last = last_stream(m, to_host);
  (to_host ? m->d2h_seq : m->h2d_seq) = seq;
  rc = record_call(to_host ? m->d2h_ring : m->h2d_ring, seq, last);
  if (rc != TS_OK) {
    cudaEventSynchronize(ev->done);
    drop_event_locked(ev);
    return rc;
  }
  for (size_t i = 0; i < p.src.size(); ++i) {
    const size_t si = size_t(p.src[i]), di = size_t(p.dst[i]);
    if (to_host) {
      m->dev_d2h_seq[si] = seq;
      m->host_d2h_seq[di] = seq;
      m->dev_d2h_chunk[si] = m->host_d2h_chunk[di] = chunk_of[i];
    } else {
      m->host_h2d_seq[si] = seq;
      m->dev_h2d_seq[di] = seq;
      m->host_h2d_chunk[si] = m->dev_h2d_chunk[di] = chunk_of[i];
    }
  }
  *out = ev;
  return TS_OK;
}

// Implicit pools (EnsureImplicitPools, kv_cache_manager_base.cc:1554-1590):
// one per storage (layer) with positive block bytes, num_blocks = the host
// mirror size (host_blocks x layer-0 block bytes) / that layer's block bytes;
// storages without one are skipped, so later pool indices shift as there.
const std::vector<pool::Pool>& pools_of(const ts_manager* m, std::vector<pool::Pool>* scratch) {
  if (m->explicit_pools) return m->pools;
  scratch->clear();
  for (int l = 0; l < m->num_layers; ++l) {
    const int64_t stride = int64_t(m->st[size_t(l * m->num_shards)].bb);
    if (stride <= 0) continue;
    const int64_t nb = m->host_blocks * int64_t(m->bytes_per_block) / stride;
    if (nb <= 0) continue;
    pool::Pool p;
    p.tag = "opaque";
    p.storage_index = l;
    p.block_stride_bytes = stride;
    p.num_blocks = nb;
    p.regions.push_back({"block", 0, stride, stride, 1, 1});
    scratch->push_back(std::move(p));
  }
  return *scratch;
}

// Byte work of one storage's pool extents.  The host mirror shares the
// storage's byte offsets: device byte x is host block x / bb at offset
// x % bb of the storage's slot, so extents are cut at block boundaries.
// Whole blocks become strided DMAs (runs of consecutive blocks); partial
// pieces become segment-copy rows, run-length merged when they repeat with
// constant device and host deltas.
void add_pool_work(const ts_manager* m, bool to_host, const Storage& sd,
                   const std::vector<pool::Extent>& ext, Plan* plan,
                   std::set<int64_t>* blocks) {
  const int64_t bb = int64_t(sd.bb);
  int64_t run_next = -1;  // next block id that would extend the last DMA run
  const size_t dma0 = plan->dma.size();
  auto push_seg = [&](uint64_t src, uint64_t dst, uint32_t bytes) {
    if (!plan->seg.empty()) {
      SegTask& t = plan->seg.back();
      if (t.bytes == bytes && t.count < UINT32_MAX) {
        if (t.count == 1) {
          t.src_stride = int64_t(src - t.src);
          t.dst_stride = int64_t(dst - t.dst);
          t.count = 2;
          return;
        }
        if (src == t.src + uint64_t(int64_t(t.count) * t.src_stride) &&
            dst == t.dst + uint64_t(int64_t(t.count) * t.dst_stride)) {
          ++t.count;
          return;
        }
      }
    }
    plan->seg.push_back({src, dst, 0, 0, bytes, 1});
  };
  for (const pool::Extent& e : ext) {
    int64_t x = e.offset, left = e.size;
    while (left > 0) {
      const int64_t blk = x / bb, in = x % bb;
      const int64_t take = std::min(bb - in, left);
      blocks->insert(blk);
      const uint64_t dev = sd.dev_ptr + uint64_t(blk) * uint64_t(bb);
      const uint64_t slot = uint64_t(blk) * m->host_pitch + sd.host_off;
      if (in == 0 && take == bb) {
        if (blk == run_next && plan->dma.size() > dma0) {
          ++plan->dma.back().rows;
        } else {
          plan->dma.push_back({dev, reinterpret_cast<uint64_t>(m->host) + slot, uint64_t(bb),
                               uint64_t(bb), m->host_pitch, 1});
        }
        run_next = blk + 1;
      } else {
        const uint64_t hdev = reinterpret_cast<uint64_t>(m->host_dev) + slot;
        for (int64_t o = 0; o < take; o += int64_t(1) << 30) {
          const uint32_t n = uint32_t(std::min<int64_t>(take - o, int64_t(1) << 30));
          const uint64_t d = dev + uint64_t(in + o), h = hdev + uint64_t(in + o);
          if (to_host) push_seg(d, h, n); else push_seg(h, d, n);
        }
      }
      x += take;
      left -= take;
    }
  }
}

// CopyPoolBlocks' planning (kv_cache_manager_base.cc:1789-1858): the same
// checks, codes and messages, all of them before any copy is queued.
int build_pool_plan(const ts_manager* m, bool to_host, int64_t pool_idx, const int64_t* ids,
                    int64_t n, int64_t shard_idx, Plan* plan) {
  if (n < 0 || (n > 0 && !ids)) return set_error(TS_INVALID_ARGUMENT, "block_ids must be a valid array");
  if (m->fp8)
    return set_error(TS_UNIMPLEMENTED, "pool copies are not supported on an fp8 host tier");
  std::vector<pool::Pool> scratch;
  const std::vector<pool::Pool>& pools = pools_of(m, &scratch);
  if (pool_idx < 0 || pool_idx >= int64_t(pools.size()))
    return set_errorf(TS_OUT_OF_RANGE, "pool index %lld out of range: %zu pools",
                      static_cast<long long>(pool_idx), pools.size());
  const pool::Pool& pool = pools[size_t(pool_idx)];
  if (pool.storage_index >= m->num_layers)
    return set_error(TS_FAILED_PRECONDITION, "pool storage has no device buffers (host-only manager)");
  if (shard_idx >= m->num_shards) return set_error(TS_OUT_OF_RANGE, "shard index out of range");
  std::vector<pool::Extent> ext;
  int rc = pool::copy_extents(pool, ids, n, &ext);
  if (rc != TS_OK) return rc;
  plan->pool = true;
  plan->whole = false;
  std::set<int64_t> blocks;
  for (int sh = 0; sh < m->num_shards; ++sh) {
    if (shard_idx >= 0 && sh != shard_idx) continue;
    const int si = int(pool.storage_index) * m->num_shards + sh;
    const Storage& sd = m->st[size_t(si)];
    const int64_t host_size = m->host_blocks * int64_t(sd.bb);
    for (const pool::Extent& e : ext) {
      const int64_t end = e.offset + e.size;
      if (end > host_size) return set_error(TS_OUT_OF_RANGE, "pool block copy exceeds host buffer size");
      if (end > int64_t(sd.nbytes))
        return set_error(TS_OUT_OF_RANGE, "pool block copy exceeds device buffer size");
    }
    plan->storages.push_back(si);
    add_pool_work(m, to_host, sd, ext, plan, &blocks);
  }
  plan->src.assign(blocks.begin(), blocks.end());
  plan->dst = plan->src;
  return TS_OK;
}

int pool_transfer(ts_manager* m, bool to_host, int64_t pool_idx, const int64_t* ids, int64_t n,
                  int64_t shard_idx, void* stream, ts_event** out) {
  clear_error();
  if (!m || !out) return set_error(TS_INVALID_ARGUMENT, "null manager or output");
  *out = nullptr;
  std::lock_guard<std::mutex> lock(m->mu);
  if (m->closed) return set_error(TS_FAILED_PRECONDITION, "manager already destroyed");
  Plan p;
  int rc = build_pool_plan(m, to_host, pool_idx, ids, n, shard_idx, &p);
  if (rc != TS_OK) return rc;
  return submit_locked(m, to_host, p, stream, out);
}

void destroy_resources(ts_manager* m) {
  DeviceGuard g(m->device);
  sync_all(m);
  for (std::vector<Slot>* slots : {&m->out_slots, &m->in_slots})
    for (Slot& sl : *slots) {
      if (sl.buf) cudaFree(sl.buf);
      if (sl.ready) cudaEventDestroy(sl.ready);
      if (sl.free) cudaEventDestroy(sl.free);
    }
  for (CallRec* ring : {m->d2h_ring, m->h2d_ring})
    for (int i = 0; i < kEventRing; ++i) {
      if (ring[i].done) cudaEventDestroy(ring[i].done);
      for (cudaEvent_t e : ring[i].chunk_ev) cudaEventDestroy(e);
    }
  for (cudaStream_t s : {m->s_out_kernel, m->s_in_kernel, m->s_in_kernel2})
    if (s) cudaStreamDestroy(s);
  if (m->in_join) cudaEventDestroy(m->in_join);
  for (int i = 0; i < kMaxCopyStreams; ++i) {
    if (m->out_cs[i]) cudaStreamDestroy(m->out_cs[i]);
    if (m->in_cs[i]) cudaStreamDestroy(m->in_cs[i]);
    if (m->out_join[i]) cudaEventDestroy(m->out_join[i]);
  }
  for (int k = 0; k < 2; ++k)
    for (cudaEvent_t e : m->prof_ev[k]) cudaEventDestroy(e);
  for (cudaEvent_t e : m->prof_free) cudaEventDestroy(e);
  if (m->ev_user) cudaEventDestroy(m->ev_user);
  if (m->d_table) cudaFree(m->d_table);
  if (m->tier) ts_host_tier_destroy(m->tier, 0);
  m->d_table = nullptr;
  m->tier = nullptr;
}

}  // namespace
}  // namespace tsb

using tsb::set_error;
using tsb::set_errorf;

extern "C" int ts_mgr_create(const ts_storage_desc* storages, int num_layers,
                             int num_shards, const ts_manager_opts* opts,
                             ts_manager** out) {
  tsb::clear_error();
  if (!out) return set_error(TS_INVALID_ARGUMENT, "out must not be null");
  *out = nullptr;
  if (num_layers <= 0 || num_shards <= 0 || !storages)
    return set_error(TS_INVALID_ARGUMENT, "need at least one layer and one shard");
  auto* m = new ts_manager();
  m->num_layers = num_layers;
  m->num_shards = num_shards;
  m->device = storages[0].device;
  m->major_dim = storages[0].dim0;
  if (m->major_dim <= 0) {
    delete m;
    return set_error(TS_INVALID_ARGUMENT, "storage dim 0 must be positive");
  }
  m->host_blocks = opts && opts->host_blocks > 0 ? opts->host_blocks : 64;
  m->fp8 = opts && opts->fp8;
  if (opts && opts->chunk_blocks > 0)
    m->chunk_blocks = std::min<int64_t>(opts->chunk_blocks, tsb::kMaxParamIds);
  m->mode = opts ? opts->mode : 0;
  if (m->mode < 0 || m->mode > 3) {
    delete m;
    return set_error(TS_INVALID_ARGUMENT, "mode must be in 0..3");
  }
  m->ncs = opts && opts->copy_streams > 0 ? std::min(opts->copy_streams, tsb::kMaxCopyStreams) : 2;
  m->max_ctas = opts && opts->max_ctas > 0 ? opts->max_ctas : 0;
  m->reload_staged_every = opts && opts->reload_staged_every > 0 && (m->mode & 2)
                               ? opts->reload_staged_every : 0;
  m->sched = opts ? opts->sched : 0;
  if (m->sched < 0 || m->sched > (TS_SCHED_OFFLOAD_PRIORITY | TS_SCHED_RELOAD_PER_PIECE |
                                  TS_SCHED_RELOAD_OVERLAP | TS_SCHED_BULK_COPY |
                                  TS_SCHED_WIDE_LOADS)) {
    delete m;
    return set_error(TS_INVALID_ARGUMENT, "sched must be a sum of TS_SCHED_* flags");
  }
  const int n = num_layers * num_shards;
  m->st.resize(size_t(n));
  // reference: slice_byte_size from layer 0, shard 0 (GetMajorSliceByteSize)
  m->bytes_per_block = storages[0].nbytes / uint64_t(m->major_dim);
  uint64_t off = 0;
  int64_t max_dev_blocks = 0;
  for (int i = 0; i < n; ++i) {
    const ts_storage_desc& d = storages[i];
    if (d.device != m->device) {
      delete m;
      return set_error(TS_INVALID_ARGUMENT,
                       "all storages of one manager must live on one CUDA device "
                       "(create one manager per GPU)");
    }
    const int layer = i / num_shards;
    const ts_storage_desc& shard0 = storages[layer * num_shards];
    if (d.nbytes < shard0.nbytes) {
      delete m;
      return set_error(TS_INVALID_ARGUMENT, "Device buffer shard size smaller than physical size");
    }
    tsb::Storage& s = m->st[size_t(i)];
    s.dev_ptr = d.dev_ptr;
    s.nbytes = d.nbytes;
    s.dim0 = d.dim0;
    s.bb = shard0.nbytes / uint64_t(m->major_dim);
    s.host_bytes = m->fp8 ? s.bb / 2 : s.bb;
    if (m->fp8 && (s.bb % 32) != 0) {
      delete m;
      return set_error(TS_INVALID_ARGUMENT, "fp8 tier needs block bytes that are a multiple of 32");
    }
    s.host_off = off;
    off += tsb::round16(s.host_bytes);
    if (s.bb) max_dev_blocks = std::max<int64_t>(max_dev_blocks, int64_t(s.nbytes / s.bb));
    m->max_bb = std::max(m->max_bb, s.bb);
    m->vec_ok = m->vec_ok && (s.dev_ptr % 16 == 0) && (s.bb % 16 == 0);
  }
  if (m->fp8 && !m->vec_ok) {
    delete m;
    return set_error(TS_INVALID_ARGUMENT,
                     "fp8 tier needs 16-byte aligned storages (the fused cast moves 16-byte "
                     "vectors and bulk copies)");
  }
  if (m->fp8) {
    m->scale_off = off;
    off += tsb::round16(uint64_t(n) * 4);
  }
  m->host_pitch = tsb::round16(off);

  tsb::DeviceGuard g(m->device);
  int rc = TS_OK;
  auto fail = [&](int code) {
    tsb::destroy_resources(m);
    tsb::unref_manager(m);
    return code;
  };
  const char* shm = opts ? opts->shm_name : nullptr;
  const char* uid = opts && opts->model_uid ? opts->model_uid : "";
  uint64_t geometry = m->host_pitch * 1000003ull ^ uint64_t(n) * 7919ull ^ (m->fp8 ? 1 : 0);
  int warm = 0;
  // NUMA node of the host tier: the device's own (DetectAndAssignNumaNode,
  // raiden_manager_base.cc:47-78) unless the caller overrides it
  // (kv_cache_manager_base.cc:231-249); pages are placed there while the
  // tier is allocated and pinned, on hosts with more than one node.
  const int numa_opt = opts ? opts->numa_node : 0;
  m->numa_node = numa_opt > 0 ? numa_opt - 1 : numa_opt == 0 ? tsb::device_numa_node(m->device)
                                                             : -1;
  {
    const bool place = m->numa_node >= 0 && tsb::numa_node_count(nullptr) > 1;
    tsb::ScopedPreferredNode policy(place ? m->numa_node : -1);
    m->numa_placed = policy.applied();
    rc = ts_host_tier_create(uint64_t(m->host_blocks) * m->host_pitch, shm, uid, geometry, 1,
                             &m->tier, &warm);
  }
  if (rc != TS_OK) return fail(rc);
  m->host = static_cast<uint8_t*>(ts_host_tier_ptr(m->tier));
  if (!warm && (shm == nullptr || shm[0] == '\0')) {
    // reference zero-fills its mirrors (posix_memalign + memset); anonymous
    // mmap pages are already zero.
  }

  // device table
  std::vector<ts_block_storage> table(static_cast<size_t>(n));
  for (int i = 0; i < n; ++i) {
    table[size_t(i)] = {m->st[size_t(i)].dev_ptr, m->st[size_t(i)].bb, m->st[size_t(i)].nbytes,
                        m->st[size_t(i)].host_off};
  }
  cudaError_t e = cudaMalloc(&m->d_table, sizeof(ts_block_storage) * size_t(n));
  if (e == cudaSuccess)
    e = cudaMemcpy(m->d_table, table.data(), sizeof(ts_block_storage) * size_t(n),
                   cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "storage table upload"));

  int prio_least = 0, prio_greatest = 0;
  e = cudaDeviceGetStreamPriorityRange(&prio_least, &prio_greatest);
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "stream priority range"));
  const int out_prio = (m->sched & TS_SCHED_OFFLOAD_PRIORITY) ? prio_greatest : prio_least;
  e = cudaStreamCreateWithPriority(&m->s_out_kernel, cudaStreamNonBlocking, out_prio);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->s_in_kernel, cudaStreamNonBlocking);
  if (e == cudaSuccess && (m->sched & TS_SCHED_RELOAD_OVERLAP)) {
    e = cudaStreamCreateWithFlags(&m->s_in_kernel2, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->in_join, cudaEventDisableTiming);
  }
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "stream create"));
  for (int i = 0; i < m->ncs; ++i) {
    e = cudaStreamCreateWithFlags(&m->out_cs[i], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&m->in_cs[i], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&m->out_join[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return fail(tsb::cuda_error(e, "copy stream create"));
  }
  e = cudaEventCreateWithFlags(&m->ev_user, cudaEventDisableTiming);
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "event create"));
  const size_t slot_bytes = size_t(m->chunk_blocks) * m->host_pitch;
  for (int dir = 0; dir < 2; ++dir) {
    if (tsb::is_direct(m, dir == 0) && !(dir == 1 && m->reload_staged_every > 0)) continue;
    std::vector<tsb::Slot>& slots = dir == 0 ? m->out_slots : m->in_slots;
    slots.resize(size_t(2 * m->ncs));
    for (tsb::Slot& sl : slots) {
      e = cudaMalloc(&sl.buf, slot_bytes);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.ready, cudaEventDisableTiming);
      if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sl.free, cudaEventDisableTiming);
      if (e != cudaSuccess) return fail(tsb::cuda_error(e, "staging slot"));
    }
  }
  e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&m->host_dev), m->host, 0);
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "host tier mapping"));
  // 32-byte vectors need every storage, slot, block size, the pitch and the
  // mapped tier 32-byte aligned
  m->wide_ok = m->vec_ok && !m->fp8 && m->host_pitch % 32 == 0 &&
               reinterpret_cast<uintptr_t>(m->host_dev) % 32 == 0;
  for (const auto& st : m->st)
    m->wide_ok = m->wide_ok && st.dev_ptr % 32 == 0 && st.bb % 32 == 0 && st.host_off % 32 == 0;
  e = cudaHostAlloc(reinterpret_cast<void**>(&m->err_host), sizeof(int) * tsb::kErrWords,
                    cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) return fail(tsb::cuda_error(e, "error words"));
  for (int i = tsb::kErrWords - 1; i >= 0; --i) m->err_free.push_back(i);
  m->host_d2h_seq.assign(size_t(m->host_blocks), 0);
  m->host_h2d_seq.assign(size_t(m->host_blocks), 0);
  m->dev_d2h_seq.assign(size_t(max_dev_blocks), 0);
  m->dev_h2d_seq.assign(size_t(max_dev_blocks), 0);
  m->host_d2h_chunk.assign(size_t(m->host_blocks), -1);
  m->host_h2d_chunk.assign(size_t(m->host_blocks), -1);
  m->dev_d2h_chunk.assign(size_t(max_dev_blocks), -1);
  m->dev_h2d_chunk.assign(size_t(max_dev_blocks), -1);
  *out = m;
  return TS_OK;
}

extern "C" int ts_mgr_destroy(ts_manager* mgr) {
  tsb::clear_error();
  if (!mgr) return TS_OK;
  {
    std::lock_guard<std::mutex> lock(mgr->mu);
    tsb::destroy_resources(mgr);  // drains every stream first
    mgr->closed = true;
  }
  tsb::unref_manager(mgr);
  return TS_OK;
}

extern "C" int ts_d2h(ts_manager* mgr, const int64_t* src, const int64_t* dst,
                      const int64_t* sizes, int64_t n_src, int64_t n_dst,
                      int64_t n_sizes, int64_t layer_idx, int64_t shard_idx,
                      void* stream, ts_event** out) {
  return tsb::transfer(mgr, true, src, dst, sizes, n_src, n_dst, n_sizes, layer_idx,
                       shard_idx, stream, out);
}

extern "C" int ts_h2d(ts_manager* mgr, const int64_t* src, const int64_t* dst,
                      const int64_t* sizes, int64_t n_src, int64_t n_dst,
                      int64_t n_sizes, int64_t layer_idx, int64_t shard_idx,
                      void* stream, ts_event** out) {
  return tsb::transfer(mgr, false, src, dst, sizes, n_src, n_dst, n_sizes, layer_idx,
                       shard_idx, stream, out);
}

extern "C" int ts_mgr_host_block_ptr(ts_manager* mgr, int64_t layer_idx, int64_t shard_idx,
                                     int64_t block_id, uint64_t* ptr_out,
                                     uint64_t* bytes_out) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  if (layer_idx < 0 || layer_idx >= mgr->num_layers || shard_idx < 0 ||
      shard_idx >= mgr->num_shards)
    return set_error(TS_OUT_OF_RANGE, "layer or shard index out of range");
  if (block_id < 0 || block_id >= mgr->host_blocks)
    return set_errorf(TS_OUT_OF_RANGE, "Invalid host block ID: %lld", (long long)block_id);
  const tsb::Storage& s = mgr->st[size_t(layer_idx * mgr->num_shards + shard_idx)];
  if (ptr_out)
    *ptr_out = reinterpret_cast<uint64_t>(mgr->host + uint64_t(block_id) * mgr->host_pitch +
                                          s.host_off);
  if (bytes_out) *bytes_out = s.host_bytes;
  return TS_OK;
}

extern "C" int ts_mgr_numa_node(ts_manager* mgr, int* node, int* placed) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  if (node) *node = mgr->numa_node;
  if (placed) *placed = mgr->numa_placed ? 1 : 0;
  return TS_OK;
}

extern "C" int ts_mgr_info(ts_manager* mgr, int64_t* host_blocks, uint64_t* host_block_pitch,
                           int64_t* major_dim, uint64_t* bytes_per_block) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  if (host_blocks) *host_blocks = mgr->host_blocks;
  if (host_block_pitch) *host_block_pitch = mgr->host_pitch;
  if (major_dim) *major_dim = mgr->major_dim;
  if (bytes_per_block) *bytes_per_block = mgr->bytes_per_block;
  return TS_OK;
}

extern "C" int ts_mgr_storage(ts_manager* mgr, int index, int* device, uint64_t* dev_ptr,
                              uint64_t* nbytes, int64_t* dim0, uint64_t* block_bytes) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  if (index < 0 || index >= int(mgr->st.size()))
    return set_errorf(TS_OUT_OF_RANGE, "storage index %d out of range [0, %d)", index,
                      int(mgr->st.size()));
  const tsb::Storage& st = mgr->st[size_t(index)];
  if (device) *device = mgr->device;
  if (dev_ptr) *dev_ptr = st.dev_ptr;
  if (nbytes) *nbytes = st.nbytes;
  if (dim0) *dim0 = st.dim0;
  if (block_bytes) *block_bytes = st.bb;
  return TS_OK;
}

extern "C" int ts_mgr_num_storages(ts_manager* mgr, int* n) {
  tsb::clear_error();
  if (!mgr || !n) return set_error(TS_INVALID_ARGUMENT, "null argument");
  *n = int(mgr->st.size());
  return TS_OK;
}

extern "C" int ts_mgr_register_pools(ts_manager* mgr, const ts_pool_spec* pools, int64_t n) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  if (n <= 0 || !pools) return set_error(TS_INVALID_ARGUMENT, "pool table must be non-empty");
  std::vector<tsb::pool::Pool> parsed(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) {
    int rc = tsb::pool::from_c(&pools[i], &parsed[size_t(i)]);
    if (rc != TS_OK) return rc;
  }
  std::lock_guard<std::mutex> lock(mgr->mu);
  if (mgr->closed) return set_error(TS_FAILED_PRECONDITION, "manager already destroyed");
  if (mgr->fp8)
    return set_error(TS_UNIMPLEMENTED, "pools are not supported on an fp8 host tier");
  for (int64_t i = 0; i < n; ++i) {
    const tsb::pool::Pool& p = parsed[size_t(i)];
    if (p.storage_index >= mgr->num_layers)
      return set_errorf(TS_INVALID_ARGUMENT,
                        "pool %lld (%s) storage_index %lld out of range: manager wraps %d storages",
                        static_cast<long long>(i), p.tag.c_str(),
                        static_cast<long long>(p.storage_index), mgr->num_layers);
    // validated against the device storage (shard 0's physical size)
    const tsb::Storage& sd = mgr->st[size_t(p.storage_index * mgr->num_shards)];
    if (p.validate(int64_t(sd.nbytes)) != TS_OK)
      return set_errorf(TS_INVALID_ARGUMENT, "invalid pool %lld: %s", static_cast<long long>(i),
                        ts_last_error());
    // The reference grows this storage's host mirror to the pool's live end
    // (EnsureHostMirrorCovers, :1597-1651); the block-major tier is one
    // allocation, so the pool must fit what it already covers.
    const int64_t covered = mgr->host_blocks * int64_t(sd.bb);
    const int64_t end = p.storage_extent_end_bytes();
    if (end > covered)
      return set_errorf(TS_FAILED_PRECONDITION,
                        "invalid pool %lld: pool %s live extent ends at byte %lld but the host "
                        "tier mirrors %lld bytes of storage %lld (%lld host blocks)",
                        static_cast<long long>(i), p.tag.c_str(), static_cast<long long>(end),
                        static_cast<long long>(covered), static_cast<long long>(p.storage_index),
                        static_cast<long long>(mgr->host_blocks));
  }
  mgr->pools = std::move(parsed);
  mgr->explicit_pools = true;
  return TS_OK;
}

extern "C" int ts_mgr_num_pools(ts_manager* mgr, int64_t* n, int* explicit_pools) {
  tsb::clear_error();
  if (!mgr || !n) return set_error(TS_INVALID_ARGUMENT, "null manager or output");
  std::lock_guard<std::mutex> lock(mgr->mu);
  std::vector<tsb::pool::Pool> scratch;
  *n = int64_t(tsb::pools_of(mgr, &scratch).size());
  if (explicit_pools) *explicit_pools = mgr->explicit_pools ? 1 : 0;
  return TS_OK;
}

extern "C" int ts_mgr_pool_geometry(ts_manager* mgr, int64_t pool_idx, int64_t* storage_index,
                                    int64_t* block_stride_bytes, int64_t* num_blocks) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  std::lock_guard<std::mutex> lock(mgr->mu);
  std::vector<tsb::pool::Pool> scratch;
  const std::vector<tsb::pool::Pool>& pools = tsb::pools_of(mgr, &scratch);
  if (pool_idx < 0 || pool_idx >= int64_t(pools.size()))
    return set_errorf(TS_OUT_OF_RANGE, "pool index %lld out of range: %zu pools",
                      static_cast<long long>(pool_idx), pools.size());
  const tsb::pool::Pool& p = pools[size_t(pool_idx)];
  if (storage_index) *storage_index = p.storage_index;
  if (block_stride_bytes) *block_stride_bytes = p.block_stride_bytes;
  if (num_blocks) *num_blocks = p.num_blocks;
  return TS_OK;
}

extern "C" int ts_d2h_pool_blocks(ts_manager* mgr, int64_t pool_idx, const int64_t* block_ids,
                                  int64_t n_ids, int64_t shard_idx, void* stream,
                                  ts_event** out) {
  return tsb::pool_transfer(mgr, true, pool_idx, block_ids, n_ids, shard_idx, stream, out);
}

extern "C" int ts_h2d_pool_blocks(ts_manager* mgr, int64_t pool_idx, const int64_t* block_ids,
                                  int64_t n_ids, int64_t shard_idx, void* stream,
                                  ts_event** out) {
  return tsb::pool_transfer(mgr, false, pool_idx, block_ids, n_ids, shard_idx, stream, out);
}

extern "C" int ts_mgr_pool_block_ref(ts_manager* mgr, int64_t pool_idx, int64_t shard_idx,
                                     int64_t block_id, uint64_t* host_ptr) {
  tsb::clear_error();
  if (!mgr || !host_ptr) return set_error(TS_INVALID_ARGUMENT, "null manager or output");
  std::lock_guard<std::mutex> lock(mgr->mu);
  std::vector<tsb::pool::Pool> scratch;
  const std::vector<tsb::pool::Pool>& pools = tsb::pools_of(mgr, &scratch);
  if (pool_idx < 0 || pool_idx >= int64_t(pools.size()))
    return set_errorf(TS_OUT_OF_RANGE, "pool index %lld out of range: %zu pools",
                      static_cast<long long>(pool_idx), pools.size());
  if (block_id < 0) return set_error(TS_INVALID_ARGUMENT, "block_id must be non-negative");
  const tsb::pool::Pool& p = pools[size_t(pool_idx)];
  if (p.storage_index >= mgr->num_layers || shard_idx < 0 || shard_idx >= mgr->num_shards)
    return set_error(TS_OUT_OF_RANGE, "storage or shard index out of range");
  if (block_id >= p.num_blocks)
    return set_errorf(TS_OUT_OF_RANGE, "block_id %lld out of range for pool %lld (%s): num_blocks=%lld",
                      static_cast<long long>(block_id), static_cast<long long>(pool_idx),
                      p.tag.c_str(), static_cast<long long>(p.num_blocks));
  const tsb::Storage& sd = mgr->st[size_t(p.storage_index * mgr->num_shards + shard_idx)];
  const int64_t host_size = mgr->host_blocks * int64_t(sd.bb);
  const int64_t off = p.base_offset_bytes + block_id * p.block_stride_bytes;
  const int64_t live_end = p.block_live_end();
  if (off > host_size || live_end > host_size - off)
    return set_error(TS_OUT_OF_RANGE, "block live regions exceed host buffer");
  const int64_t bb = int64_t(sd.bb);
  if (live_end > 0 && off / bb != (off + live_end - 1) / bb)
    return set_error(TS_FAILED_PRECONDITION,
                     "pool block spans several host blocks of the block-major host tier; "
                     "copy it with d2h_pool_blocks / h2d_pool_blocks instead");
  *host_ptr = reinterpret_cast<uint64_t>(mgr->host) + uint64_t(off / bb) * mgr->host_pitch +
              sd.host_off + uint64_t(off % bb);
  return TS_OK;
}

extern "C" int ts_mgr_set_profiling(ts_manager* mgr, int on) {
  tsb::clear_error();
  if (!mgr) return set_error(TS_INVALID_ARGUMENT, "null manager");
  std::lock_guard<std::mutex> lock(mgr->mu);
  mgr->profiling = on != 0;
  return TS_OK;
}

extern "C" int ts_mgr_kernel_stats(ts_manager* mgr, int which, int64_t* launches,
                                   double* total_ms, uint64_t* bytes) {
  tsb::clear_error();
  if (!mgr || which < 0 || which > 1) return set_error(TS_INVALID_ARGUMENT, "bad arguments");
  std::lock_guard<std::mutex> lock(mgr->mu);
  tsb::DeviceGuard g(mgr->device);
  double ms = 0;
  uint64_t b = 0;
  std::vector<cudaEvent_t>& ev = mgr->prof_ev[which];
  // Launch intervals relative to the first launch's start; their union is
  // the time the kernels ran (launches on two streams may overlap).
  std::vector<std::pair<double, double>> iv;
  for (size_t i = 0; i + 1 < ev.size(); i += 2) {
    TS_CUDA_RET(cudaEventSynchronize(ev[i + 1]), "profiling event");
    float t0 = 0, t1 = 0;
    if (i > 0) TS_CUDA_RET(cudaEventElapsedTime(&t0, ev[0], ev[i]), "profiling event");
    TS_CUDA_RET(cudaEventElapsedTime(&t1, ev[0], ev[i + 1]), "profiling event");
    iv.emplace_back(double(t0), double(t1));
  }
  std::sort(iv.begin(), iv.end());
  double cur0 = 0, cur1 = -1;
  for (const auto& x : iv) {
    if (x.first > cur1) {
      if (cur1 > cur0) ms += cur1 - cur0;
      cur0 = x.first;
      cur1 = x.second;
    } else if (x.second > cur1) {
      cur1 = x.second;
    }
  }
  if (cur1 > cur0) ms += cur1 - cur0;
  for (uint64_t x : mgr->prof_bytes[which]) b += x;
  if (launches) *launches = int64_t(ev.size() / 2);
  if (total_ms) *total_ms = ms;
  if (bytes) *bytes = b;
  for (cudaEvent_t e : ev) mgr->prof_free.push_back(e);
  ev.clear();
  mgr->prof_bytes[which].clear();
  return TS_OK;
}

// ---------------------------------------------------------------------------
// Events
// ---------------------------------------------------------------------------

extern "C" int ts_event_query(ts_event* ev) {
  tsb::clear_error();
  if (!ev) return set_error(TS_INVALID_ARGUMENT, "null event");
  if (ev->finished) {
    if (ev->status != TS_OK) tsb::set_error(ev->status, ev->message);
    return ev->status;
  }
  tsb::DeviceGuard g(ev->device);
  cudaError_t e = cudaEventQuery(ev->done);
  if (e == cudaErrorNotReady) return TS_PENDING;
  ev->finished = true;
  if (e != cudaSuccess) {
    ev->status = tsb::cuda_error(e, "transfer");
    ev->message = ts_last_error();
    return ev->status;
  }
  const int word = *reinterpret_cast<volatile int*>(ev->err_word);
  if (word != 0) {
    ev->status = TS_INTERNAL;
    ev->message = "block id out of the storage bounds in the transfer kernel";
    return set_error(ev->status, ev->message);
  }
  ev->status = TS_OK;
  return TS_OK;
}

extern "C" int ts_event_wait(ts_event* ev, int64_t timeout_ms) {
  if (!ev) return set_error(TS_INVALID_ARGUMENT, "null event");
  const auto t0 = std::chrono::steady_clock::now();
  int sleep_us = 2;
  for (;;) {
    const int rc = ts_event_query(ev);
    if (rc != TS_PENDING) return rc;
    if (timeout_ms >= 0 &&
        std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
      return set_error(TS_DEADLINE_EXCEEDED, "transfer did not complete before the timeout");
    std::this_thread::sleep_for(std::chrono::microseconds(sleep_us));
    sleep_us = std::min(sleep_us * 2, 200);
  }
}

extern "C" int ts_event_error(ts_event* ev, char* buf, size_t len) {
  if (!ev || !buf || len == 0) return TS_INVALID_ARGUMENT;
  const std::string msg = ev->finished && ev->status != TS_OK ? ev->message : std::string();
  std::snprintf(buf, len, "%s", msg.c_str());
  return TS_OK;
}

extern "C" int ts_event_stream_wait(ts_event* ev, void* stream) {
  tsb::clear_error();
  if (!ev) return set_error(TS_INVALID_ARGUMENT, "null event");
  TS_CUDA_RET(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), ev->done, 0),
              "stream wait");
  return TS_OK;
}

extern "C" int ts_event_elapsed_ms(ts_event* ev, float* ms) {
  tsb::clear_error();
  if (!ev || !ms) return set_error(TS_INVALID_ARGUMENT, "null argument");
  TS_CUDA_RET(cudaEventElapsedTime(ms, ev->start, ev->done), "elapsed time");
  return TS_OK;
}

extern "C" void ts_event_release(ts_event* ev) {
  if (!ev) return;
  tsb::DeviceGuard g(ev->device);
  // The kernels of a pending transfer may still write its error word.
  if (!ev->finished) cudaEventSynchronize(ev->done);
  ts_manager* m = ev->mgr;
  if (m && ev->err_index >= 0) {
    std::lock_guard<std::mutex> lock(m->mu);
    m->err_free.push_back(ev->err_index);
  }
  cudaEventDestroy(ev->start);
  cudaEventDestroy(ev->done);
  delete ev;
  if (m) tsb::unref_manager(m);
}

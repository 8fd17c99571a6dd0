// Weight synchronizer object of the C ABI: a trainer's [layer][shard] device
// buffers, a registered push plan (the controller's ShardPushEntry lists) and
// its execution as one strided-copy kernel per source GPU.
//
// Reference: WeightSynchronizerBase::PushWeightsResharded
// (tpu_sync/weight_sync/weight_synchronizer_base.cc:558-760).  Kept: for
// every local shard i in order, for its entries in order, the layer is the
// entry's layer_idx or, when it has none, the layer named by the request's
// first source unit ("src_units list cannot be empty" / "Layer name not found
// in WeightSynchronizer: <name>", :566-587); "Layer index out of bounds: <i>"
// (:612-616); count 0 means 1 (:627); an entry with count 1 or strides equal
// to its size is one contiguous payload whose source range is checked once,
// otherwise every repeat is checked ("Push range out of bounds", :633-663).
// Every check runs before any byte moves.  New here, because the bytes no
// longer travel through a receiver that bounds them: the destination of
// every entry must be registered and must hold the entry's range ("No
// destination for peer <p> layer <l> shard <s>", "Push destination range out
// of bounds").  A zero-byte entry is checked and then moves nothing.
//
// Execution: the reference expands each entry into per-repeat host-to-host
// pushes over TCP followed by an H2D on the receiver (:606-667, :824-845).
// Here each entry is one strided task of the reshard kernel (rows of `size`
// bytes at src_off + c*src_stride -> dst_off + c*dst_stride), all tasks of one
// source GPU in one launch that stores straight into the destination (its
// own memory, a peer GPU's memory with peer access, or a CUDA IPC mapping
// opened for that GPU) over NVLink.

#include <cuda_runtime.h>

#include <chrono>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "ts_internal.h"

struct ts_wsync {
  struct Prog {
    int device = 0;
    cudaStream_t stream = nullptr;
    cudaEvent_t done = nullptr;
    ts_reshard_chunk* d_chunks = nullptr;
    int64_t* d_prefix = nullptr;
    int64_t n_chunks = 0, n_items = 0;
    uint64_t bytes = 0;
  };
  int num_layers = 0, num_shards = 0;
  std::vector<ts_wsync_buffer> buf;  // [layer * num_shards + shard]
  std::vector<std::string> names;
  std::map<int, Prog> progs;                  // by source device
  std::map<int, cudaEvent_t> user_ev;         // ordering event per user-stream device
  bool pushed = false;
  std::mutex mu;
};

namespace tsb {
namespace {

// Drains a previous push before the plan's device tables are replaced.
void drain(ts_wsync* w) {
  if (!w->pushed) return;
  for (auto& kv : w->progs) {
    DeviceGuard g(kv.first);
    cudaEventSynchronize(kv.second.done);
  }
  w->pushed = false;
}

void free_tables(ts_wsync* w) {
  for (auto& kv : w->progs) {
    DeviceGuard g(kv.first);
    if (kv.second.d_chunks) cudaFree(kv.second.d_chunks);
    if (kv.second.d_prefix) cudaFree(kv.second.d_prefix);
    kv.second.d_chunks = nullptr;
    kv.second.d_prefix = nullptr;
    kv.second.n_chunks = kv.second.n_items = 0;
    kv.second.bytes = 0;
  }
}

// off + n * stride + len <= limit, without unsigned wrap-around.
bool fits(uint64_t off, uint64_t n, uint64_t stride, uint64_t len, uint64_t limit) {
  if (off > limit || len > limit - off) return false;
  return stride == 0 || n <= (limit - off - len) / stride;
}

int prog_for(ts_wsync* w, int device, ts_wsync::Prog** out) {
  auto it = w->progs.find(device);
  if (it == w->progs.end()) {
    ts_wsync::Prog p;
    p.device = device;
    DeviceGuard g(device);
    TS_CUDA_RET(cudaStreamCreateWithFlags(&p.stream, cudaStreamNonBlocking), "stream create");
    TS_CUDA_RET(cudaEventCreateWithFlags(&p.done, cudaEventDisableTiming), "event create");
    it = w->progs.emplace(device, p).first;
  }
  *out = &it->second;
  return TS_OK;
}

}  // namespace
}  // namespace tsb

using tsb::set_error;
using tsb::set_errorf;

extern "C" int ts_wsync_create(const ts_wsync_buffer* buffers, int num_layers, int num_shards,
                               const char* const* layer_names, ts_wsync** out) {
  tsb::clear_error();
  if (!out) return set_error(TS_INVALID_ARGUMENT, "out must not be null");
  *out = nullptr;
  if (num_layers <= 0 || num_shards <= 0 || !buffers)
    return set_error(TS_INVALID_ARGUMENT, "need at least one layer and one shard");
  auto* w = new ts_wsync();
  w->num_layers = num_layers;
  w->num_shards = num_shards;
  w->buf.assign(buffers, buffers + size_t(num_layers) * size_t(num_shards));
  for (int l = 0; l < num_layers; ++l)
    w->names.push_back(layer_names && layer_names[l] ? layer_names[l] : std::to_string(l));
  *out = w;
  return TS_OK;
}

extern "C" int ts_wsync_register_plan(ts_wsync* w, const ts_shard_push_entry* entries,
                                      int64_t n_entries, const char* src_data_name,
                                      const ts_wsync_dest* dests, int64_t n_dests) {
  tsb::clear_error();
  if (!w || n_entries < 0 || n_dests < 0 || (n_entries > 0 && !entries) ||
      (n_dests > 0 && !dests))
    return set_error(TS_INVALID_ARGUMENT, "bad arguments");
  std::lock_guard<std::mutex> lock(w->mu);
  std::map<std::tuple<std::string, int64_t, int64_t>, const ts_wsync_dest*> dest_of;
  for (int64_t d = 0; d < n_dests; ++d)
    dest_of[{dests[d].peer ? dests[d].peer : "", dests[d].layer_idx, dests[d].dst_shard_idx}] =
        &dests[d];

  int fallback = -1;
  bool checked_fallback = false;
  std::map<int, std::vector<ts_reshard_chunk>> tasks;  // by source device
  std::vector<std::pair<int, int>> peers;              // (source device, destination device)
  for (int i = 0; i < w->num_shards; ++i) {
    for (int64_t k = 0; k < n_entries; ++k) {
      const ts_shard_push_entry& e = entries[k];
      if (e.src_shard_idx != i) continue;
      int64_t layer = -1;
      if (e.has_layer_idx) {
        layer = e.layer_idx;
      } else {
        if (!checked_fallback) {
          checked_fallback = true;
          if (src_data_name == nullptr)
            return set_error(TS_INVALID_ARGUMENT, "src_units list cannot be empty");
          for (int l = 0; l < w->num_layers; ++l)
            if (w->names[size_t(l)] == src_data_name) {
              fallback = l;
              break;
            }
        }
        if (fallback == -1) {
          if (src_data_name == nullptr)
            return set_error(TS_INVALID_ARGUMENT, "src_units list cannot be empty");
          return set_errorf(TS_NOT_FOUND, "Layer name not found in WeightSynchronizer: %s",
                            src_data_name);
        }
        layer = fallback;
      }
      if (layer < 0 || layer >= w->num_layers)
        return set_errorf(TS_INVALID_ARGUMENT, "Layer index out of bounds: %lld",
                          (long long)layer);
      const ts_wsync_buffer& b = w->buf[size_t(layer) * size_t(w->num_shards) + size_t(i)];
      if (b.dev_ptr == 0) return set_error(TS_INTERNAL, "Host pointer is null during resharded push");
      const uint64_t shard_size = b.nbytes;
      const uint64_t count = e.count > 0 ? uint64_t(e.count) : 1;
      const uint64_t size = e.size_bytes, so = e.src_offset_bytes, do_ = e.dst_offset_bytes;
      const uint64_t ss = e.src_stride_bytes, ds = e.dst_stride_bytes;
      const bool contiguous = count == 1 || (ss == size && ds == size);
      // Per repeat the reference checks so + c*ss + size; with ss >= 0 the
      // last repeat is the largest, so checking it finds the same failure.
      if (contiguous ? !tsb::fits(so, count, size, 0, shard_size)
                     : !tsb::fits(so, count - 1, ss, size, shard_size))
        return set_error(TS_INVALID_ARGUMENT, "Push range out of bounds");
      if (size == 0) continue;
      if (count > (uint64_t(1) << 31))
        return set_errorf(TS_INVALID_ARGUMENT, "entry count %llu is too large",
                          (unsigned long long)count);
      const std::string peer = e.dst_peer ? e.dst_peer : "";
      auto it = dest_of.find({peer, layer, e.dst_shard_idx});
      if (it == dest_of.end())
        return set_errorf(TS_INVALID_ARGUMENT, "No destination for peer %s layer %lld shard %lld",
                          peer.c_str(), (long long)layer, (long long)e.dst_shard_idx);
      const ts_wsync_dest& d = *it->second;
      if (contiguous ? !tsb::fits(do_, count, size, 0, d.nbytes)
                     : !tsb::fits(do_, count - 1, ds, size, d.nbytes))
        return set_error(TS_INVALID_ARGUMENT, "Push destination range out of bounds");
      ts_reshard_chunk c;
      c.src_ptr = b.dev_ptr;
      c.dst_ptr = d.dst_ptr;
      c.src_off = int64_t(so);
      c.dst_off = int64_t(do_);
      c.size = int64_t(contiguous ? count * size : size);
      c.src_stride = contiguous ? 0 : int64_t(ss);
      c.dst_stride = contiguous ? 0 : int64_t(ds);
      c.count = contiguous ? 1 : int64_t(count);
      tasks[b.device].push_back(c);
      if (d.device >= 0 && d.device != b.device) peers.emplace_back(b.device, d.device);
    }
  }
  for (const auto& p : peers) {
    const int rc = ts_enable_peer_access(p.first, p.second);
    if (rc != TS_OK) return rc;
  }
  // Valid: replace the plan (after any push still using the old tables).
  tsb::drain(w);
  tsb::free_tables(w);
  for (auto& kv : tasks) {
    ts_wsync::Prog* p = nullptr;
    int rc = tsb::prog_for(w, kv.first, &p);
    if (rc != TS_OK) return rc;
    std::vector<int64_t> prefix(kv.second.size() + 1);
    rc = ts_reshard_work_items(kv.second.data(), int64_t(kv.second.size()), TS_DTYPE_U8,
                               TS_DTYPE_U8, prefix.data());
    if (rc != TS_OK) return rc;
    tsb::DeviceGuard g(kv.first);
    TS_CUDA_RET(cudaMalloc(&p->d_chunks, sizeof(ts_reshard_chunk) * kv.second.size()),
                "plan table");
    TS_CUDA_RET(cudaMalloc(&p->d_prefix, sizeof(int64_t) * prefix.size()), "plan table");
    TS_CUDA_RET(cudaMemcpy(p->d_chunks, kv.second.data(),
                           sizeof(ts_reshard_chunk) * kv.second.size(), cudaMemcpyHostToDevice),
                "plan upload");
    TS_CUDA_RET(cudaMemcpy(p->d_prefix, prefix.data(), sizeof(int64_t) * prefix.size(),
                           cudaMemcpyHostToDevice),
                "plan upload");
    p->n_chunks = int64_t(kv.second.size());
    p->n_items = prefix.back();
    for (const ts_reshard_chunk& c : kv.second) p->bytes += uint64_t(c.size) * uint64_t(c.count);
  }
  return TS_OK;
}

extern "C" int ts_wsync_push(ts_wsync* w, void* stream) {
  tsb::clear_error();
  if (!w) return set_error(TS_INVALID_ARGUMENT, "null synchronizer");
  std::lock_guard<std::mutex> lock(w->mu);
  cudaStream_t us = reinterpret_cast<cudaStream_t>(stream);
  int udev = 0;
  if (us != nullptr) {
    TS_CUDA_RET(cudaStreamGetDevice(us, &udev), "stream device");
  } else {
    TS_CUDA_RET(cudaGetDevice(&udev), "current device");
  }
  tsb::DeviceGuard g(udev);
  cudaEvent_t& ue = w->user_ev[udev];
  if (ue == nullptr) TS_CUDA_RET(cudaEventCreateWithFlags(&ue, cudaEventDisableTiming), "event create");
  TS_CUDA_RET(cudaEventRecord(ue, us), "event record");
  for (auto& kv : w->progs) {
    ts_wsync::Prog& p = kv.second;
    tsb::DeviceGuard gd(p.device);
    TS_CUDA_RET(cudaStreamWaitEvent(p.stream, ue, 0), "stream wait");
    if (p.n_items > 0) {
      const int rc = ts_reshard_copy(p.device, p.d_chunks, p.d_prefix, p.n_chunks, p.n_items,
                                     TS_DTYPE_U8, TS_DTYPE_U8, p.stream);
      if (rc != TS_OK) return rc;
    }
    TS_CUDA_RET(cudaEventRecord(p.done, p.stream), "event record");
  }
  w->pushed = true;
  return TS_OK;
}

extern "C" int ts_wsync_query(ts_wsync* w) {
  tsb::clear_error();
  if (!w) return set_error(TS_INVALID_ARGUMENT, "null synchronizer");
  std::lock_guard<std::mutex> lock(w->mu);
  for (auto& kv : w->progs) {
    tsb::DeviceGuard g(kv.first);
    const cudaError_t e = cudaEventQuery(kv.second.done);
    if (e == cudaErrorNotReady) return TS_PENDING;
    TS_CUDA_RET(e, "weight push");
  }
  return TS_OK;
}

extern "C" int ts_wsync_wait(ts_wsync* w, int64_t timeout_ms) {
  tsb::clear_error();
  if (!w) return set_error(TS_INVALID_ARGUMENT, "null synchronizer");
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const int rc = ts_wsync_query(w);
    if (rc != TS_PENDING) return rc;
    const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (timeout_ms >= 0 && ms >= timeout_ms)
      return set_errorf(TS_DEADLINE_EXCEEDED, "weight push did not finish within %lld ms",
                        (long long)timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

extern "C" int ts_wsync_stream_wait(ts_wsync* w, void* stream) {
  tsb::clear_error();
  if (!w) return set_error(TS_INVALID_ARGUMENT, "null synchronizer");
  std::lock_guard<std::mutex> lock(w->mu);
  for (auto& kv : w->progs)
    TS_CUDA_RET(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), kv.second.done, 0),
                "stream wait");
  return TS_OK;
}

extern "C" int ts_wsync_info(ts_wsync* w, int64_t* n_tasks, uint64_t* bytes) {
  tsb::clear_error();
  if (!w) return set_error(TS_INVALID_ARGUMENT, "null synchronizer");
  std::lock_guard<std::mutex> lock(w->mu);
  int64_t n = 0;
  uint64_t b = 0;
  for (auto& kv : w->progs) {
    n += kv.second.n_chunks;
    b += kv.second.bytes;
  }
  if (n_tasks) *n_tasks = n;
  if (bytes) *bytes = b;
  return TS_OK;
}

extern "C" void ts_wsync_destroy(ts_wsync* w) {
  if (!w) return;
  {
    std::lock_guard<std::mutex> lock(w->mu);
    tsb::drain(w);
    tsb::free_tables(w);
    for (auto& kv : w->progs) {
      tsb::DeviceGuard g(kv.first);
      cudaStreamDestroy(kv.second.stream);
      cudaEventDestroy(kv.second.done);
    }
    for (auto& kv : w->user_ev) {
      tsb::DeviceGuard g(kv.first);
      cudaEventDestroy(kv.second);
    }
  }
  delete w;
}

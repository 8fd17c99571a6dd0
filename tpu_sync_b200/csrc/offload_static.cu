// Offload of KV blocks into caller-owned pinned host memory that allocates
// nothing on the device.
//
// Who needs this: a serving engine usually hands almost all of HBM to its own
// allocator up front (a KV pool sized by a memory-utilisation fraction, or a
// framework that preallocates the device), so a library that calls
// cudaMalloc for its staging either fails with out-of-memory or fragments the
// pool the engine manages; cudaMalloc / cudaFree can also synchronise the
// device, stalling the engine's in-flight work.  Such a caller cannot create a
// KVCacheManager (whose staging slots are cudaMalloc'ed), but it can call
// this entry point: the only staging it uses is the fixed array below.
//
// The scratch is a file-scope __device__ array of kStaticScratchBytes (64 MiB).
// Every GPU that loads this library holds that much device memory until the
// process exits.  Host code cannot use the array's name as a device address
// (in host code it is a host-side stand-in), so the address is looked up once
// per device with cudaGetSymbolAddress while that device is current: the
// first call on a device does this set-up, so make that first call before
// any stream capture begins.  The array is shared by every call on a device
// and keeps the previous call's contents; calls that overlap on the GPU (on
// different streams) race on it, so issue them on one stream or serialise
// them.

#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <vector>

#include "ts_internal.h"

namespace {
constexpr uint64_t kStaticScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;
}  // namespace

static __device__ __align__(256) uint8_t g_offload_scratch[kStaticScratchBytes];

namespace {

std::mutex g_scratch_mu;
uint8_t* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_offload_scratch on `device` (set-up on first use).
int scratch_address(int device, uint8_t** out) {
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (device < 0 || device >= kMaxDevices)
    return tsb::set_errorf(TS_INVALID_ARGUMENT, "device %d out of range", device);
  if (g_scratch_ptr[device] == nullptr) {
    tsb::DeviceGuard g(device);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_offload_scratch);
    if (e != cudaSuccess) return tsb::cuda_error(e, "cudaGetSymbolAddress of the static staging");
    g_scratch_ptr[device] = static_cast<uint8_t*>(p);
  }
  *out = g_scratch_ptr[device];
  return TS_OK;
}

}  // namespace

extern "C" int ts_kv_offload_noalloc(int device, const ts_block_storage* d_storages,
                                     int n_storages, const int64_t* src_ids,
                                     const int64_t* dst_ids, int64_t n_blocks,
                                     void* host_dst, uint64_t host_pitch,
                                     int64_t host_blocks, void* stream) {
  tsb::clear_error();
  if (n_blocks < 0 || n_storages < 0 || host_blocks < 0)
    return tsb::set_error(TS_INVALID_ARGUMENT, "counts must be non-negative");
  if (n_blocks == 0 || n_storages == 0) return TS_OK;
  if (!d_storages || !src_ids || !dst_ids || !host_dst)
    return tsb::set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  if (host_pitch == 0 || host_pitch % 16 != 0)
    return tsb::set_error(TS_INVALID_ARGUMENT, "host_pitch must be a positive multiple of 16");
  if (host_pitch > kStaticScratchBytes)
    return tsb::set_errorf(TS_OUT_OF_RANGE,
                           "block pitch of %llu bytes exceeds the static staging capacity "
                           "of %llu bytes",
                           (unsigned long long)host_pitch,
                           (unsigned long long)kStaticScratchBytes);
  // Storage table: alignment, largest block, shortest storage, slot coverage.
  std::vector<ts_block_storage> st(static_cast<size_t>(n_storages));
  tsb::DeviceGuard g(device);
  TS_CUDA_RET(cudaMemcpy(st.data(), d_storages, sizeof(ts_block_storage) * st.size(),
                         cudaMemcpyDeviceToHost),
              "read storage table");
  bool vec_ok = true;
  uint64_t max_bb = 0, covered = 0;
  int64_t dev_blocks = INT64_MAX;
  for (const ts_block_storage& s : st) {
    if (s.block_bytes == 0 || s.stage_off + s.block_bytes > host_pitch)
      return tsb::set_error(TS_INVALID_ARGUMENT, "storage slot outside the host block pitch");
    vec_ok = vec_ok && s.dev_ptr % 16 == 0 && s.block_bytes % 16 == 0 && s.stage_off % 16 == 0;
    max_bb = s.block_bytes > max_bb ? s.block_bytes : max_bb;
    covered += s.block_bytes;
    const int64_t nb = int64_t(s.dev_bytes / s.block_bytes);
    dev_blocks = nb < dev_blocks ? nb : dev_blocks;
  }
  for (int64_t k = 0; k < n_blocks; ++k) {
    if (src_ids[k] < 0 || src_ids[k] >= dev_blocks)
      return tsb::set_error(TS_INVALID_ARGUMENT, "Copy range exceeds source device buffer size");
    if (dst_ids[k] < 0 || dst_ids[k] >= host_blocks)
      return tsb::set_error(TS_INVALID_ARGUMENT, "Copy range exceeds destination host buffer size");
  }
  uint8_t* scratch = nullptr;
  int rc = scratch_address(device, &scratch);
  if (rc != TS_OK) return rc;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool has_gaps = covered < host_pitch;  // padding between / after slots
  int64_t chunk = int64_t(kStaticScratchBytes / host_pitch);
  if (chunk > tsb::kMaxParamIds) chunk = tsb::kMaxParamIds;
  uint8_t* host = static_cast<uint8_t*>(host_dst);
  for (int64_t c0 = 0; c0 < n_blocks; c0 += chunk) {
    const int64_t cn = n_blocks - c0 < chunk ? n_blocks - c0 : chunk;
    // Padding bytes would otherwise carry the previous call's data to the host.
    if (has_gaps)
      TS_CUDA_RET(cudaMemsetAsync(scratch, 0, size_t(cn) * host_pitch, s), "clear staging");
    tsb::ParamIds ids;
    ids.direct = 0;
    for (int64_t k = 0; k < cn; ++k) ids.v[k] = src_ids[c0 + k];
    rc = tsb::mgr_extract(device, d_storages, n_storages, ids, cn, scratch, host_pitch,
                          nullptr, s, vec_ok, max_bb, false, 0, 0);
    if (rc != TS_OK) return rc;
    // One DMA per run of consecutive host block ids (same stream: the next
    // chunk's gather waits for these copies).
    int64_t k = 0;
    while (k < cn) {
      int64_t e = k + 1;
      while (e < cn && dst_ids[c0 + e] == dst_ids[c0 + e - 1] + 1) ++e;
      TS_CUDA_RET(cudaMemcpyAsync(host + uint64_t(dst_ids[c0 + k]) * host_pitch,
                                  scratch + uint64_t(k) * host_pitch,
                                  size_t(e - k) * host_pitch, cudaMemcpyDeviceToHost, s),
                  "D2H DMA");
      k = e;
    }
  }
  return TS_OK;
}

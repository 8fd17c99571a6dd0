// Error plumbing, device queries and the pure host copy-spec logic.
//
// ts_validate_copy_spec restates ValidateOffsetsAndSizes
// (tpu_sync/kv_cache/kv_cache_manager_base.cc:72-102) with the same checks,
// order, codes and messages; ts_coalesce_runs restates CoalesceMajorDimCopies
// (tpu_sync/kv_cache/kv_cache_manager_base.cc:121-141).

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "ts_internal.h"

namespace tsb {
namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int set_errorf(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int cuda_error(cudaError_t e, const char* what) {
  const int code = e == cudaErrorMemoryAllocation ? TS_RESOURCE_EXHAUSTED : TS_INTERNAL;
  return set_errorf(code, "%s: CUDA error %d (%s)", what, int(e), cudaGetErrorString(e));
}

int sm_count(int device) {
  static std::mutex mu;
  static std::vector<int> cache;
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0) device = 0;
  if (size_t(device) >= cache.size()) cache.resize(device + 1, 0);
  if (cache[device] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n <= 0)
      n = 148;
    cache[device] = n;
  }
  return cache[device];
}

}  // namespace tsb

extern "C" const char* ts_last_error(void) { return tsb::g_last_error.c_str(); }

extern "C" const char* ts_version(void) { return "tpusync_b200 0.1.0 (sm_100a)"; }

extern "C" int ts_validate_copy_spec(const int64_t* src, int64_t n_src,
                                     const int64_t* dst, int64_t n_dst,
                                     const int64_t* sizes, int64_t n_sizes) {
  tsb::clear_error();
  if (n_src < 0 || n_dst < 0 || n_sizes < 0)
    return tsb::set_error(TS_INVALID_ARGUMENT, "list lengths must be non-negative");
  if (n_dst != 0 && n_src != n_dst)
    return tsb::set_error(TS_INVALID_ARGUMENT,
                          "src_offsets, dst_offsets, and sizes must have the same length");
  if (n_sizes != 0 && n_src != n_sizes)
    return tsb::set_error(TS_INVALID_ARGUMENT,
                          "src_offsets, dst_offsets, and sizes must have the same length");
  for (int64_t i = 0; i < n_src; ++i)
    if (src[i] < 0)
      return tsb::set_error(TS_INVALID_ARGUMENT, "copy offsets and sizes must be non-negative");
  for (int64_t i = 0; i < n_dst; ++i)
    if (dst[i] < 0)
      return tsb::set_error(TS_INVALID_ARGUMENT, "copy offsets and sizes must be non-negative");
  for (int64_t i = 0; i < n_sizes; ++i)
    if (sizes[i] < 0)
      return tsb::set_error(TS_INVALID_ARGUMENT, "copy offsets and sizes must be non-negative");
  return TS_OK;
}

extern "C" int ts_coalesce_runs(const int64_t* src, const int64_t* dst,
                                const int64_t* sizes, int64_t n, int64_t* out_src,
                                int64_t* out_dst, int64_t* out_sizes,
                                int64_t* n_out) {
  tsb::clear_error();
  if (!n_out) return tsb::set_error(TS_INVALID_ARGUMENT, "n_out must not be null");
  int64_t m = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (m > 0 && src[i] == out_src[m - 1] + out_sizes[m - 1] &&
        dst[i] == out_dst[m - 1] + out_sizes[m - 1]) {
      out_sizes[m - 1] += sizes[i];
    } else {
      out_src[m] = src[i];
      out_dst[m] = dst[i];
      out_sizes[m] = sizes[i];
      ++m;
    }
  }
  *n_out = m;
  return TS_OK;
}

extern "C" int ts_enable_peer_access(int device, int peer) {
  tsb::clear_error();
  if (device == peer) return TS_OK;
  int can = 0;
  TS_CUDA_RET(cudaDeviceCanAccessPeer(&can, device, peer), "peer query");
  if (!can) return tsb::set_errorf(TS_UNAVAILABLE, "device %d cannot access device %d", device, peer);
  tsb::DeviceGuard g(device);
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();  // clear the sticky-free "already enabled" status
    return TS_OK;
  }
  TS_CUDA_RET(e, "enable peer access");
  return TS_OK;
}

namespace {
// Process-wide IPC mappings by (device, handle): CUDA opens a handle once per
// device in a process, so every user shares one mapping, reference-counted.
std::mutex g_ipc_mu;
std::map<std::pair<int, std::string>, std::pair<void*, int>> g_ipc;  // base, references
}  // namespace

extern "C" int ts_ipc_open(int device, const void* handle_bytes, void** base_out) {
  tsb::clear_error();
  if (!handle_bytes || !base_out) return tsb::set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  cudaIpcMemHandle_t h;
  static_assert(sizeof(h) == 64, "cudaIpcMemHandle_t is 64 bytes");
  std::memcpy(&h, handle_bytes, sizeof(h));
  const auto key = std::make_pair(device, std::string(static_cast<const char*>(handle_bytes), 64));
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  auto it = g_ipc.find(key);
  if (it != g_ipc.end()) {
    ++it->second.second;
    *base_out = it->second.first;
    return TS_OK;
  }
  tsb::DeviceGuard g(device);
  void* p = nullptr;
  TS_CUDA_RET(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  g_ipc.emplace(key, std::make_pair(p, 1));
  *base_out = p;
  return TS_OK;
}

extern "C" int ts_ipc_close(int device, void* base) {
  tsb::clear_error();
  std::lock_guard<std::mutex> lock(g_ipc_mu);
  for (auto it = g_ipc.begin(); it != g_ipc.end(); ++it) {
    if (it->first.first != device || it->second.first != base) continue;
    if (--it->second.second > 0) return TS_OK;
    g_ipc.erase(it);
    tsb::DeviceGuard g(device);
    TS_CUDA_RET(cudaIpcCloseMemHandle(base), "cudaIpcCloseMemHandle");
    return TS_OK;
  }
  return tsb::set_error(TS_NOT_FOUND, "no such IPC mapping on this device");
}

extern "C" int ts_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
  tsb::clear_error();
  if (!dev_ptr || !handle_out || !offset_out)
    return tsb::set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  // Allocation base through the driver entry point (no link-time libcuda).
  using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static AddressRangeFn range_fn = nullptr;
  if (range_fn == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    TS_CUDA_RET(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q),
                "driver entry point");
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return tsb::set_error(TS_UNAVAILABLE, "cuMemGetAddressRange is not available");
    range_fn = reinterpret_cast<AddressRangeFn>(fn);
  }
  cudaPointerAttributes attr;
  TS_CUDA_RET(cudaPointerGetAttributes(&attr, dev_ptr), "pointer attributes");
  if (attr.type != cudaMemoryTypeDevice)
    return tsb::set_error(TS_INVALID_ARGUMENT, "ipc export needs device memory");
  tsb::DeviceGuard g(attr.device);
  CUdeviceptr base = 0;
  size_t size = 0;
  const CUresult r = range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr));
  if (r != CUDA_SUCCESS)
    return tsb::set_errorf(TS_INTERNAL, "cuMemGetAddressRange failed (%d)", int(r));
  cudaIpcMemHandle_t h;
  TS_CUDA_RET(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = uint64_t(reinterpret_cast<uintptr_t>(dev_ptr) - uintptr_t(base));
  return TS_OK;
}

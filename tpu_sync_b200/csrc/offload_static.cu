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
// this entry point: the only staging it uses is the fixed array below, and it
// takes its storage table in HOST memory (a caller that cannot allocate
// device memory has nowhere to put one), passed to the gather kernel by value.
//
// The scratch is a file-scope __device__ array of kStaticScratchBytes (64 MiB).
// Every GPU that loads this library holds that much device memory until the
// process exits.  Host code cannot use the array's name as a device address
// (in host code it is a host-side stand-in), so every call looks the address
// up with cudaGetSymbolAddress while the call's device is current (the first
// lookup on a device also loads this library's device code there).  The array
// is shared by every call on a device and keeps the previous call's contents:
// padding between storage slots is cleared at the start of each call, and
// calls that overlap on the GPU (on different streams) race on the array, so
// issue them on one stream or serialise them.

#include <cuda_runtime.h>

#include <cstdint>

#include "ts_internal.h"

namespace {
constexpr uint64_t kStaticScratchBytes = 64ull << 20;
constexpr int kMaxTableStorages = 512;     // storages per call (kernel parameters)
constexpr int kThreads = 256;
constexpr uint64_t kPieceBytes = uint64_t(kThreads) * 4 * 16;  // 16 KiB per CTA item
}  // namespace

static __device__ __align__(256) uint8_t g_offload_scratch[kStaticScratchBytes];

namespace {

// Everything one gather launch needs, by value in the kernel parameters
// (about 18.5 KB of the 32 KB parameter space).
struct GatherArgs {
  ts_block_storage st[kMaxTableStorages];
  int64_t ids[tsb::kMaxParamIds];
  uint8_t* scratch;
  uint64_t pitch;
  int32_t n_st;
  int32_t n_blocks;
  uint32_t ppu;  // 16 KiB pieces per (block, storage) unit, for the largest block
  int32_t vec;   // every address, size and offset is a multiple of 16
};

// scratch[k*pitch + st[s].stage_off + b] = storage s block ids[k] byte b: the
// extract gather of the manager-free path, one 16 KiB piece per CTA item,
// 16-byte vectors (all loads of a thread before its stores) or bytes.  Ids
// were range-checked on the host.
__global__ void __launch_bounds__(kThreads) noalloc_gather_kernel(const __grid_constant__ GatherArgs a) {
  const int64_t items = int64_t(a.n_blocks) * a.n_st * a.ppu;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int64_t unit = w / a.ppu;
    const uint64_t piece = uint64_t(w - unit * a.ppu);
    const int k = int(unit / a.n_st);
    const int s = int(unit - int64_t(k) * a.n_st);
    const ts_block_storage& e = a.st[s];
    const uint64_t off = piece * kPieceBytes;
    if (off >= e.block_bytes) continue;
    const uint64_t rem = e.block_bytes - off;
    const uint64_t nbytes = rem < kPieceBytes ? rem : kPieceBytes;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(e.dev_ptr) +
                         uint64_t(a.ids[k]) * e.block_bytes + off;
    uint8_t* dst = a.scratch + uint64_t(k) * a.pitch + e.stage_off + off;
    if (a.vec) {
      const int nvec = int(nbytes >> 4);
      int4 v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        if (idx < nvec) v[i] = __ldcs(reinterpret_cast<const int4*>(src) + idx);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        if (idx < nvec) reinterpret_cast<int4*>(dst)[idx] = v[i];
      }
    } else {
      for (uint64_t b = threadIdx.x; b < nbytes; b += kThreads) dst[b] = src[b];
    }
  }
}

}  // namespace

extern "C" int ts_kv_offload_noalloc(int device, const ts_block_storage* storages,
                                     int n_storages, const int64_t* src_ids,
                                     const int64_t* dst_ids, int64_t n_blocks,
                                     void* host_dst, uint64_t host_pitch,
                                     int64_t host_blocks, void* stream) {
  tsb::clear_error();
  if (n_blocks < 0 || n_storages < 0 || host_blocks < 0)
    return tsb::set_error(TS_INVALID_ARGUMENT, "counts must be non-negative");
  if (n_blocks == 0 || n_storages == 0) return TS_OK;
  if (!storages || !src_ids || !dst_ids || !host_dst)
    return tsb::set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  if (n_storages > kMaxTableStorages)
    return tsb::set_errorf(TS_OUT_OF_RANGE, "%d storages exceed the %d one call can take",
                           n_storages, kMaxTableStorages);
  if (host_pitch == 0 || host_pitch % 16 != 0)
    return tsb::set_error(TS_INVALID_ARGUMENT, "host_pitch must be a positive multiple of 16");
  if (host_pitch > kStaticScratchBytes)
    return tsb::set_errorf(TS_OUT_OF_RANGE,
                           "block pitch of %llu bytes exceeds the static staging capacity "
                           "of %llu bytes",
                           (unsigned long long)host_pitch,
                           (unsigned long long)kStaticScratchBytes);
  // Storage table (host memory): slots inside the pitch, alignment, largest
  // block, the shortest storage (for the id check) and the bytes it covers.
  GatherArgs a;
  bool vec = true;
  uint64_t max_bb = 0, covered = 0;
  int64_t dev_blocks = INT64_MAX;
  for (int i = 0; i < n_storages; ++i) {
    const ts_block_storage& s = storages[i];
    if (s.block_bytes == 0 || s.stage_off + s.block_bytes > host_pitch)
      return tsb::set_error(TS_INVALID_ARGUMENT, "storage slot outside the host block pitch");
    vec = vec && s.dev_ptr % 16 == 0 && s.block_bytes % 16 == 0 && s.stage_off % 16 == 0;
    max_bb = s.block_bytes > max_bb ? s.block_bytes : max_bb;
    covered += s.block_bytes;
    const int64_t nb = int64_t(s.dev_bytes / s.block_bytes);
    dev_blocks = nb < dev_blocks ? nb : dev_blocks;
    a.st[i] = s;
  }
  for (int64_t k = 0; k < n_blocks; ++k) {
    if (src_ids[k] < 0 || src_ids[k] >= dev_blocks)
      return tsb::set_error(TS_INVALID_ARGUMENT, "Copy range exceeds source device buffer size");
    if (dst_ids[k] < 0 || dst_ids[k] >= host_blocks)
      return tsb::set_error(TS_INVALID_ARGUMENT, "Copy range exceeds destination host buffer size");
  }
  tsb::DeviceGuard g(device);
  void* sym = nullptr;
  TS_CUDA_RET(cudaGetSymbolAddress(&sym, g_offload_scratch),
              "cudaGetSymbolAddress of the static staging");
  uint8_t* scratch = static_cast<uint8_t*>(sym);

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int64_t chunk = int64_t(kStaticScratchBytes / host_pitch);
  if (chunk > tsb::kMaxParamIds) chunk = tsb::kMaxParamIds;
  // Padding bytes between / after the slots would otherwise carry an earlier
  // call's data to the host; gathers only write slots, so one clear of the
  // rows this call uses covers all of its chunks.
  if (covered < host_pitch) {
    const int64_t rows = n_blocks < chunk ? n_blocks : chunk;
    TS_CUDA_RET(cudaMemsetAsync(scratch, 0, size_t(rows) * host_pitch, s), "clear staging");
  }
  a.scratch = scratch;
  a.pitch = host_pitch;
  a.n_st = n_storages;
  a.ppu = uint32_t((max_bb + kPieceBytes - 1) / kPieceBytes);
  a.vec = vec ? 1 : 0;
  const int64_t wave = int64_t(tsb::sm_count(device)) * 8;
  uint8_t* host = static_cast<uint8_t*>(host_dst);
  for (int64_t c0 = 0; c0 < n_blocks; c0 += chunk) {
    const int64_t cn = n_blocks - c0 < chunk ? n_blocks - c0 : chunk;
    for (int64_t k = 0; k < cn; ++k) a.ids[k] = src_ids[c0 + k];
    a.n_blocks = int32_t(cn);
    const int64_t items = cn * n_storages * int64_t(a.ppu);
    const int grid = int(items < wave ? items : wave);
    // Same stream: this gather starts after the previous chunk's DMAs have
    // read the scratch rows it overwrites.
    noalloc_gather_kernel<<<grid, kThreads, 0, s>>>(a);
    TS_CUDA_RET(cudaGetLastError(), "gather launch");
    // One DMA per run of consecutive host block ids.
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

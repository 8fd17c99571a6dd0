// Internal helpers shared by the C-ABI translation units.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "tpusync_b200.h"

namespace tsb {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
int set_errorf(int code, const char* fmt, ...);
void clear_error();

// Maps a CUDA runtime error to a ts_status (and records the message).
int cuda_error(cudaError_t e, const char* what);

// Number of SMs of `device` (cached).
int sm_count(int device);

// Block ids passed by value in kernel parameters (one pipelined chunk):
// dev(k) = device block id of the k-th block, stage(k) = its block index in
// the staging buffer (k) or, in direct mode, its host-tier block id (the
// kernel then reads / writes the mapped host tier itself).
constexpr int kMaxParamIds = 256;
struct ParamIds {
  int64_t v[kMaxParamIds];
  int64_t s[kMaxParamIds];
  int32_t direct;
#ifdef __CUDACC__
  __device__ __forceinline__ int64_t dev(int64_t k) const { return v[k]; }
  __device__ __forceinline__ int64_t stage(int64_t k) const { return direct ? s[k] : k; }
#endif
};

// Chunk launchers of kv_block_kernels.cu used by the manager.  max_ctas caps
// the grid (0 = a full wave of every SM); max_ctas < 0 launches one CTA per
// work item (16 KiB piece) instead of a persistent grid (plain copies only).
// variant picks the plain-copy kernel: kCopyVec (16-byte vectors), kCopyBulk
// (the bulk-copy kernel, both sides device memory) or kCopyWide (32-byte
// vectors, every address and size a multiple of 32); ignored for fp8, and
// the byte kernel runs for tables that are not 16-byte aligned.
enum CopyVariant : int { kCopyVec = 0, kCopyBulk = 1, kCopyWide = 2 };
int mgr_extract(int device, const ts_block_storage* d_st, int n_st,
                const ParamIds& ids, int64_t n_blocks, void* staging,
                uint64_t pitch, int* err_flag, cudaStream_t s, bool vec_ok,
                uint64_t max_bb, bool fp8, uint64_t scale_off, int max_ctas, int variant);
int mgr_insert(int device, const ts_block_storage* d_st, int n_st,
               const ParamIds& ids, int64_t n_blocks, const void* staging,
               uint64_t pitch, int* err_flag, cudaStream_t s, bool vec_ok,
               uint64_t max_bb, bool fp8, uint64_t scale_off, int max_ctas, int variant);

// Strided byte runs for seg_copy (seg_copy.cu): row r of `count` rows of
// `bytes` bytes goes from src + r*src_stride to dst + r*dst_stride.  src / dst
// are addresses the launching device can access (its memory, mapped host
// memory, or a peer's memory with peer access enabled).
struct SegTask {
  uint64_t src;
  uint64_t dst;
  int64_t src_stride;
  int64_t dst_stride;
  uint32_t bytes;
  uint32_t count;
};
constexpr int kMaxSegTasks = 512;  // tasks per launch (kernel parameters)
int seg_copy(int device, const SegTask* tasks, int64_t n, cudaStream_t s, int max_ctas);

// NUMA placement (numa.cu).  pci_numa_node: the node sysfs lists for a PCI
// bus id (CUDA's "00000000:1b:00.0" or "0000:1b:00.0"), -1 when unknown;
// sysfs_root NULL = "/sys".  numa_node_count: nodes under
// <root>/devices/system/node (1 when unreadable).  device_numa_node: the
// node of a CUDA device's PCI function.
int pci_numa_node(const char* bus_id, const char* sysfs_root);
int numa_node_count(const char* sysfs_root);
int device_numa_node(int device);

// While alive, the calling thread's memory policy prefers `node` (pages it
// faults in, including those a cudaHostAlloc / cudaHostRegister pins, come
// from that node when it has room); the previous policy is restored after.
// applied() is false when the kernel refused the policy.
class ScopedPreferredNode {
 public:
  explicit ScopedPreferredNode(int node);
  ~ScopedPreferredNode();
  bool applied() const { return applied_; }

 private:
  static constexpr int kMaskWords = 16;
  bool applied_ = false;
  int prev_mode_ = 0;
  unsigned long prev_mask_[kMaskWords] = {0};
};

// Scoped switch of the current CUDA device.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (prev_ != device) cudaSetDevice(device);
    dev_ = device;
  }
  ~DeviceGuard() {
    if (prev_ != dev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0;
  int dev_ = 0;
};

}  // namespace tsb

#define TS_CUDA_RET(expr, what)                      \
  do {                                               \
    cudaError_t _e = (expr);                         \
    if (_e != cudaSuccess) return tsb::cuda_error(_e, what); \
  } while (0)

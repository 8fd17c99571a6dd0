// Segment copy: one launch moves any list of strided byte runs.
//
// A task is `count` rows of `bytes` bytes: row r goes from src + r*src_stride
// to dst + r*dst_stride.  Addresses are generic: device memory, the mapped
// pinned host tier (SM-driven PCIe reads / writes) or a peer GPU's memory.
// It executes the partial-region pool copies of the manager (live extents
// that are not whole blocks) and the pool reshard plans' (src block, dst
// block, offset, size) entries.
//
// Work split: every row is cut into pieces of at most 4 KiB; one warp copies
// one piece.  Tasks travel by value in the kernel parameters (up to
// kMaxSegTasks per launch) with an exclusive prefix of their piece counts; a
// warp finds its task by binary search over that prefix.  A piece moves with
// 16-byte vectors when the task's addresses, strides and row size are all
// 16-byte multiples (all eight loads of a lane issued before its stores),
// else with 4-byte words, else bytes.

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "ts_internal.h"

namespace tsb {
namespace {

constexpr int kSegThreads = 256;
constexpr uint32_t kSegPiece = 4096;

struct SegBatch {
  SegTask t[kMaxSegTasks];
  uint32_t first[kMaxSegTasks + 1];  // exclusive prefix of pieces
  uint8_t align[kMaxSegTasks];       // 16, 4 or 1
  int32_t n;
};

__device__ __forceinline__ void copy_piece(const uint8_t* __restrict__ src,
                                           uint8_t* __restrict__ dst, uint32_t len, int align,
                                           int lane) {
  if (align == 16) {
    const int nvec = int(len >> 4);  // <= 256
    int4 v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) v[i] = *reinterpret_cast<const int4*>(src + (k << 4));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int k = lane + 32 * i;
      if (k < nvec) *reinterpret_cast<int4*>(dst + (k << 4)) = v[i];
    }
  } else if (align == 4) {
    const int nw = int(len >> 2);  // <= 1024
    for (int base = 0; base < nw; base += 256) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = base + lane + 32 * i;
        if (k < nw) w[i] = *reinterpret_cast<const uint32_t*>(src + (k << 2));
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int k = base + lane + 32 * i;
        if (k < nw) *reinterpret_cast<uint32_t*>(dst + (k << 2)) = w[i];
      }
    }
  } else {
    for (uint32_t k = uint32_t(lane); k < len; k += 32) dst[k] = src[k];
  }
}

__global__ void __launch_bounds__(kSegThreads) seg_copy_kernel(const __grid_constant__ SegBatch b) {
  const int lane = threadIdx.x & 31;
  const uint32_t warp = (blockIdx.x * uint32_t(kSegThreads) + threadIdx.x) >> 5;
  const uint32_t nwarps = (gridDim.x * uint32_t(kSegThreads)) >> 5;
  const uint32_t total = b.first[b.n];
  for (uint32_t p = warp; p < total; p += nwarps) {
    int lo = 0, hi = b.n - 1;  // last task with first <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (b.first[mid] <= p) lo = mid; else hi = mid - 1;
    }
    const SegTask& t = b.t[lo];
    const uint32_t per_row = (t.bytes + kSegPiece - 1) / kSegPiece;
    const uint32_t local = p - b.first[lo];
    const uint32_t row = local / per_row;
    const uint32_t off = (local - row * per_row) * kSegPiece;
    const uint32_t len = min(kSegPiece, t.bytes - off);
    const uint8_t* src =
        reinterpret_cast<const uint8_t*>(t.src + uint64_t(int64_t(row) * t.src_stride) + off);
    uint8_t* dst = reinterpret_cast<uint8_t*>(t.dst + uint64_t(int64_t(row) * t.dst_stride) + off);
    copy_piece(src, dst, len, b.align[lo], lane);
  }
}

int task_align(const SegTask& t) {
  const uint64_t bits = t.src | t.dst | uint64_t(t.src_stride) | uint64_t(t.dst_stride) |
                        uint64_t(t.bytes);
  if ((bits & 15) == 0) return 16;
  if ((bits & 3) == 0) return 4;
  return 1;
}

}  // namespace

int seg_copy(int device, const SegTask* tasks, int64_t n, cudaStream_t s, int max_ctas) {
  if (n <= 0) return TS_OK;
  // Split tasks by rows so none exceeds 2^24 pieces; a launch then takes
  // whole tasks while its piece count stays within 2^30 (uint32 prefix).
  constexpr uint64_t kTaskPieces = uint64_t(1) << 24;
  constexpr uint64_t kLaunchPieces = uint64_t(1) << 30;
  std::vector<SegTask> work;
  work.reserve(size_t(n));
  for (int64_t i = 0; i < n; ++i) {
    SegTask t = tasks[i];
    if (t.bytes == 0 || t.count == 0) continue;
    const uint64_t per_row = (uint64_t(t.bytes) + kSegPiece - 1) / kSegPiece;
    const uint64_t rows_max = std::max<uint64_t>(1, kTaskPieces / per_row);
    while (t.count > 0) {
      SegTask h = t;
      h.count = uint32_t(std::min<uint64_t>(t.count, rows_max));
      work.push_back(h);
      t.src += uint64_t(int64_t(h.count) * t.src_stride);
      t.dst += uint64_t(int64_t(h.count) * t.dst_stride);
      t.count -= h.count;
    }
  }
  int ctas_cap = sm_count(device) * 4;  // 64 registers / thread: 4 CTAs resident per SM
  if (max_ctas > 0) ctas_cap = std::min(ctas_cap, max_ctas);
  SegBatch* b = new SegBatch();
  int rc = TS_OK;
  size_t i = 0;
  while (i < work.size() && rc == TS_OK) {
    b->n = 0;
    uint64_t pieces = 0;
    while (i < work.size() && b->n < kMaxSegTasks) {
      const SegTask& t = work[i];
      const uint64_t tp = (uint64_t(t.bytes) + kSegPiece - 1) / kSegPiece * t.count;
      if (pieces + tp > kLaunchPieces) break;
      b->first[b->n] = uint32_t(pieces);
      b->align[b->n] = uint8_t(task_align(t));
      b->t[b->n++] = t;
      pieces += tp;
      ++i;
    }
    b->first[b->n] = uint32_t(pieces);
    const uint64_t want = (pieces + (kSegThreads / 32) - 1) / (kSegThreads / 32);
    const int ctas = int(std::max<uint64_t>(1, std::min<uint64_t>(want, uint64_t(ctas_cap))));
    seg_copy_kernel<<<ctas, kSegThreads, 0, s>>>(*b);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = cuda_error(e, "segment copy launch");
  }
  delete b;
  return rc;
}

}  // namespace tsb

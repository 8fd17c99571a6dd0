// Weight-sync reshard pushed by the copy engines.
//
// The SM path (ts_reshard_copy) casts fp32 -> bf16 and stores straight into
// the peer's memory; NVLink stores issued by the SMs top out near 0.92 of
// the copy engines' peer copy on this platform.  This program splits the
// work: the reshard kernel casts every chunk into a local staging buffer
// (rows packed back to back, HBM-bound), and the copy engines move each
// staged chunk to its destination with one cudaMemcpy2DAsync (strided rows
// when the destination is strided).  Chunks are cut into groups; group g's
// copies start as soon as its cast has finished, while later groups are
// still being cast, so the push runs at the copy engines' NVLink rate plus
// the first group's cast.  Same-dtype chunks skip the cast and the staging.
//
// Replaces, for one source GPU, the reference's per-layer D2H + TCP push of
// strided chunks + receiver H2D (WeightSynchronizerBase::PushWeightsResharded,
// tpu_sync/weight_sync/weight_synchronizer_base.cc:558-760).

#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "ts_internal.h"

using tsb::set_error;
using tsb::set_errorf;

namespace {

constexpr int kDmaStreams = 2;

struct Copy2D {
  void* dst;
  size_t dpitch;
  const void* src;
  size_t spitch;
  size_t width;   // bytes per row
  size_t height;  // rows
};

int elem_size(int dtype) {
  switch (dtype) {
    case TS_DTYPE_U8: return 1;
    case TS_DTYPE_BF16: return 2;
    case TS_DTYPE_F16: return 2;
    case TS_DTYPE_F32: return 4;
    default: return 0;
  }
}

}  // namespace

struct ts_reshard_ce {
  int device = 0;
  int src_dtype = 0, dst_dtype = 0;
  bool cast = false;
  uint8_t* staging = nullptr;
  uint64_t staging_bytes = 0;
  struct Group {
    ts_reshard_chunk* d_chunks = nullptr;  // cast chunks (into the staging)
    int64_t* d_prefix = nullptr;
    int64_t n_chunks = 0, n_items = 0;
    std::vector<Copy2D> dmas;
    cudaEvent_t cast_done = nullptr, dma_done = nullptr;
  };
  std::vector<Group> groups;
  cudaStream_t dma[kDmaStreams] = {};
  cudaEvent_t start = nullptr, join = nullptr;
};

namespace {

void release(ts_reshard_ce* p) {
  tsb::DeviceGuard g(p->device);
  for (auto& gr : p->groups) {
    if (gr.d_chunks) cudaFree(gr.d_chunks);
    if (gr.d_prefix) cudaFree(gr.d_prefix);
    if (gr.cast_done) cudaEventDestroy(gr.cast_done);
    if (gr.dma_done) cudaEventDestroy(gr.dma_done);
  }
  for (cudaStream_t s : p->dma)
    if (s) cudaStreamDestroy(s);
  if (p->start) cudaEventDestroy(p->start);
  if (p->join) cudaEventDestroy(p->join);
  if (p->staging) cudaFree(p->staging);
  delete p;
}

}  // namespace

extern "C" int ts_reshard_ce_create(int device, const ts_reshard_chunk* chunks, int64_t n,
                                    int src_dtype, int dst_dtype, int n_groups,
                                    ts_reshard_ce** out) {
  tsb::clear_error();
  if (!out || n < 0 || (n > 0 && !chunks)) return set_error(TS_INVALID_ARGUMENT, "invalid arguments");
  *out = nullptr;
  const int es_src = elem_size(src_dtype), es_dst = elem_size(dst_dtype);
  if (es_src == 0 || es_dst == 0) return set_error(TS_INVALID_ARGUMENT, "unknown dtype");
  const bool cast = src_dtype != dst_dtype;
  if (cast && !(src_dtype == TS_DTYPE_F32 && dst_dtype == TS_DTYPE_BF16))
    return set_error(TS_UNIMPLEMENTED, "only identity and f32->bf16 reshards are supported");
  if (n_groups <= 0) n_groups = 1;
  for (int64_t i = 0; i < n; ++i) {
    const ts_reshard_chunk& c = chunks[i];
    if (c.size < 0 || c.count < 0 || c.src_off < 0 || c.dst_off < 0 || c.src_stride < 0 ||
        c.dst_stride < 0 || (c.count > 1 && (c.src_stride < c.size || c.dst_stride < c.size)))
      return set_errorf(TS_INVALID_ARGUMENT, "chunk %lld: negative fields or rows that overlap",
                        (long long)i);
  }
  auto* p = new ts_reshard_ce();
  p->device = device;
  p->src_dtype = src_dtype;
  p->dst_dtype = dst_dtype;
  p->cast = cast;
  tsb::DeviceGuard g(device);
  // packed staging offsets (elements of the destination dtype)
  std::vector<int64_t> packed(size_t(n) + 1, 0);
  for (int64_t i = 0; i < n; ++i)
    packed[size_t(i) + 1] = packed[size_t(i)] + chunks[i].size * std::max<int64_t>(chunks[i].count, 0);
  const uint64_t total_bytes = uint64_t(packed[size_t(n)]) * uint64_t(es_dst);
  cudaError_t ce = cudaSuccess;
  if (cast && total_bytes > 0) {
    p->staging_bytes = total_bytes;
    ce = cudaMalloc(&p->staging, total_bytes);
    if (ce != cudaSuccess) {
      release(p);
      return tsb::cuda_error(ce, "reshard staging");
    }
  }
  // groups of about equal bytes, in chunk order
  const uint64_t target = std::max<uint64_t>(1, total_bytes / uint64_t(n_groups));
  int64_t i0 = 0;
  while (i0 < n) {
    int64_t i1 = i0;
    uint64_t bytes = 0;
    while (i1 < n && (bytes < target || i1 == i0)) {
      bytes += uint64_t(chunks[i1].size * std::max<int64_t>(chunks[i1].count, 0)) * uint64_t(es_dst);
      ++i1;
    }
    ts_reshard_ce::Group gr;
    std::vector<ts_reshard_chunk> cast_chunks;
    for (int64_t i = i0; i < i1; ++i) {
      const ts_reshard_chunk& c = chunks[i];
      if (c.size == 0 || c.count == 0) continue;
      const size_t width = size_t(c.size) * size_t(es_dst);
      Copy2D d;
      d.dst = reinterpret_cast<uint8_t*>(c.dst_ptr) + uint64_t(c.dst_off) * uint64_t(es_dst);
      d.dpitch = c.count > 1 ? size_t(c.dst_stride) * size_t(es_dst) : width;
      if (cast) {
        ts_reshard_chunk k = c;
        k.dst_ptr = reinterpret_cast<uint64_t>(p->staging);
        k.dst_off = packed[size_t(i)];
        k.dst_stride = c.size;  // rows packed back to back
        cast_chunks.push_back(k);
        d.src = p->staging + uint64_t(packed[size_t(i)]) * uint64_t(es_dst);
        d.spitch = width;
      } else {
        d.src = reinterpret_cast<const uint8_t*>(c.src_ptr) + uint64_t(c.src_off) * uint64_t(es_src);
        d.spitch = c.count > 1 ? size_t(c.src_stride) * size_t(es_src) : width;
      }
      d.width = width;
      d.height = size_t(c.count);
      if (d.height > 1 && d.spitch == width && d.dpitch == width) {  // contiguous both sides
        d.width = width * d.height;
        d.height = 1;
      }
      gr.dmas.push_back(d);
    }
    if (!cast_chunks.empty()) {
      gr.n_chunks = int64_t(cast_chunks.size());
      std::vector<int64_t> prefix(cast_chunks.size() + 1);
      int rc = ts_reshard_work_items(cast_chunks.data(), gr.n_chunks, src_dtype, dst_dtype,
                                     prefix.data());
      if (rc != TS_OK) {
        p->groups.push_back(gr);
        release(p);
        return rc;
      }
      gr.n_items = prefix.back();
      ce = cudaMalloc(&gr.d_chunks, sizeof(ts_reshard_chunk) * cast_chunks.size());
      if (ce == cudaSuccess) ce = cudaMalloc(&gr.d_prefix, sizeof(int64_t) * prefix.size());
      if (ce == cudaSuccess)
        ce = cudaMemcpy(gr.d_chunks, cast_chunks.data(), sizeof(ts_reshard_chunk) * cast_chunks.size(),
                        cudaMemcpyHostToDevice);
      if (ce == cudaSuccess)
        ce = cudaMemcpy(gr.d_prefix, prefix.data(), sizeof(int64_t) * prefix.size(),
                        cudaMemcpyHostToDevice);
    }
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&gr.cast_done, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&gr.dma_done, cudaEventDisableTiming);
    p->groups.push_back(gr);
    if (ce != cudaSuccess) {
      release(p);
      return tsb::cuda_error(ce, "reshard copy-engine program");
    }
    i0 = i1;
  }
  for (int k = 0; k < kDmaStreams && ce == cudaSuccess; ++k)
    ce = cudaStreamCreateWithFlags(&p->dma[k], cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->start, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&p->join, cudaEventDisableTiming);
  if (ce != cudaSuccess) {
    release(p);
    return tsb::cuda_error(ce, "reshard copy-engine streams");
  }
  *out = p;
  return TS_OK;
}

extern "C" int ts_reshard_ce_launch(ts_reshard_ce* p, void* stream) {
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null program");
  tsb::DeviceGuard g(p->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  TS_CUDA_RET(cudaEventRecord(p->start, s), "event record");
  for (cudaStream_t d : p->dma) TS_CUDA_RET(cudaStreamWaitEvent(d, p->start, 0), "stream wait");
  for (size_t gi = 0; gi < p->groups.size(); ++gi) {
    ts_reshard_ce::Group& gr = p->groups[gi];
    cudaStream_t d = p->dma[gi % kDmaStreams];
    if (gr.n_chunks > 0) {
      // the previous launch's copies of this group have left the staging
      TS_CUDA_RET(cudaStreamWaitEvent(s, gr.dma_done, 0), "stream wait");
      int rc = ts_reshard_copy(p->device, gr.d_chunks, gr.d_prefix, gr.n_chunks, gr.n_items,
                               p->src_dtype, p->dst_dtype, s);
      if (rc != TS_OK) return rc;
      TS_CUDA_RET(cudaEventRecord(gr.cast_done, s), "event record");
      TS_CUDA_RET(cudaStreamWaitEvent(d, gr.cast_done, 0), "stream wait");
    }
    for (const Copy2D& c : gr.dmas) {
      if (c.height == 1) {
        TS_CUDA_RET(cudaMemcpyAsync(c.dst, c.src, c.width, cudaMemcpyDefault, d), "chunk copy");
      } else {
        TS_CUDA_RET(cudaMemcpy2DAsync(c.dst, c.dpitch, c.src, c.spitch, c.width, c.height,
                                      cudaMemcpyDefault, d),
                    "strided chunk copy");
      }
    }
    TS_CUDA_RET(cudaEventRecord(gr.dma_done, d), "event record");
  }
  // the caller's stream continues once every copy stream is through
  for (cudaStream_t d : p->dma) {
    TS_CUDA_RET(cudaEventRecord(p->join, d), "event record");
    TS_CUDA_RET(cudaStreamWaitEvent(s, p->join, 0), "stream wait");
  }
  return TS_OK;
}

extern "C" int ts_reshard_ce_info(ts_reshard_ce* p, int64_t* groups, uint64_t* staging_bytes,
                                  int64_t* copies) {
  tsb::clear_error();
  if (!p) return set_error(TS_INVALID_ARGUMENT, "null program");
  int64_t nc = 0;
  for (const auto& gr : p->groups) nc += int64_t(gr.dmas.size());
  if (groups) *groups = int64_t(p->groups.size());
  if (staging_bytes) *staging_bytes = p->staging_bytes;
  if (copies) *copies = nc;
  return TS_OK;
}

extern "C" int ts_reshard_ce_destroy(ts_reshard_ce* p) {
  if (!p) return TS_OK;
  {
    tsb::DeviceGuard g(p->device);
    for (cudaStream_t d : p->dma)
      if (d) cudaStreamSynchronize(d);
  }
  release(p);
  return TS_OK;
}

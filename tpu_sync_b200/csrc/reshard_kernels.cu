// Weight-sync reshard executor (strided chunk copy with optional fp32 -> bf16
// cast) and the paged-KV relayout kernel of the prefill -> decode hand-off.
//
// Reshard: the reference expands each ShardPushEntryProto into `count`
// copies of `size` bytes at src_off + c*src_stride -> dst_off + c*dst_stride
// (tpu_sync/weight_sync/weight_synchronizer_base.cc:606-667) and pushes each
// copy over TCP into the peer's host buffer, followed by an H2D there.  Here
// the chunks execute as one kernel that reads the local shard in HBM and
// stores straight into the destination tensor, which may live on a peer GPU
// (P2P stores over NVLink through a peer-mapped pointer).  Work is flattened
// over (chunk, row, 8-element vector); per CTA work item 256 threads x 4
// vectors, all four loads of a thread issued before its stores, on a
// persistent grid of as many CTAs as fit on the SMs at once.  Loads use
// 16-byte vectors when the chunk's rows are 16-byte aligned on both sides,
// else a scalar path.  Bound: NVLink (peer) or HBM.
//
// Relayout: destination-block-centric copy of 16-byte vectors of head
// vectors between two page geometries (tokens per block, head-major or
// token-major), using per-sequence block tables on both sides.

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "ts_internal.h"

namespace tsb {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr int kCtasPerSm = 8;

__device__ __forceinline__ int4 ld_nc(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_v4(void* p, const int4& v) {
  asm volatile("st.global.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat16 a = __float2bfloat16_rn(lo);
  const __nv_bfloat16 b = __float2bfloat16_rn(hi);
  return uint32_t(__bfloat16_as_ushort(a)) | (uint32_t(__bfloat16_as_ushort(b)) << 16);
}

// Element transfer policies.  VEC elements per vector step.
// Element transfer policies: load() one vector of VEC elements into
// registers, store() it (converted) to the destination.
struct CopyBytes {  // raw bytes: 16 per vector
  static constexpr int VEC = 16;
  static constexpr int SRC_ES = 1;
  static constexpr int DST_ES = 1;
  using Reg = int4;
  __device__ static Reg load(const uint8_t* s) { return ld_nc(s); }
  __device__ static void store(uint8_t* d, const Reg& v) { st_v4(d, v); }
  __device__ static void one(const uint8_t* s, uint8_t* d) { *d = *s; }
};

struct F32ToBf16 {  // 8 floats (32 B) -> 8 bf16 (16 B)
  static constexpr int VEC = 8;
  static constexpr int SRC_ES = 4;
  static constexpr int DST_ES = 2;
  struct Reg {
    int4 a, b;
  };
  __device__ static Reg load(const uint8_t* s) { return Reg{ld_nc(s), ld_nc(s + 16)}; }
  __device__ static void store(uint8_t* d, const Reg& v) {
    int4 o;
    o.x = int(pack_bf16x2(__int_as_float(v.a.x), __int_as_float(v.a.y)));
    o.y = int(pack_bf16x2(__int_as_float(v.a.z), __int_as_float(v.a.w)));
    o.z = int(pack_bf16x2(__int_as_float(v.b.x), __int_as_float(v.b.y)));
    o.w = int(pack_bf16x2(__int_as_float(v.b.z), __int_as_float(v.b.w)));
    st_v4(d, o);
  }
  __device__ static void one(const uint8_t* s, uint8_t* d) {
    *reinterpret_cast<__nv_bfloat16*>(d) =
        __float2bfloat16_rn(*reinterpret_cast<const float*>(s));
  }
};

// `scale` converts chunk element units into transfer elements (element size
// of an identity copy when it runs as bytes).
template <typename P>
__global__ void __launch_bounds__(kThreads)
    reshard_kernel(const ts_reshard_chunk* __restrict__ chunks,
                   const int64_t* __restrict__ prefix, int64_t n_chunks,
                   int64_t n_items, int64_t scale) {
  int64_t lo = 0;  // chunk of this CTA's previous item (prefix[lo] <= w)
  for (int64_t w = blockIdx.x; w < n_items; w += gridDim.x) {
    // chunk c with prefix[c] <= w < prefix[c+1]: the previous item's chunk,
    // or a binary search over the chunks after it (a CTA's items grow)
    if (prefix[lo + 1] <= w) {
      int64_t hi = n_chunks;
      ++lo;
      while (hi - lo > 1) {
        const int64_t mid = (lo + hi) >> 1;
        if (prefix[mid] <= w) lo = mid; else hi = mid;
      }
    }
    const ts_reshard_chunk c = chunks[lo];
    const int64_t size = c.size * scale;
    const int64_t src_off = c.src_off * scale, dst_off = c.dst_off * scale;
    const int64_t src_stride = c.src_stride * scale, dst_stride = c.dst_stride * scale;
    const uint8_t* src = reinterpret_cast<const uint8_t*>(c.src_ptr);
    uint8_t* dst = reinterpret_cast<uint8_t*>(c.dst_ptr);
    const int64_t vpr = (size + P::VEC - 1) / P::VEC;  // vectors per row
    const int64_t total = vpr * c.count;
    const uint64_t a_src = c.src_ptr + uint64_t(src_off) * P::SRC_ES;
    const uint64_t a_dst = c.dst_ptr + uint64_t(dst_off) * P::DST_ES;
    const bool aligned = ((a_src | (uint64_t(src_stride) * P::SRC_ES)) & 15u) == 0 &&
                         ((a_dst | (uint64_t(dst_stride) * P::DST_ES)) & 15u) == 0;
    const int64_t g0 = (w - prefix[lo]) * int64_t(kThreads) * kVecPerThread;
    // every vector load of the thread is issued before its first store
    // (kVecPerThread loads in flight: what hides NVLink latency when the
    // source is a peer's memory)
    typename P::Reg v[kVecPerThread];
    uint8_t* dv[kVecPerThread];
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i) {
      dv[i] = nullptr;
      const int64_t g = g0 + threadIdx.x + int64_t(i) * kThreads;
      if (g >= total) continue;
      const int64_t row = g / vpr;
      const int64_t e0 = (g - row * vpr) * P::VEC;
      const int64_t n = size - e0 < P::VEC ? size - e0 : P::VEC;
      const uint8_t* s = src + (src_off + row * src_stride + e0) * P::SRC_ES;
      uint8_t* d = dst + (dst_off + row * dst_stride + e0) * P::DST_ES;
      if (aligned && n == P::VEC) {
        v[i] = P::load(s);
        dv[i] = d;
      } else {
        for (int64_t e = 0; e < n; ++e) P::one(s + e * P::SRC_ES, d + e * P::DST_ES);
      }
    }
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i)
      if (dv[i] != nullptr) P::store(dv[i], v[i]);
  }
}

int64_t items_for(const ts_reshard_chunk& c, int vec_elems, int64_t scale) {
  if (c.count <= 0 || c.size <= 0) return 0;
  const int64_t size = c.size * scale;
  const int64_t vpr = (size + vec_elems - 1) / vec_elems;
  const int64_t per_item = int64_t(kThreads) * kVecPerThread;
  return (vpr * c.count + per_item - 1) / per_item;
}

int es_of(int dtype) {
  switch (dtype) {
    case TS_DTYPE_U8: return 1;
    case TS_DTYPE_BF16: return 2;
    case TS_DTYPE_F16: return 2;
    case TS_DTYPE_F32: return 4;
    default: return 0;
  }
}

// ---------------------------------------------------------------------------
// Relayout
// ---------------------------------------------------------------------------

constexpr int kRelayoutVecPerThread = 8;
constexpr uint32_t kSkip = 0xFFFFFFFFu;  // no store (16-byte offsets never equal it)

// Index arithmetic of the relayout: 32-bit division by the page geometry, or
// shifts and masks when every divisor is a power of two (all real KV
// layouts: vectors per head vector, heads, tokens per page).
template <bool kPow2>
struct Div32 {
  uint32_t d, shift;
  __device__ __forceinline__ uint32_t div(uint32_t x) const { return kPow2 ? x >> shift : x / d; }
};

template <bool kPow2>
__global__ void __launch_bounds__(kThreads, 4)
    relayout_kernel(const uint64_t* __restrict__ src_bases,
                    const uint64_t* __restrict__ dst_bases, int n_st,
                    ts_page_geometry sg, ts_page_geometry dg,
                    const int32_t* __restrict__ src_table, int64_t src_ts,
                    const int32_t* __restrict__ dst_table, int64_t dst_ts,
                    int64_t n_seqs, int64_t seq_tokens, int64_t dst_blocks_per_seq,
                    int64_t src_pages, int64_t dst_pages, int* err) {
  // Token, head and vector indices fit 32 bits (checked on the host), so the
  // per-vector divisions are 32-bit.
  const uint32_t vph = uint32_t(sg.head_bytes >> 4);       // 16-byte vectors per head vector
  const uint32_t vpt = vph * uint32_t(dg.heads);           // vectors per token
  const uint32_t sbt = uint32_t(sg.block_tokens);
  const Div32<kPow2> by_vph{vph, uint32_t(__ffs(vph) - 1)};
  const Div32<kPow2> by_vpt{vpt, uint32_t(__ffs(vpt) - 1)};
  const Div32<kPow2> by_sbt{sbt, uint32_t(__ffs(sbt) - 1)};
  const int64_t src_block_bytes = sg.block_tokens * sg.heads * sg.head_bytes;
  const int64_t dst_block_bytes = dg.block_tokens * dg.heads * dg.head_bytes;
  const int64_t items = int64_t(n_st) * n_seqs * dst_blocks_per_seq;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int64_t jb = w % dst_blocks_per_seq;
    const int64_t sq = w / dst_blocks_per_seq;
    const int64_t q = sq % n_seqs;
    const int s = int(sq / n_seqs);
    const int64_t t0 = jb * dg.block_tokens;
    int64_t nt = seq_tokens - t0;
    if (nt > dg.block_tokens) nt = dg.block_tokens;
    const uint32_t nvec = uint32_t(nt) * vpt;
    const int64_t dbi = dst_table[q * dst_ts + jb];
    if (dbi < 0 || dbi >= dst_pages) {  // the whole destination page is skipped
      if (err != nullptr && threadIdx.x == 0) *reinterpret_cast<volatile int*>(err) = 1;
      continue;
    }
    const uint8_t* sbase = reinterpret_cast<const uint8_t*>(src_bases[s]);
    uint8_t* dblk = reinterpret_cast<uint8_t*>(dst_bases[s]) + dbi * dst_block_bytes;
    const int32_t* srow = src_table + q * src_ts;
    for (uint32_t base = 0; base < nvec; base += uint32_t(kThreads) * kRelayoutVecPerThread) {
      int4 v[kRelayoutVecPerThread];
      uint32_t doff[kRelayoutVecPerThread];  // byte offset in the dst page; kSkip = none
#pragma unroll
      for (int i = 0; i < kRelayoutVecPerThread; ++i) {
        const uint32_t g = base + threadIdx.x + uint32_t(i) * kThreads;
        doff[i] = kSkip;
        if (g < nvec) {
          const uint32_t tl = by_vpt.div(g);        // token within dst block
          const uint32_t r = g - tl * vpt;
          const uint32_t h = by_vph.div(r);
          const uint32_t vv = r - h * vph;
          const uint32_t t = uint32_t(t0) + tl;     // token within sequence
          const uint32_t sbi = by_sbt.div(t);
          const uint32_t st = t - sbi * sbt;
          const int64_t sb = srow[sbi];
          if (sb < 0 || sb >= src_pages) {
            if (err != nullptr) *reinterpret_cast<volatile int*>(err) = 1;
            continue;
          }
          const uint32_t so = sg.head_major ? (h * sbt + st) : (st * uint32_t(sg.heads) + h);
          const uint32_t dpos = dg.head_major ? (h * uint32_t(dg.block_tokens) + tl)
                                              : (tl * uint32_t(dg.heads) + h);
          v[i] = ld_nc(sbase + sb * src_block_bytes + int64_t(so) * sg.head_bytes +
                       (int64_t(vv) << 4));
          doff[i] = dpos * uint32_t(dg.head_bytes) + (vv << 4);
        }
      }
#pragma unroll
      for (int i = 0; i < kRelayoutVecPerThread; ++i)
        if (doff[i] != kSkip) st_v4(dblk + doff[i], v[i]);
    }
  }
}

// Fast path for power-of-two geometries whose token (heads x head vectors)
// fits the CTA: a thread keeps one (head, 16-byte vector) of the token for
// the whole page and steps through tokens, so per vector it only derives the
// token's source page and position (shifts and masks) and issues the load.
// lv = log2(vectors per head vector), lh = log2(heads), ls / ld = log2(tokens
// per source / destination page).
__global__ void __launch_bounds__(kThreads, 4)
    relayout_pow2_kernel(const uint64_t* __restrict__ src_bases,
                         const uint64_t* __restrict__ dst_bases, int n_st,
                         int src_head_major, int dst_head_major, uint32_t lv, uint32_t lh,
                         uint32_t ls, uint32_t ld,
                         const int32_t* __restrict__ src_table, int64_t src_ts,
                         const int32_t* __restrict__ dst_table, int64_t dst_ts,
                         int64_t n_seqs, int64_t seq_tokens, int64_t dst_blocks_per_seq,
                         int64_t src_pages, int64_t dst_pages, int* err) {
  const uint32_t lhb = lv + 4;                        // log2(head bytes)
  const uint32_t tshift = lv + lh;                    // log2(vectors per token)
  const uint32_t tstep = uint32_t(kThreads) >> tshift;  // tokens per step of the CTA
  const uint32_t r = threadIdx.x & ((1u << tshift) - 1);
  const uint32_t h = r >> lv;
  const uint32_t voff = (r & ((1u << lv) - 1)) << 4;  // byte offset in the head vector
  const uint32_t tl0 = threadIdx.x >> tshift;
  const int64_t src_block_bytes = int64_t(1) << (ls + lh + lhb);
  const int64_t dst_block_bytes = int64_t(1) << (ld + lh + lhb);
  const uint32_t dbt = 1u << ld;
  // Two page-id buffers used alternately: a tile's writes go to the buffer
  // whose readers (two tiles back) all passed the previous tile's barrier,
  // so one barrier per tile suffices.
  __shared__ int32_t spage_buf[2][kThreads];
  uint32_t parity = 0;
  const int64_t items = int64_t(n_st) * n_seqs * dst_blocks_per_seq;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    const int64_t jb = w % dst_blocks_per_seq;
    const int64_t sq = w / dst_blocks_per_seq;
    const int64_t q = sq % n_seqs;
    const int s = int(sq / n_seqs);
    const int64_t t0 = jb << ld;
    const uint32_t nt = uint32_t(seq_tokens - t0 < int64_t(dbt) ? seq_tokens - t0 : dbt);
    const int64_t dbi = dst_table[q * dst_ts + jb];
    if (dbi < 0 || dbi >= dst_pages) {
      if (err != nullptr && threadIdx.x == 0) *reinterpret_cast<volatile int*>(err) = 1;
      continue;
    }
    const uint8_t* sbase = reinterpret_cast<const uint8_t*>(src_bases[s]);
    uint8_t* dblk = reinterpret_cast<uint8_t*>(dst_bases[s]) + dbi * dst_block_bytes;
    const int32_t* srow = src_table + q * src_ts;
    const uint32_t tile = tstep * kRelayoutVecPerThread;  // tokens per step of the CTA
    for (uint32_t tb = 0; tb < nt; tb += tile) {
      // The tile's source page ids, loaded once into shared memory so that
      // the data loads below do not wait on a dependent table load.
      const uint32_t first = (uint32_t(t0) + tb) >> ls;
      const uint32_t last = (uint32_t(t0) + min(tb + tile, nt) - 1) >> ls;
      int32_t* spage = spage_buf[parity];
      parity ^= 1u;
      if (threadIdx.x <= last - first) spage[threadIdx.x] = srow[first + threadIdx.x];
      __syncthreads();
      int4 v[kRelayoutVecPerThread];
      uint32_t doff[kRelayoutVecPerThread];
#pragma unroll
      for (int i = 0; i < kRelayoutVecPerThread; ++i) {
        const uint32_t tl = tb + tl0 + uint32_t(i) * tstep;  // token within the dst page
        doff[i] = kSkip;
        if (tl < nt) {
          const uint32_t t = uint32_t(t0) + tl;
          const int64_t sb = spage[(t >> ls) - first];
          if (sb < 0 || sb >= src_pages) {
            if (err != nullptr) *reinterpret_cast<volatile int*>(err) = 1;
            continue;
          }
          const uint32_t st = t & ((1u << ls) - 1);
          const uint32_t so = src_head_major ? ((h << ls) + st) : ((st << lh) + h);
          const uint32_t dpos = dst_head_major ? ((h << ld) + tl) : ((tl << lh) + h);
          v[i] = ld_nc(sbase + sb * src_block_bytes + (int64_t(so) << lhb) + voff);
          doff[i] = (dpos << lhb) + voff;
        }
      }
#pragma unroll
      for (int i = 0; i < kRelayoutVecPerThread; ++i)
        if (doff[i] != kSkip) st_v4(dblk + doff[i], v[i]);
    }
  }
}

}  // namespace
}  // namespace tsb

using tsb::set_error;

extern "C" int ts_reshard_work_items(const ts_reshard_chunk* h_chunks,
                                     int64_t n_chunks, int src_dtype,
                                     int dst_dtype, int64_t* h_prefix_out) {
  tsb::clear_error();
  if (n_chunks < 0 || !h_prefix_out || (n_chunks > 0 && !h_chunks))
    return set_error(TS_INVALID_ARGUMENT, "bad chunk list");
  const int es = tsb::es_of(src_dtype);
  if (es == 0 || tsb::es_of(dst_dtype) == 0) return set_error(TS_INVALID_ARGUMENT, "unknown dtype");
  // Must match the kernel's vector width: 16 bytes for identity copies,
  // 8 elements for the f32 -> bf16 cast.
  const bool identity = src_dtype == dst_dtype;
  const int vec = identity ? 16 : 8;
  const int64_t scale = identity ? es : 1;
  h_prefix_out[0] = 0;
  for (int64_t i = 0; i < n_chunks; ++i) {
    const ts_reshard_chunk& c = h_chunks[i];
    if (c.src_off < 0 || c.dst_off < 0 || c.size < 0 || c.src_stride < 0 ||
        c.dst_stride < 0 || c.count < 0)
      return set_error(TS_INVALID_ARGUMENT, "copy offsets and sizes must be non-negative");
    h_prefix_out[i + 1] = h_prefix_out[i] + tsb::items_for(c, vec, scale);
  }
  return TS_OK;
}

extern "C" int ts_reshard_copy(int device, const ts_reshard_chunk* d_chunks,
                               const int64_t* d_item_prefix, int64_t n_chunks,
                               int64_t n_items, int src_dtype, int dst_dtype,
                               void* stream) {
  tsb::clear_error();
  if (n_chunks == 0 || n_items == 0) return TS_OK;
  if (!d_chunks || !d_item_prefix) return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  const int es = tsb::es_of(src_dtype);
  if (es == 0 || tsb::es_of(dst_dtype) == 0) return set_error(TS_INVALID_ARGUMENT, "unknown dtype");
  tsb::DeviceGuard g(device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // a persistent grid: the CTAs that fit on the SMs at once
  auto grid_for = [&](const void* fn) {
    static int per_sm[2] = {0, 0};
    int& occ = per_sm[fn == reinterpret_cast<const void*>(tsb::reshard_kernel<tsb::CopyBytes>)];
    if (occ == 0 && cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, tsb::kThreads, 0) !=
                        cudaSuccess)
      occ = 4;
    const int64_t cap = int64_t(tsb::sm_count(device)) * (occ > 0 ? occ : 1);
    return int(n_items < cap ? n_items : cap);
  };
  if (src_dtype == dst_dtype) {
    // Identity copies run as raw bytes: chunk element units scaled by es.
    const int grid = grid_for(reinterpret_cast<const void*>(tsb::reshard_kernel<tsb::CopyBytes>));
    tsb::reshard_kernel<tsb::CopyBytes><<<grid, tsb::kThreads, 0, s>>>(
        d_chunks, d_item_prefix, n_chunks, n_items, es);
  } else if (src_dtype == TS_DTYPE_F32 && dst_dtype == TS_DTYPE_BF16) {
    const int grid = grid_for(reinterpret_cast<const void*>(tsb::reshard_kernel<tsb::F32ToBf16>));
    tsb::reshard_kernel<tsb::F32ToBf16><<<grid, tsb::kThreads, 0, s>>>(
        d_chunks, d_item_prefix, n_chunks, n_items, 1);
  } else {
    return set_error(TS_UNIMPLEMENTED, "only identity and f32->bf16 reshards are supported");
  }
  TS_CUDA_RET(cudaGetLastError(), "reshard launch");
  return TS_OK;
}

extern "C" int ts_kv_relayout(int device, const uint64_t* d_src_bases,
                              const uint64_t* d_dst_bases, int n_storages,
                              ts_page_geometry src, ts_page_geometry dst,
                              const int32_t* d_src_table, int64_t src_table_stride,
                              const int32_t* d_dst_table, int64_t dst_table_stride,
                              int64_t n_seqs, int64_t seq_tokens, int64_t src_pages,
                              int64_t dst_pages, int* d_err, void* stream) {
  tsb::clear_error();
  if (n_storages < 0 || n_seqs < 0 || seq_tokens < 0 || src_pages < 0 || dst_pages < 0)
    return set_error(TS_INVALID_ARGUMENT, "counts must be non-negative");
  if (n_storages == 0 || n_seqs == 0 || seq_tokens == 0) return TS_OK;
  if (src.heads != dst.heads || src.head_bytes != dst.head_bytes)
    return set_error(TS_INVALID_ARGUMENT, "source and destination must have the same heads and head bytes");
  if (src.block_tokens <= 0 || dst.block_tokens <= 0 || src.heads <= 0 ||
      src.head_bytes <= 0 || (src.head_bytes & 15) != 0)
    return set_error(TS_INVALID_ARGUMENT, "page geometry needs positive sizes and 16-byte head vectors");
  if (!d_src_bases || !d_dst_bases || !d_src_table || !d_dst_table)
    return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  const int64_t vectors_per_block =
      dst.block_tokens * dst.heads * (src.head_bytes >> 4);
  if (seq_tokens > INT32_MAX || vectors_per_block > INT32_MAX ||
      src.block_tokens > INT32_MAX || src.heads * src.block_tokens > INT32_MAX ||
      dst.block_tokens * dst.heads * dst.head_bytes > int64_t(UINT32_MAX) - 16)
    return set_error(TS_INVALID_ARGUMENT, "sequence or page too large for the relayout kernel");
  const int64_t dst_blocks_per_seq = (seq_tokens + dst.block_tokens - 1) / dst.block_tokens;
  const int64_t items = int64_t(n_storages) * n_seqs * dst_blocks_per_seq;
  tsb::DeviceGuard g(device);
  const int64_t cap = int64_t(tsb::sm_count(device)) * tsb::kCtasPerSm;
  const int grid = int(items < cap ? items : cap);
  auto pow2 = [](int64_t v) { return v > 0 && (v & (v - 1)) == 0; };
  auto lg = [](int64_t v) { uint32_t l = 0; while ((int64_t(1) << l) < v) ++l; return l; };
  const bool p2 = pow2(src.head_bytes >> 4) && pow2(src.heads) && pow2(src.block_tokens);
  // the fast kernel stages a tile's source page ids in kThreads entries: a
  // tile of (kThreads / vectors per token) * vectors-per-thread tokens spans
  // at most tile / src.block_tokens + 2 pages
  const int64_t vpt = (src.head_bytes >> 4) * src.heads;
  const int64_t tile = vpt <= tsb::kThreads ? (tsb::kThreads / vpt) * tsb::kRelayoutVecPerThread : 0;
  if (p2 && pow2(dst.block_tokens) && vpt <= tsb::kThreads &&
      tile / src.block_tokens + 2 <= tsb::kThreads) {
    tsb::relayout_pow2_kernel<<<grid, tsb::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        d_src_bases, d_dst_bases, n_storages, src.head_major != 0, dst.head_major != 0,
        lg(src.head_bytes >> 4), lg(src.heads), lg(src.block_tokens), lg(dst.block_tokens),
        d_src_table, src_table_stride, d_dst_table, dst_table_stride, n_seqs, seq_tokens,
        dst_blocks_per_seq, src_pages, dst_pages, d_err);
    TS_CUDA_RET(cudaGetLastError(), "relayout launch");
    return TS_OK;
  }
  auto kernel = p2 ? tsb::relayout_kernel<true> : tsb::relayout_kernel<false>;
  kernel<<<grid, tsb::kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_src_bases, d_dst_bases, n_storages, src, dst, d_src_table, src_table_stride,
      d_dst_table, dst_table_stride, n_seqs, seq_tokens, dst_blocks_per_seq, src_pages,
      dst_pages, d_err);
  TS_CUDA_RET(cudaGetLastError(), "relayout launch");
  return TS_OK;
}

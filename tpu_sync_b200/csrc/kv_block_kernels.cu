// Block extract (gather) / insert (scatter) kernels between paged KV storages
// in HBM and a block-major staging buffer, plus the fused bf16 <-> fp8 e4m3
// variants.
//
// Semantics: the reference copies, per (layer, shard) storage and per
// coalesced run, bytes [src*bb, +n*bb) of the device buffer to host offset
// dst*bb (tpu_sync/kv_cache/kv_cache_manager_base.cc:2036-2124, inverse at
// :1945-2033).  Here one launch moves whole blocks of every storage at once:
// work unit = (block k, storage s) = one contiguous run of bb_s bytes, split
// into 16 KiB pieces; one CTA copies one piece with 16-byte vector accesses,
// all loads of a thread issued before its stores (64 B in flight per thread).
// The grid is persistent: a multiple of the SM count, grid-striding over the
// pieces.  Nothing here is a contraction, so no tensor cores are used; the
// bound is HBM bandwidth (read bb + write bb per unit).

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "ts_internal.h"

namespace tsb {
namespace {

constexpr int kThreads = 256;
constexpr int kVecPerThread = 4;
constexpr uint64_t kPieceBytes = uint64_t(kThreads) * kVecPerThread * 16;  // 16 KiB
constexpr int kCtasPerSm = 8;

// Block ids come from a device array (manager-free entry points) or by value
// inside the kernel parameters (the manager's pipelined chunks: the launch
// snapshots them, so no device id buffer or host->device id copy is needed).
struct DevIds {
  const int64_t* p;
  __device__ __forceinline__ int64_t dev(int64_t k) const { return p[k]; }
  __device__ __forceinline__ int64_t stage(int64_t k) const { return k; }
};

__device__ __forceinline__ int4 ld_stream(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_vec(void* p, const int4& v) {
  asm volatile("st.global.v4.s32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Resolves work item w into (block k, storage s, piece).  Returns false when
// the piece lies past the end of the storage's block (heterogeneous storages)
// or the block id is out of bounds (err_flag set).
struct Unit {
  uint8_t* dev;
  uint8_t* stg;
  uint64_t nbytes;
};

template <typename Ids>
__device__ __forceinline__ bool resolve(const ts_block_storage* __restrict__ st,
                                        int n_st, const Ids& ids,
                                        uint8_t* staging, uint64_t pitch,
                                        uint32_t ppu, int64_t w, int* err_flag,
                                        Unit* u) {
  const int64_t unit = w / ppu;
  const uint64_t piece = uint64_t(w - unit * ppu);
  const int64_t k = unit / n_st;
  const int s = int(unit - k * n_st);
  const uint64_t bb = st[s].block_bytes;
  const uint64_t off = piece * kPieceBytes;
  if (off >= bb) return false;
  const int64_t id = ids.dev(k);
  const uint64_t dev_off = uint64_t(id) * bb;
  if (id < 0 || dev_off + bb > st[s].dev_bytes) {
    // lane 0 of every warp: the bulk kernel resolves pieces on lane 0 only
    if (err_flag != nullptr && (threadIdx.x & 31) == 0)
      *reinterpret_cast<volatile int*>(err_flag) = 1;
    return false;
  }
  u->dev = reinterpret_cast<uint8_t*>(st[s].dev_ptr) + dev_off + off;
  u->stg = staging + uint64_t(ids.stage(k)) * pitch + st[s].stage_off + off;
  const uint64_t rem = bb - off;
  u->nbytes = rem < kPieceBytes ? rem : kPieceBytes;
  return true;
}

// 16-byte vector path: every block_bytes, stage_off, pitch and base address is
// a multiple of 16 (checked on the host before choosing this kernel).
template <bool kToStaging, typename Ids>
__global__ void __launch_bounds__(kThreads)
    block_copy_vec_kernel(const ts_block_storage* __restrict__ st, int n_st,
                          const __grid_constant__ Ids ids, int64_t n_blocks,
                          uint8_t* staging, uint64_t pitch, uint32_t ppu,
                          int* err_flag) {
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    Unit u;
    if (!resolve(st, n_st, ids, staging, pitch, ppu, w, err_flag, &u)) continue;
    const uint8_t* src = kToStaging ? u.dev : u.stg;
    uint8_t* dst = kToStaging ? u.stg : u.dev;
    const int nvec = int(u.nbytes >> 4);
    int4 v[kVecPerThread];
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < nvec) v[i] = ld_stream(src + (uint64_t(idx) << 4));
    }
#pragma unroll
    for (int i = 0; i < kVecPerThread; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < nvec) st_vec(dst + (uint64_t(idx) << 4), v[i]);
    }
  }
}

// Byte path for storages whose sizes or addresses are not 16-byte multiples.
template <bool kToStaging, typename Ids>
__global__ void __launch_bounds__(kThreads)
    block_copy_byte_kernel(const ts_block_storage* __restrict__ st, int n_st,
                           const __grid_constant__ Ids ids, int64_t n_blocks,
                           uint8_t* staging, uint64_t pitch, uint32_t ppu,
                           int* err_flag) {
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    Unit u;
    if (!resolve(st, n_st, ids, staging, pitch, ppu, w, err_flag, &u)) continue;
    const uint8_t* src = kToStaging ? u.dev : u.stg;
    uint8_t* dst = kToStaging ? u.stg : u.dev;
    for (uint64_t b = threadIdx.x; b < u.nbytes; b += kThreads) dst[b] = src[b];
  }
}

// 32-byte vector path (sm_100 256-bit loads and stores): every address,
// block size, slot offset and pitch is a multiple of 32 (checked on the host
// before choosing this kernel); each thread moves two 32-byte vectors of a
// 16 KiB piece, both loads before its stores, the loads asking L2 to fetch
// 256-byte spans (.L2::256B).  Used for the direct reload, whose loads read
// the mapped host tier over PCIe.
__device__ __forceinline__ void ld_wide(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}

__device__ __forceinline__ void st_wide(void* p, const uint32_t (&r)[8]) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

constexpr int kWidePerThread = int(kPieceBytes / 32 / kThreads);  // 2

template <bool kToStaging, typename Ids>
__global__ void __launch_bounds__(kThreads)
    block_copy_wide_kernel(const ts_block_storage* __restrict__ st, int n_st,
                           const __grid_constant__ Ids ids, int64_t n_blocks,
                           uint8_t* staging, uint64_t pitch, uint32_t ppu,
                           int* err_flag) {
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    Unit u;
    if (!resolve(st, n_st, ids, staging, pitch, ppu, w, err_flag, &u)) continue;
    const uint8_t* src = kToStaging ? u.dev : u.stg;
    uint8_t* dst = kToStaging ? u.stg : u.dev;
    const int nvec = int(u.nbytes >> 5);
    uint32_t v[kWidePerThread][8];
#pragma unroll
    for (int i = 0; i < kWidePerThread; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < nvec) ld_wide(src + (uint64_t(idx) << 5), v[i]);
    }
#pragma unroll
    for (int i = 0; i < kWidePerThread; ++i) {
      const int idx = threadIdx.x + i * kThreads;
      if (idx < nvec) st_wide(dst + (uint64_t(idx) << 5), v[i]);
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy variant (HBM -> HBM only): each warp's lane 0 moves 16 KiB pieces
// with the Blackwell bulk-copy engine, global -> shared (completion counted
// on an mbarrier) then shared -> global (bulk async-group), two shared-memory
// buffers per warp so the next piece's load overlaps the current piece's
// store.  Six warps per CTA and one CTA per SM keep up to twelve 16 KiB loads
// in flight per SM in 192 KiB of shared memory while occupying 6 of the SM's
// 64 warp slots, so the gather can run beside another kernel that holds most
// of the SM.  Plain single-CTA copies of this GPU's own memory only;
// every address and size is a multiple of 16 (the caller checks vec_ok).
// Each wait on a load is bounded: past ~2^32 cycles the warp stops, records
// 3 in err_flag, waits for its issued stores and leaves.
// ---------------------------------------------------------------------------

constexpr int kBulkWarps = 6;
constexpr int kBulkBufs = 2;
constexpr uint32_t kBulkSmem = uint32_t(kBulkWarps) * kBulkBufs * uint32_t(kPieceBytes);

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void bulk_load(uint32_t dst_smem, const void* src, uint32_t bytes,
                                          uint32_t bar) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n\t"
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%2], [%3], %1, [%0];"
      ::"r"(bar), "r"(bytes), "r"(dst_smem), "l"(src)
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, uint32_t src_smem, uint32_t bytes) {
  asm volatile(
      "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
      "cp.async.bulk.commit_group;"
      ::"l"(dst), "r"(src_smem), "r"(bytes)
      : "memory");
}

__device__ __forceinline__ void bulk_wait_reads_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// True once the mbarrier's phase `parity` completed; false after ~2^32 cycles.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > (1ll << 32)) return false;
  }
}

template <bool kToStaging, typename Ids>
__global__ void __launch_bounds__(kBulkWarps * 32, 1)
    block_copy_bulk_kernel(const ts_block_storage* __restrict__ st, int n_st,
                           const __grid_constant__ Ids ids, int64_t n_blocks,
                           uint8_t* staging, uint64_t pitch, uint32_t ppu, int* err_flag) {
  extern __shared__ __align__(128) uint8_t bulk_smem[];
  __shared__ __align__(8) uint64_t bars[kBulkWarps][kBulkBufs];
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) != 0) return;  // one issuing lane per warp
  uint32_t bar[kBulkBufs], buf[kBulkBufs], phase[kBulkBufs];
  for (int b = 0; b < kBulkBufs; ++b) {
    bar[b] = smem_u32(&bars[warp][b]);
    buf[b] = smem_u32(bulk_smem + (size_t(warp) * kBulkBufs + b) * kPieceBytes);
    phase[b] = 0;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar[b]) : "memory");
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  const int64_t stride = int64_t(gridDim.x) * kBulkWarps;
  int64_t w = int64_t(blockIdx.x) * kBulkWarps + warp;
  // next valid piece at or after w (pieces past a block's end and blocks
  // whose id is out of range are skipped, the latter flagged by resolve)
  auto next = [&](Unit* u) {
    while (w < items) {
      const bool ok = resolve(st, n_st, ids, staging, pitch, ppu, w, err_flag, u);
      w += stride;
      if (ok) return true;
    }
    return false;
  };
  Unit cur, nxt;
  if (!next(&cur)) return;
  int b = 0;
  bulk_load(buf[b], kToStaging ? cur.dev : cur.stg, uint32_t(cur.nbytes), bar[b]);
  for (;;) {
    const bool more = next(&nxt);
    if (more) {
      // the other buffer's last store must have read it out of shared memory
      bulk_wait_reads_all();
      bulk_load(buf[b ^ 1], kToStaging ? nxt.dev : nxt.stg, uint32_t(nxt.nbytes), bar[b ^ 1]);
    }
    if (!bar_wait(bar[b], phase[b])) {
      if (err_flag != nullptr) *reinterpret_cast<volatile int*>(err_flag) = 3;
      if (more) bar_wait(bar[b ^ 1], phase[b ^ 1]);  // the next piece's load (bounded)
      break;
    }
    phase[b] ^= 1;
    bulk_store(kToStaging ? cur.stg : cur.dev, buf[b], uint32_t(cur.nbytes));
    if (!more) break;
    cur = nxt;
    b ^= 1;
  }
  bulk_wait_all();
}

// ---------------------------------------------------------------------------
// Manager-free entry points with a device-resident storage table: every CTA
// first scans the (small, L2-resident) table for the largest block and for
// 16-byte alignment, so the host never reads the table back (no blocking
// copy on the launch path).
// ---------------------------------------------------------------------------

struct TableScan {
  uint64_t max_bb;
  bool aligned;  // every dev_ptr, block_bytes, stage_off (and pitch, staging) % 16 == 0
};

__device__ __forceinline__ TableScan scan_table(const ts_block_storage* __restrict__ st,
                                                int n_st, uint64_t extra_align) {
  __shared__ unsigned long long s_max;
  __shared__ int s_bad;
  if (threadIdx.x == 0) {
    s_max = 0;
    s_bad = (extra_align & 15u) != 0;
  }
  __syncthreads();
  unsigned long long m = 0;
  int bad = 0;
  for (int i = threadIdx.x; i < n_st; i += blockDim.x) {
    const ts_block_storage e = st[i];
    m = e.block_bytes > m ? e.block_bytes : m;
    bad |= ((e.dev_ptr | e.block_bytes | e.stage_off) & 15u) != 0;
  }
  if (m) atomicMax(&s_max, m);
  if (bad) atomicOr(&s_bad, 1);
  __syncthreads();
  return TableScan{s_max, s_bad == 0};
}

template <bool kToStaging>
__global__ void __launch_bounds__(kThreads)
    block_copy_scan_kernel(const ts_block_storage* __restrict__ st, int n_st,
                           const int64_t* __restrict__ d_ids, int64_t n_blocks,
                           uint8_t* staging, uint64_t pitch, int* err_flag) {
  const TableScan t = scan_table(st, n_st, pitch | reinterpret_cast<uint64_t>(staging));
  const uint32_t ppu = uint32_t((t.max_bb + kPieceBytes - 1) / kPieceBytes);
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  const DevIds ids{d_ids};
  for (int64_t w = blockIdx.x; w < items; w += gridDim.x) {
    Unit u;
    if (!resolve(st, n_st, ids, staging, pitch, ppu, w, err_flag, &u)) continue;
    const uint8_t* src = kToStaging ? u.dev : u.stg;
    uint8_t* dst = kToStaging ? u.stg : u.dev;
    if (t.aligned) {  // uniform per CTA
      const int nvec = int(u.nbytes >> 4);
      int4 v[kVecPerThread];
#pragma unroll
      for (int i = 0; i < kVecPerThread; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        if (idx < nvec) v[i] = ld_stream(src + (uint64_t(idx) << 4));
      }
#pragma unroll
      for (int i = 0; i < kVecPerThread; ++i) {
        const int idx = threadIdx.x + i * kThreads;
        if (idx < nvec) st_vec(dst + (uint64_t(idx) << 4), v[i]);
      }
    } else {
      for (uint64_t b = threadIdx.x; b < u.nbytes; b += kThreads) dst[b] = src[b];
    }
  }
}

// The fp8 kernels of the manager-free entry points check the table before
// touching anything: a storage that is not 16-byte aligned sets *err_flag to
// 2 (first CTA) and no CTA moves a byte.
__device__ __forceinline__ bool fp8_table_ok(const ts_block_storage* __restrict__ st, int n_st,
                                             int check, int* err_flag) {
  if (!check) return true;
  const TableScan t = scan_table(st, n_st, 0);
  if (!t.aligned && blockIdx.x == 0 && threadIdx.x == 0 && err_flag != nullptr)
    *reinterpret_cast<volatile int*>(err_flag) = 2;
  return t.aligned;
}

// ---------------------------------------------------------------------------
// fp8 e4m3 fused cast.  One CTA per (block, storage) unit of bf16 values.
// scale = amax / 448 (IEEE round-to-nearest division; 1 when amax == 0),
// q = cvt.rn.satfinite.e4m3(x / scale) with x / scale an IEEE RN division,
// dequant x' = bf16_rn(float(q) * scale).
// ---------------------------------------------------------------------------


template <int T = kThreads>
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read by a previous unit
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = red[0];
#pragma unroll
  for (int i = 1; i < T / 32; ++i) r = fmaxf(r, red[i]);
  return r;
}

__device__ __forceinline__ float bf16_bits_to_float(uint32_t h) {
  return __uint_as_float(h << 16);
}

// Running |x| maximum of 8 bf16 values on packed pairs: clearing the sign
// bits gives |x|, and the bf16x2 maximum ignores NaN like fmaxf.
__device__ __forceinline__ __nv_bfloat162 amax8_pairs(const int4& v, __nv_bfloat162 m) {
  const uint32_t w[4] = {uint32_t(v.x), uint32_t(v.y), uint32_t(v.z), uint32_t(v.w)};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t a = w[j] & 0x7fff7fffu;
    m = __hmax2(m, *reinterpret_cast<const __nv_bfloat162*>(&a));
  }
  return m;
}

__device__ __forceinline__ float pair_max(__nv_bfloat162 m) {
  return fmaxf(__bfloat162float(m.x), __bfloat162float(m.y));
}

__device__ __forceinline__ float amax8(const int4& v, float m) {
  return fmaxf(m, pair_max(amax8_pairs(v, __floats2bfloat162_rn(0.f, 0.f))));
}

// Correctly rounded quotient x / scale.  Markstein's method (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 1990; Muller et al., Handbook of Floating-Point Arithmetic,
// Markstein's theorem): with r = RN(1/scale) and q = RN(x*r) within one ulp of
// x/scale, the FMA residual e = x - q*scale is exact and RN(q + e*r) is the
// correctly rounded quotient.  The residual is a multiple of 2^(exp(x) - 46),
// so it is exactly representable (no underflow) when |x| >= 2^-96; smaller x
// take the IEEE division, as do units whose scale or reciprocal is not a
// normal finite number (use_div, uniform per unit).  The quotient's sign is
// x's (scale > 0), which copysign restores for zero results.
struct Divider {
  float scale, r;
  bool use_div;
  __device__ __forceinline__ explicit Divider(float s) : scale(s) {
    r = __frcp_rn(s);
    use_div = !(s >= 1.17549435e-38f && s <= 3.40282347e38f && r >= 1.17549435e-38f &&
                r <= 3.40282347e38f);
  }
  __device__ __forceinline__ float operator()(float x) const {
    if (use_div || fabsf(x) < 1.2621774e-29f /* 2^-96 */) return __fdiv_rn(x, scale);
    return fast(x);
  }
  // Markstein only.  Exact in the e4m3 result for every x of a unit whose
  // amax >= 2^-64 (and !use_div): x >= 2^-96 is exact as above, and for
  // |x| < 2^-96 both the true quotient and this one are below 2^-23 in
  // magnitude (scale >= 2^-64/448), far under half the smallest e4m3
  // subnormal (2^-10), so both round to zero with x's sign.
  __device__ __forceinline__ float fast(float x) const {
    const float q = __fmul_rn(x, r);
    const float e = __fmaf_rn(-q, scale, x);
    return copysignf(__fmaf_rn(e, r, q), x);  // scale > 0: sign of x (also for zeros)
  }
};

// A unit's amax from which Divider::fast is exact for all of its elements.
constexpr float kFastAmax = 5.42101086e-20f;  // 2^-64

// Packed fp32 pairs (sm_100 .f32x2): each lane of the pair is the IEEE
// round-to-nearest result of the scalar operation.
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Divider::fast on both bf16 of one 32-bit word, as a pair: q = x*r,
// e = fma(q, -scale, x), q' = fma(e, r, q) lane by lane, then the pair's
// e4m3 bytes.  The sign is not restored here (see quant8_fast).
__device__ __forceinline__ uint32_t quant2_fast(uint32_t w, uint64_t r2, uint64_t ns2) {
  const uint64_t x2 = uint64_t(w << 16) | (uint64_t(w & 0xffff0000u) << 32);
  const uint64_t q = mul_f32x2(x2, r2);
  const uint64_t e = fma_f32x2(q, ns2, x2);
  const uint64_t qq = fma_f32x2(e, r2, q);
  const float lo = __uint_as_float(uint32_t(qq)), hi = __uint_as_float(uint32_t(qq >> 32));
  return uint32_t(__nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3));
}

// 8 bf16 -> 8 e4m3 bytes through quant2_fast, for units that allow
// Divider::fast for every element.  For a nonzero x the exact corrected
// quotient q + e*r is nonzero with x's sign (|e*r| < |q| when q != 0, and
// e = x when x*r underflows to zero), and a result that rounds to zero keeps
// that sign; only x = -0 comes out +0 (the sum of opposite zeros).  So x's
// sign bit is OR-ed into each e4m3 byte, a no-op wherever it is already set.
__device__ __forceinline__ uint2 quant8_fast(const int4& v, uint64_t r2, uint64_t ns2) {
  const uint32_t w0 = uint32_t(v.x), w1 = uint32_t(v.y), w2 = uint32_t(v.z), w3 = uint32_t(v.w);
  uint32_t a = quant2_fast(w0, r2, ns2) | (quant2_fast(w1, r2, ns2) << 16);
  uint32_t b = quant2_fast(w2, r2, ns2) | (quant2_fast(w3, r2, ns2) << 16);
  a |= __byte_perm(w0, w1, 0x7531) & 0x80808080u;  // high bytes of the four bf16
  b |= __byte_perm(w2, w3, 0x7531) & 0x80808080u;
  return make_uint2(a, b);
}

// 8 bf16 -> 8 e4m3 bytes (packed in a uint2).  kFast: the unit allows
// Divider::fast for every element.
template <bool kFast>
__device__ __forceinline__ uint2 quant8(const int4& v, const Divider& div) {
  const uint32_t w[4] = {uint32_t(v.x), uint32_t(v.y), uint32_t(v.z), uint32_t(v.w)};
  uint32_t out[2] = {0u, 0u};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float xl = bf16_bits_to_float(w[j] & 0xffffu);
    const float xh = bf16_bits_to_float(w[j] >> 16);
    const float lo = kFast ? div.fast(xl) : div(xl);
    const float hi = kFast ? div.fast(xh) : div(xh);
    const __nv_fp8x2_storage_t p =
        __nv_cvt_float2_to_fp8x2(make_float2(lo, hi), __NV_SATFINITE, __NV_E4M3);
    out[j >> 1] |= uint32_t(p) << (16 * (j & 1));
  }
  return make_uint2(out[0], out[1]);
}

// 8 e4m3 bytes -> 8 bf16 (packed in an int4).
__device__ __forceinline__ int4 dequant8(uint2 q, float scale) {
  const uint32_t in[2] = {q.x, q.y};
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_fp8x2_storage_t p =
        __nv_fp8x2_storage_t((in[j >> 1] >> (16 * (j & 1))) & 0xffffu);
    const __half2_raw h2 = __nv_cvt_fp8x2_to_halfraw2(p, __NV_E4M3);
    // e4m3 -> f16 is exact; f16 -> f32 is exact.
    const float lo = __half2float(__half(__half_raw{h2.x}));
    const float hi = __half2float(__half(__half_raw{h2.y}));
    const __nv_bfloat16 blo = __float2bfloat16_rn(__fmul_rn(lo, scale));
    const __nv_bfloat16 bhi = __float2bfloat16_rn(__fmul_rn(hi, scale));
    w[j] = uint32_t(__bfloat16_as_ushort(blo)) | (uint32_t(__bfloat16_as_ushort(bhi)) << 16);
  }
  return make_int4(int(w[0]), int(w[1]), int(w[2]), int(w[3]));
}

// Units (block k, storage s) in grid-stride order, stepped without a
// division per unit.
struct UnitWalk {
  int64_t k;
  int s;
  int step_k, step_s, n_st;
  __device__ __forceinline__ UnitWalk(int n) : n_st(n) {
    k = int64_t(blockIdx.x / uint32_t(n));
    s = int(blockIdx.x - uint32_t(k) * uint32_t(n));
    step_k = int(gridDim.x / uint32_t(n));
    step_s = int(gridDim.x - uint32_t(step_k) * uint32_t(n));
  }
  __device__ __forceinline__ void next() {
    k += step_k;
    s += step_s;
    if (s >= n_st) {
      s -= n_st;
      ++k;
    }
  }
};

template <typename Ids>
__device__ __forceinline__ bool unit_addr(const ts_block_storage* __restrict__ st,
                                          const Ids& ids, int64_t k, int s, int* err_flag,
                                          int64_t* k_out, uint8_t** dev_out, uint64_t* bb_out) {
  const uint64_t bb = st[s].block_bytes;
  const int64_t id = ids.dev(k);
  const uint64_t dev_off = uint64_t(id) * bb;
  if (id < 0 || dev_off + bb > st[s].dev_bytes) {
    if (err_flag != nullptr && threadIdx.x == 0) *reinterpret_cast<volatile int*>(err_flag) = 1;
    return false;
  }
  *k_out = ids.stage(k);
  *dev_out = reinterpret_cast<uint8_t*>(st[s].dev_ptr) + dev_off;
  *bb_out = bb;
  return true;
}

// V = 16-byte vectors per thread held in registers (V*4 KiB per unit); a
// unit larger than that takes the two-pass path.
// Resident CTAs per SM the fp8 extract is compiled for, by threads per CTA
// and register tile (registers per thread x threads x CTAs <= 64K); its grid
// uses the same.  128 threads with 8 vectors each carry a 16 KiB unit with
// half the per-unit overhead (address walk, reduction, loop) of 256 threads.
constexpr int fp8_extract_ctas_per_sm(int v, int t) {
  return t == 128 ? 8 : (v <= 4 ? 6 : 4);
}

template <typename Ids, int V, int T = kThreads>
__global__ void __launch_bounds__(T, fp8_extract_ctas_per_sm(V, T))
    extract_fp8_kernel(const ts_block_storage* __restrict__ st, int n_st,
                       const __grid_constant__ Ids ids, int64_t n_blocks,
                       uint8_t* staging, uint64_t pitch, uint64_t scale_off,
                       int* err_flag, int check) {
  constexpr int kThreads = T;
  __shared__ float red[T / 32];
  if (!fp8_table_ok(st, n_st, check, err_flag)) return;
  for (UnitWalk u(n_st); u.k < n_blocks; u.next()) {
    const int s = u.s;
    int64_t k;
    uint8_t* dev;
    uint64_t bb;
    if (!unit_addr(st, ids, u.k, s, err_flag, &k, &dev, &bb)) continue;
    uint8_t* stg_blk = staging + uint64_t(k) * pitch;
    uint8_t* q_out = stg_blk + st[s].stage_off;
    const int64_t nvec = int64_t(bb >> 4);  // 8 bf16 per vector
    float m = 0.f;
    if (nvec <= int64_t(kThreads) * V) {
      int4 v[V];
      __nv_bfloat162 mp = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const int64_t idx = threadIdx.x + int64_t(i) * kThreads;
        if (idx < nvec) {
          v[i] = ld_stream(dev + (idx << 4));
          mp = amax8_pairs(v[i], mp);
        }
      }
      m = pair_max(mp);
      const float amax = block_max<T>(m, red);
      const float scale = amax == 0.f ? 1.f : __fdiv_rn(amax, 448.f);
      const Divider div(scale);
      if (!div.use_div && amax >= kFastAmax) {  // uniform per unit
        const uint32_t rb = __float_as_uint(div.r), nsb = __float_as_uint(-scale);
        const uint64_t r2 = uint64_t(rb) | (uint64_t(rb) << 32);
        const uint64_t ns2 = uint64_t(nsb) | (uint64_t(nsb) << 32);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int64_t idx = threadIdx.x + int64_t(i) * kThreads;
          if (idx < nvec) *reinterpret_cast<uint2*>(q_out + (idx << 3)) = quant8_fast(v[i], r2, ns2);
        }
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const int64_t idx = threadIdx.x + int64_t(i) * kThreads;
          if (idx < nvec) *reinterpret_cast<uint2*>(q_out + (idx << 3)) = quant8<false>(v[i], div);
        }
      }
      if (threadIdx.x == 0) *reinterpret_cast<float*>(stg_blk + scale_off + 4u * s) = scale;
    } else {
      // Large blocks: pass 1 reduces, pass 2 re-reads (L2-resident) and casts.
      for (int64_t idx = threadIdx.x; idx < nvec; idx += kThreads)
        m = amax8(ld_stream(dev + (idx << 4)), m);
      const float amax = block_max<T>(m, red);
      const float scale = amax == 0.f ? 1.f : __fdiv_rn(amax, 448.f);
      const Divider div(scale);
      for (int64_t idx = threadIdx.x; idx < nvec; idx += kThreads)
        *reinterpret_cast<uint2*>(q_out + (idx << 3)) =
            quant8<false>(*reinterpret_cast<const int4*>(dev + (idx << 4)), div);
      if (threadIdx.x == 0) *reinterpret_cast<float*>(stg_blk + scale_off + 4u * s) = scale;
    }
  }
}

// VPT fp8 vectors (8 bytes each) per thread, T threads per CTA.  16 KiB
// units run on 128 threads x 8 vectors: 64 bytes of loads in flight per
// thread and 16 CTAs per SM.
template <typename Ids, int VPT = kVecPerThread, int T = kThreads>
__global__ void __launch_bounds__(T, T == 128 ? 16 : 8)
    insert_fp8_kernel(const ts_block_storage* __restrict__ st, int n_st,
                      const __grid_constant__ Ids ids, int64_t n_blocks,
                      const uint8_t* staging, uint64_t pitch, uint64_t scale_off,
                      int* err_flag, int check) {
  constexpr int kThreads = T, kVecPerThread = VPT;
  if (!fp8_table_ok(st, n_st, check, err_flag)) return;
  for (UnitWalk u(n_st); u.k < n_blocks; u.next()) {
    const int s = u.s;
    int64_t k;
    uint8_t* dev;
    uint64_t bb;
    if (!unit_addr(st, ids, u.k, s, err_flag, &k, &dev, &bb)) continue;
    const uint8_t* stg_blk = staging + uint64_t(k) * pitch;
    const uint8_t* q_in = stg_blk + st[s].stage_off;
    const float scale = *reinterpret_cast<const float*>(stg_blk + scale_off + 4u * s);
    const int64_t nvec = int64_t(bb >> 4);
    for (int64_t base = 0; base < nvec; base += int64_t(kThreads) * kVecPerThread) {
      uint2 q[kVecPerThread];
#pragma unroll
      for (int i = 0; i < kVecPerThread; ++i) {
        const int64_t idx = base + threadIdx.x + int64_t(i) * kThreads;
        if (idx < nvec) q[i] = *reinterpret_cast<const uint2*>(q_in + (idx << 3));
      }
#pragma unroll
      for (int i = 0; i < kVecPerThread; ++i) {
        const int64_t idx = base + threadIdx.x + int64_t(i) * kThreads;
        if (idx < nvec) st_vec(dev + (idx << 4), dequant8(q[i], scale));
      }
    }
  }
}

bool aligned16(uint64_t v) { return (v & 15u) == 0; }

// max_ctas > 0 caps the persistent grid; max_ctas < 0 asks for one CTA per
// item (CTAs retire as their piece lands instead of grid-striding).
int launch_grid(int device, int64_t items, int max_ctas = 0) {
  int64_t cap = int64_t(sm_count(device)) * kCtasPerSm;
  if (max_ctas > 0 && max_ctas < cap) cap = max_ctas;
  if (max_ctas < 0) cap = INT32_MAX;
  return int(items < cap ? items : cap);
}

// Manager chunks: storage table inspected on the host when the manager was
// created (vec_ok, max_block_bytes).  bulk: the bulk-copy kernel (one CTA per
// SM), for 16-byte aligned tables whose both sides are device memory.
template <bool kToStaging, typename Ids>
int block_copy(int device, const ts_block_storage* d_st, int n_st,
               const Ids& d_ids, int64_t n_blocks, uint8_t* staging,
               uint64_t pitch, int* err_flag, void* stream, bool vec_ok,
               uint64_t max_block_bytes, int max_ctas = 0, int variant = kCopyVec) {
  if (n_blocks == 0 || n_st == 0) return TS_OK;
  const uint32_t ppu = uint32_t((max_block_bytes + kPieceBytes - 1) / kPieceBytes);
  if (ppu == 0) return TS_OK;
  const int64_t items = n_blocks * int64_t(n_st) * ppu;
  DeviceGuard g(device);
  const int grid = launch_grid(device, items, max_ctas);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (variant == kCopyBulk && vec_ok) {
    // opt in to 192 KiB of dynamic shared memory (per device: set each launch)
    TS_CUDA_RET(cudaFuncSetAttribute(block_copy_bulk_kernel<kToStaging, Ids>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     int(kBulkSmem)),
                "bulk copy shared memory attribute");
    const int64_t ctas = (items + kBulkWarps - 1) / kBulkWarps;
    int bgrid = sm_count(device);
    if (max_ctas > 0 && max_ctas < bgrid) bgrid = max_ctas;
    if (ctas < bgrid) bgrid = int(ctas);
    block_copy_bulk_kernel<kToStaging, Ids><<<bgrid, kBulkWarps * 32, kBulkSmem, s>>>(
        d_st, n_st, d_ids, n_blocks, staging, pitch, ppu, err_flag);
  } else if (variant == kCopyWide && vec_ok) {
    block_copy_wide_kernel<kToStaging, Ids><<<grid, kThreads, 0, s>>>(
        d_st, n_st, d_ids, n_blocks, staging, pitch, ppu, err_flag);
  } else if (vec_ok) {
    block_copy_vec_kernel<kToStaging, Ids><<<grid, kThreads, 0, s>>>(
        d_st, n_st, d_ids, n_blocks, staging, pitch, ppu, err_flag);
  } else {
    block_copy_byte_kernel<kToStaging, Ids><<<grid, kThreads, 0, s>>>(
        d_st, n_st, d_ids, n_blocks, staging, pitch, ppu, err_flag);
  }
  TS_CUDA_RET(cudaGetLastError(), "block copy launch");
  return TS_OK;
}

// Device-table entry points: the kernel scans the table itself.  The grid
// is a full wave, or 8 CTAs per (block, storage) unit when that is fewer.
template <bool kToStaging>
int block_copy_scan(int device, const ts_block_storage* d_st, int n_st, const int64_t* d_ids,
                    int64_t n_blocks, uint8_t* staging, uint64_t pitch, int* err_flag,
                    cudaStream_t s) {
  DeviceGuard g(device);
  const int grid = launch_grid(device, n_blocks * int64_t(n_st) * 8);
  block_copy_scan_kernel<kToStaging><<<grid, kThreads, 0, s>>>(d_st, n_st, d_ids, n_blocks,
                                                               staging, pitch, err_flag);
  TS_CUDA_RET(cudaGetLastError(), "block copy launch");
  return TS_OK;
}

// fp8 launchers.  max_bb picks the kernel shape only (units <= 16 KiB run on
// 128-thread CTAs); every shape handles every unit size.  check = 1 makes
// the kernel validate the table's alignment first (device-table entry
// points; the manager validated its table when it was created).
template <typename Ids>
int launch_extract_fp8(int device, const ts_block_storage* d_st, int n_st,
                       const Ids& ids, int64_t n_blocks, void* staging,
                       uint64_t pitch, uint64_t scale_off, int* err_flag,
                       cudaStream_t s, uint64_t max_bb, int max_ctas, int check) {
  if (n_blocks == 0 || n_st == 0) return TS_OK;
  DeviceGuard g(device);
  uint8_t* stg = static_cast<uint8_t*>(staging);
  // register tile sized to the largest unit (16-byte vectors per thread)
  const uint64_t vecs = (max_bb / 16 + kThreads - 1) / kThreads;
  const bool narrow = vecs <= 4;  // units <= 16 KiB: 128 threads x 8 vectors
  int64_t cap = int64_t(sm_count(device)) *
                (narrow ? fp8_extract_ctas_per_sm(8, 128) : fp8_extract_ctas_per_sm(8, kThreads));
  if (max_ctas > 0 && max_ctas < cap) cap = max_ctas;
  const int64_t units = n_blocks * int64_t(n_st);
  const int grid = int(units < cap ? units : cap);
  if (narrow)
    extract_fp8_kernel<Ids, 8, 128><<<grid, 128, 0, s>>>(d_st, n_st, ids, n_blocks, stg, pitch,
                                                         scale_off, err_flag, check);
  else
    extract_fp8_kernel<Ids, 8><<<grid, kThreads, 0, s>>>(d_st, n_st, ids, n_blocks, stg, pitch,
                                                         scale_off, err_flag, check);
  TS_CUDA_RET(cudaGetLastError(), "extract_fp8 launch");
  return TS_OK;
}

template <typename Ids>
int launch_insert_fp8(int device, const ts_block_storage* d_st, int n_st,
                      const Ids& ids, int64_t n_blocks, const void* staging,
                      uint64_t pitch, uint64_t scale_off, int* err_flag,
                      cudaStream_t s, uint64_t max_bb, int max_ctas, int check) {
  if (n_blocks == 0 || n_st == 0) return TS_OK;
  DeviceGuard g(device);
  const uint8_t* stg = static_cast<const uint8_t*>(staging);
  const int64_t units = n_blocks * int64_t(n_st);
  if (max_bb <= 16 * 1024) {
    int64_t cap = int64_t(sm_count(device)) * 16;
    if (max_ctas > 0 && max_ctas < cap) cap = max_ctas;
    const int grid = int(units < cap ? units : cap);
    insert_fp8_kernel<Ids, 8, 128><<<grid, 128, 0, s>>>(d_st, n_st, ids, n_blocks, stg, pitch,
                                                         scale_off, err_flag, check);
  } else {
    const int grid = launch_grid(device, units, max_ctas);
    insert_fp8_kernel<Ids><<<grid, kThreads, 0, s>>>(d_st, n_st, ids, n_blocks, stg, pitch,
                                                     scale_off, err_flag, check);
  }
  TS_CUDA_RET(cudaGetLastError(), "insert_fp8 launch");
  return TS_OK;
}

// Block bytes of an fp8 table's storages, estimated from its staging pitch
// (sum of 16-byte-rounded halves plus the scale words): exact for equal
// storages, and used only to pick a kernel shape.
uint64_t fp8_block_bytes_hint(int n_st, uint64_t pitch, uint64_t scale_off) {
  const uint64_t payload = scale_off < pitch ? scale_off : pitch;
  return n_st > 0 ? 2 * (payload / uint64_t(n_st)) : 0;
}

}  // namespace

// Entry points for the manager (ids by value, at most kMaxParamIds blocks).
int mgr_extract(int device, const ts_block_storage* d_st, int n_st,
                const ParamIds& ids, int64_t n_blocks, void* staging,
                uint64_t pitch, int* err_flag, cudaStream_t s, bool vec_ok,
                uint64_t max_bb, bool fp8, uint64_t scale_off, int max_ctas, int variant) {
  if (fp8)
    return launch_extract_fp8(device, d_st, n_st, ids, n_blocks, staging, pitch,
                              scale_off, err_flag, s, max_bb, max_ctas, 0);
  return block_copy<true>(device, d_st, n_st, ids, n_blocks, static_cast<uint8_t*>(staging),
                          pitch, err_flag, s, vec_ok, max_bb, max_ctas, variant);
}

int mgr_insert(int device, const ts_block_storage* d_st, int n_st,
               const ParamIds& ids, int64_t n_blocks, const void* staging,
               uint64_t pitch, int* err_flag, cudaStream_t s, bool vec_ok,
               uint64_t max_bb, bool fp8, uint64_t scale_off, int max_ctas, int variant) {
  if (fp8)
    return launch_insert_fp8(device, d_st, n_st, ids, n_blocks, staging, pitch,
                             scale_off, err_flag, s, max_bb, max_ctas, 0);
  return block_copy<false>(device, d_st, n_st, ids, n_blocks,
                           static_cast<uint8_t*>(const_cast<void*>(staging)), pitch, err_flag,
                           s, vec_ok, max_bb, max_ctas, variant);
}

}  // namespace tsb

using tsb::set_error;

namespace {
int check_args(int64_t n_blocks, int n_storages, const void* d_storages, const void* d_ids,
               const void* d_staging) {
  if (n_blocks < 0) return set_error(TS_INVALID_ARGUMENT, "n_blocks must be >= 0");
  if (n_storages < 0) return set_error(TS_INVALID_ARGUMENT, "n_storages must be >= 0");
  if (n_blocks > 0 && n_storages > 0 && (!d_storages || !d_ids || !d_staging))
    return set_error(TS_INVALID_ARGUMENT, "null pointer argument");
  return TS_OK;
}

int check_fp8_args(uint64_t pitch, uint64_t scale_off, const void* staging) {
  // The fp8 kernels move 16 B of bf16 / 8 B of fp8 per vector.
  if (!tsb::aligned16(pitch) || !tsb::aligned16(reinterpret_cast<uint64_t>(staging)) ||
      (scale_off & 3u) != 0)
    return set_error(TS_INVALID_ARGUMENT,
                     "fp8 path needs 16-byte aligned storages, block sizes, "
                     "stage offsets and pitch, and a 4-byte aligned scale offset");
  return TS_OK;
}
}  // namespace

extern "C" int ts_kv_extract(int device, const ts_block_storage* d_storages,
                             int n_storages, const int64_t* d_ids,
                             int64_t n_blocks, void* d_staging,
                             uint64_t stage_pitch, int* err_flag, void* stream) {
  tsb::clear_error();
  int rc = check_args(n_blocks, n_storages, d_storages, d_ids, d_staging);
  if (rc != TS_OK || n_blocks == 0 || n_storages == 0) return rc;
  return tsb::block_copy_scan<true>(device, d_storages, n_storages, d_ids, n_blocks,
                                    static_cast<uint8_t*>(d_staging), stage_pitch, err_flag,
                                    reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ts_kv_insert(int device, const ts_block_storage* d_storages,
                            int n_storages, const int64_t* d_ids,
                            int64_t n_blocks, const void* d_staging,
                            uint64_t stage_pitch, int* err_flag, void* stream) {
  tsb::clear_error();
  int rc = check_args(n_blocks, n_storages, d_storages, d_ids, d_staging);
  if (rc != TS_OK || n_blocks == 0 || n_storages == 0) return rc;
  return tsb::block_copy_scan<false>(device, d_storages, n_storages, d_ids, n_blocks,
                                     static_cast<uint8_t*>(const_cast<void*>(d_staging)),
                                     stage_pitch, err_flag,
                                     reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ts_kv_extract_fp8(int device, const ts_block_storage* d_storages,
                                 int n_storages, const int64_t* d_ids,
                                 int64_t n_blocks, void* d_staging,
                                 uint64_t stage_pitch, uint64_t scale_off,
                                 int* err_flag, void* stream) {
  tsb::clear_error();
  int rc = check_args(n_blocks, n_storages, d_storages, d_ids, d_staging);
  if (rc != TS_OK || n_blocks == 0 || n_storages == 0) return rc;
  rc = check_fp8_args(stage_pitch, scale_off, d_staging);
  if (rc != TS_OK) return rc;
  return tsb::launch_extract_fp8(device, d_storages, n_storages, tsb::DevIds{d_ids}, n_blocks,
                                 d_staging, stage_pitch, scale_off, err_flag,
                                 reinterpret_cast<cudaStream_t>(stream),
                                 tsb::fp8_block_bytes_hint(n_storages, stage_pitch, scale_off),
                                 0, 1);
}

extern "C" int ts_kv_insert_fp8(int device, const ts_block_storage* d_storages,
                                int n_storages, const int64_t* d_ids,
                                int64_t n_blocks, const void* d_staging,
                                uint64_t stage_pitch, uint64_t scale_off,
                                int* err_flag, void* stream) {
  tsb::clear_error();
  int rc = check_args(n_blocks, n_storages, d_storages, d_ids, d_staging);
  if (rc != TS_OK || n_blocks == 0 || n_storages == 0) return rc;
  rc = check_fp8_args(stage_pitch, scale_off, d_staging);
  if (rc != TS_OK) return rc;
  return tsb::launch_insert_fp8(device, d_storages, n_storages, tsb::DevIds{d_ids}, n_blocks,
                                d_staging, stage_pitch, scale_off, err_flag,
                                reinterpret_cast<cudaStream_t>(stream),
                                tsb::fp8_block_bytes_hint(n_storages, stage_pitch, scale_off),
                                0, 1);
}

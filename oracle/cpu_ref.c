/*
 * cpu_ref.c -- C restatement of the reference's host copy loops.
 * TEST / BASELINE INFRASTRUCTURE ONLY: loaded by tests/ and by bench.py's
 * cpu_baseline leg and `--impl reference` arm; never by the product.
 *
 * On the reference's own fake device (the XLA CPU PJRT client used by its
 * tests) device buffers are host memory and CopyRawDeviceToHost /
 * CopyRawHostToDevice are memcpys, so the reference's offload / reload of a
 * block list is:
 *
 *   for each (layer, shard) storage s:                 DispatchD2hWork
 *     for each coalesced run (src, dst, n):            kv_cache_manager_base.cc:2036-2124
 *       memcpy(host_s + dst*bb_s, dev_s + src*bb_s, n*bb_s)
 *
 * and the mirror image for H2D (kv_cache_manager_base.cc:1945-2033).  The
 * reference issues the runs of one NUMA group from one dispatch task
 * (kv_cache_manager_base.cc:652-790); here the storages are split over
 * `threads` POSIX threads so the baseline uses every host core it is given.
 *
 * The reshard executor (weight_synchronizer_base.cc:606-667 expansion, each
 * copy landing at dst_offset of the receiver's buffer) is restated in
 * oref_reshard_f32_bf16 with the fp32 -> bf16 round-to-nearest-even cast of
 * the B200 path; oref_extract_fp8 (C2: gather + per-unit absmax scale +
 * e4m3 cast) and oref_relayout (C3: the hand-off permute) are the host-core
 * baselines of the other configurations.
 */
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  uint8_t* const* dst;   /* per storage */
  const uint8_t* const* src;
  const uint64_t* bb;    /* per storage block bytes */
  const int64_t* src_ids;
  const int64_t* dst_ids;
  const int64_t* n;
  int64_t runs;
  int s_begin, s_end;
} copy_job;

static void* copy_worker(void* arg) {
  const copy_job* j = (const copy_job*)arg;
  for (int s = j->s_begin; s < j->s_end; ++s) {
    const uint64_t bb = j->bb[s];
    for (int64_t r = 0; r < j->runs; ++r) {
      memcpy(j->dst[s] + (uint64_t)j->dst_ids[r] * bb,
             j->src[s] + (uint64_t)j->src_ids[r] * bb, (uint64_t)j->n[r] * bb);
    }
  }
  return NULL;
}

/* Copies runs (src_ids[r], dst_ids[r], n[r]) in block units of every storage
 * from src[s] to dst[s]; D2H passes (host, dev), H2D passes (dev, host). */
int oref_copy_runs(uint8_t* const* dst, const uint8_t* const* src, const uint64_t* bb,
                   int n_storages, const int64_t* src_ids, const int64_t* dst_ids,
                   const int64_t* n, int64_t runs, int threads) {
  if (threads < 1) threads = 1;
  if (threads > n_storages) threads = n_storages;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  copy_job jobs[256];
  for (int t = 0; t < threads; ++t) {
    jobs[t] = (copy_job){dst, src, bb, src_ids, dst_ids, n, runs,
                         (int)((int64_t)n_storages * t / threads),
                         (int)((int64_t)n_storages * (t + 1) / threads)};
  }
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, copy_worker, &jobs[t]);
  copy_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
  return 0;
}

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x007fffffu)) /* NaN */
    return (uint16_t)(((b >> 16) & 0x8000u) | 0x7fc0u);
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

typedef struct {
  const float* src;
  uint16_t* dst;
  const int64_t* chunks; /* n x 6: src_off dst_off size src_stride dst_stride count (elements) */
  int64_t n_chunks;
  int t, threads;
} reshard_job;

static void* reshard_worker(void* arg) {
  const reshard_job* j = (const reshard_job*)arg;
  for (int64_t c = 0; c < j->n_chunks; ++c) {
    const int64_t* k = j->chunks + 6 * c;
    const int64_t count = k[5] > 0 ? k[5] : 1;
    for (int64_t r = j->t; r < count; r += j->threads) {
      const float* s = j->src + k[0] + r * k[3];
      uint16_t* d = j->dst + k[1] + r * k[4];
      for (int64_t e = 0; e < k[2]; ++e) d[e] = f32_to_bf16_rne(s[e]);
    }
  }
  return NULL;
}

/* Executes element-unit strided chunks fp32 -> bf16 with `threads` threads. */
int oref_reshard_f32_bf16(const float* src, uint16_t* dst, const int64_t* chunks,
                          int64_t n_chunks, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  reshard_job jobs[256];
  for (int t = 0; t < threads; ++t) jobs[t] = (reshard_job){src, dst, chunks, n_chunks, t, threads};
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, reshard_worker, &jobs[t]);
  reshard_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
  return 0;
}

/* ------------------------------------------------------------------------
 * C2 baseline: gather + per-(block, storage) absmax scale + e4m3 cast
 * (the fused fp8 offload of the B200 path, restated for the host cores).
 * scale = RN(amax / 448) (1 if amax == 0); q = e4m3_rn_satfinite(RN(x / scale)).
 * ------------------------------------------------------------------------ */

/* float -> e4m3 (1 sign, 4 exponent bits with bias 7, 3 mantissa bits; max
 * finite 448, no infinities), round to nearest even, saturating to +-448.
 * Written from the format definition. */
static inline uint8_t f32_to_e4m3_satfinite(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  const uint8_t sign = (uint8_t)((b >> 24) & 0x80u);
  const uint32_t a = b & 0x7fffffffu;
  if (a > 0x7f800000u) return sign | 0x7fu;   /* NaN */
  if (a >= 0x43e00000u) return sign | 0x7eu;  /* |x| >= 448: saturate */
  const int e = (int)(a >> 23) - 127;
  if (e >= -6) {                              /* e4m3 normal range */
    uint32_t keep = (a & 0x7fffffu) >> 20, rest = a & 0xfffffu;
    if (rest > 0x80000u || (rest == 0x80000u && (keep & 1u))) ++keep;
    uint32_t ee = (uint32_t)(e + 7);
    if (keep == 8u) {
      keep = 0u;
      ++ee;
    }
    return sign | (uint8_t)(ee << 3) | (uint8_t)keep;
  }
  /* subnormal: multiples of 2^-9; |x| * 512 is exact, then ties-to-even */
  float q;
  memcpy(&q, &a, 4);
  q *= 512.0f;
  uint32_t m = (uint32_t)q;
  const float frac = q - (float)m;
  if (frac > 0.5f || (frac == 0.5f && (m & 1u))) ++m;
  return m >= 8u ? (uint8_t)(sign | 0x08u) : (uint8_t)(sign | m);
}

uint8_t oref_e4m3(float f) { return f32_to_e4m3_satfinite(f); }

typedef struct {
  const uint16_t* const* st;  /* per storage: bf16 blocks */
  const uint64_t* elems;      /* per storage: bf16 values per block */
  const uint64_t* stage_off;  /* per storage: byte offset inside a staging block */
  const int64_t* ids;
  int64_t n_blocks;
  int n_st;
  uint8_t* staging;
  uint64_t pitch, scale_off;
  int t, threads;
} fp8_job;

static void* fp8_worker(void* arg) {
  const fp8_job* j = (const fp8_job*)arg;
  const int64_t units = j->n_blocks * j->n_st;
  for (int64_t u = j->t; u < units; u += j->threads) {
    const int64_t k = u / j->n_st;
    const int s = (int)(u % j->n_st);
    const uint64_t n = j->elems[s];
    const uint16_t* x = j->st[s] + (uint64_t)j->ids[k] * n;
    float amax = 0.f;
    for (uint64_t i = 0; i < n; ++i) {
      const uint32_t bits = (uint32_t)(x[i] & 0x7fffu) << 16;
      float v;
      memcpy(&v, &bits, 4);
      if (v > amax) amax = v;
    }
    const float scale = amax == 0.f ? 1.f : amax / 448.0f;
    uint8_t* blk = j->staging + (uint64_t)k * j->pitch;
    uint8_t* q = blk + j->stage_off[s];
    for (uint64_t i = 0; i < n; ++i) {
      const uint32_t bits = (uint32_t)x[i] << 16;
      float v;
      memcpy(&v, &bits, 4);
      q[i] = f32_to_e4m3_satfinite(v / scale);
    }
    memcpy(blk + j->scale_off + 4u * (uint64_t)s, &scale, 4);
  }
  return NULL;
}

int oref_extract_fp8(const uint16_t* const* storages, const uint64_t* elems,
                     const uint64_t* stage_off, int n_st, const int64_t* ids, int64_t n_blocks,
                     uint8_t* staging, uint64_t pitch, uint64_t scale_off, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  fp8_job jobs[256];
  for (int t = 0; t < threads; ++t)
    jobs[t] = (fp8_job){storages, elems, stage_off, ids, n_blocks, n_st, staging, pitch,
                        scale_off, t, threads};
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, fp8_worker, &jobs[t]);
  fp8_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
  return 0;
}

/* ------------------------------------------------------------------------
 * C3 baseline: the hand-off permute, head vector by head vector, from
 * head-major source pages of st_tok tokens to token-major destination pages
 * of dt_tok tokens (per storage, per sequence, per token, per head).
 * ------------------------------------------------------------------------ */

typedef struct {
  const uint8_t* const* src;
  uint8_t* const* dst;
  int n_st, heads;
  uint64_t hb;
  int64_t st_tok, dt_tok, tokens, n_seqs, sbps, dbps;
  const int32_t* stab;
  const int32_t* dtab;
  int t, threads;
} relayout_job;

static void* relayout_worker(void* arg) {
  const relayout_job* j = (const relayout_job*)arg;
  const uint64_t sbb = (uint64_t)j->st_tok * j->heads * j->hb;
  const uint64_t dbb = (uint64_t)j->dt_tok * j->heads * j->hb;
  for (int s = j->t; s < j->n_st; s += j->threads)
    for (int64_t q = 0; q < j->n_seqs; ++q)
      for (int64_t tk = 0; tk < j->tokens; ++tk) {
        const uint8_t* sp = j->src[s] + (uint64_t)j->stab[q * j->sbps + tk / j->st_tok] * sbb;
        uint8_t* dp = j->dst[s] + (uint64_t)j->dtab[q * j->dbps + tk / j->dt_tok] * dbb;
        for (int h = 0; h < j->heads; ++h)
          memcpy(dp + ((uint64_t)(tk % j->dt_tok) * j->heads + h) * j->hb,
                 sp + ((uint64_t)h * j->st_tok + (uint64_t)(tk % j->st_tok)) * j->hb, j->hb);
      }
  return NULL;
}

int oref_relayout(const uint8_t* const* src, uint8_t* const* dst, int n_st, int heads,
                  uint64_t head_bytes, int64_t st_tok, int64_t dt_tok, const int32_t* stab,
                  const int32_t* dtab, int64_t n_seqs, int64_t tokens, int threads) {
  if (threads < 1) threads = 1;
  if (threads > n_st) threads = n_st;
  if (threads > 256) threads = 256;
  pthread_t tid[256];
  relayout_job jobs[256];
  for (int t = 0; t < threads; ++t)
    jobs[t] = (relayout_job){src, dst, n_st, heads, head_bytes, st_tok, dt_tok, tokens, n_seqs,
                             tokens / st_tok, tokens / dt_tok, stab, dtab, t, threads};
  for (int t = 1; t < threads; ++t) pthread_create(&tid[t], NULL, relayout_worker, &jobs[t]);
  relayout_worker(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(tid[t], NULL);
  return 0;
}

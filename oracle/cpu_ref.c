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
 * the B200 path.
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

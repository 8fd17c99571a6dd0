/*
 * tpusync_b200.h -- C ABI of the B200-native tpu_sync data-movement hot path.
 *
 * Every entry point is `extern "C"`, takes plain pointers and sizes, never
 * throws and returns a status code (ts_status).  The last error message of
 * the calling thread is available through ts_last_error().
 *
 * Units follow the reference: block offsets are "major-dim" units (one block of
 * one (layer, shard) storage = its dim-0 slice), byte offsets are bytes.
 *
 * Device pointers are CUDA device addresses of the device given in the call;
 * `stream` arguments are cudaStream_t handles (NULL = legacy default stream).
 */
#ifndef TPUSYNC_B200_H_
#define TPUSYNC_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TS_API __attribute__((visibility("default")))
#else
#define TS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: the absl::StatusCode values the reference returns
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:72-102, :2005-2012, :2096-2103). */
typedef enum ts_status {
  TS_OK = 0,
  TS_CANCELLED = 1,
  TS_UNKNOWN = 2,
  TS_INVALID_ARGUMENT = 3,
  TS_DEADLINE_EXCEEDED = 4,
  TS_NOT_FOUND = 5,
  TS_ALREADY_EXISTS = 6,
  TS_RESOURCE_EXHAUSTED = 8,
  TS_FAILED_PRECONDITION = 9,
  TS_OUT_OF_RANGE = 11,
  TS_UNIMPLEMENTED = 12,
  TS_INTERNAL = 13,
  TS_UNAVAILABLE = 14,
  /* not an error: returned by ts_event_query while the work is in flight */
  TS_PENDING = 100
} ts_status;

/* Thread-local message of the last failed call on this thread ("" if none). */
TS_API const char* ts_last_error(void);

/* Library version string. */
TS_API const char* ts_version(void);

/* ------------------------------------------------------------------------ */
/* Pure host logic (no CUDA calls; usable on a machine without a GPU).       */
/* ------------------------------------------------------------------------ */

/* Replaces ValidateOffsetsAndSizes (tpu_sync/kv_cache/kv_cache_manager_base.cc:72-102).
 * n_dst / n_sizes may be 0 (= "not given", as in the reference). */
TS_API int ts_validate_copy_spec(const int64_t* src, int64_t n_src, const int64_t* dst,
                          int64_t n_dst, const int64_t* sizes, int64_t n_sizes);

/* Replaces CoalesceMajorDimCopies (tpu_sync/kv_cache/kv_cache_manager_base.cc:121-141):
 * merges copy i into the previous run when both its src and dst continue it.
 * Outputs must hold n entries; *n_out receives the run count. */
TS_API int ts_coalesce_runs(const int64_t* src, const int64_t* dst, const int64_t* sizes,
                     int64_t n, int64_t* out_src, int64_t* out_dst,
                     int64_t* out_sizes, int64_t* n_out);

/* Pool layouts: byte-level descriptions of block pools inside a storage.
 * Replace RegionSpec / PoolSpec (tpu_sync/kv_cache/pool_layout.h:34-74); the
 * same fields and meaning (tag / dtype_tag are opaque strings). */
typedef struct ts_region_spec {
  const char* name;
  int64_t offset_bytes;      /* first unit's offset inside a block */
  int64_t stride_bytes;      /* distance between units */
  int64_t unit_bytes;
  int64_t num_units;
  int64_t units_per_stride;  /* units packed back to back at each stride */
} ts_region_spec;

typedef struct ts_pool_spec {
  const char* tag;
  int64_t storage_index;       /* which storage (layer) of the manager */
  int64_t base_offset_bytes;
  int64_t block_stride_bytes;
  int64_t num_blocks;
  const ts_region_spec* regions;
  int64_t num_regions;
  const char* dtype_tag;
} ts_pool_spec;

typedef struct ts_pool_extent {   /* PoolBlockCopyExtent (pool_layout.h:84-87) */
  int64_t offset_bytes;
  int64_t size_bytes;
} ts_pool_extent;

typedef struct ts_live_segment {  /* PoolLiveSegment (pool_layout.h:99-110) */
  int64_t logical_offset;
  int64_t physical_offset;
  int64_t size;
} ts_live_segment;

typedef struct ts_live_copy_chunk {  /* LiveCopyChunk (pool_layout.h:127-137) */
  int64_t src_physical;
  int64_t dst_physical;
  int64_t size;
} ts_live_copy_chunk;

/* RegionSpec::Validate / PoolSpec::Validate
 * (tpu_sync/kv_cache/pool_layout.cc:120-185, :187-229); storage_bytes < 0
 * checks internal consistency only.  Same codes and messages. */
TS_API int ts_region_validate(const ts_region_spec* region, int64_t slot_bytes);
TS_API int ts_pool_validate(const ts_pool_spec* pool, int64_t storage_bytes);
/* PoolSpec::storage_extent_end_bytes (pool_layout.cc:231-254), the largest
 * region extent end in one block and live_bytes_per_block
 * (tpu_sync/api/torch/pool_layout.py:129-156); INT64_MAX on overflow. */
TS_API int ts_pool_geometry(const ts_pool_spec* pool, int64_t* storage_extent_end,
                            int64_t* block_live_end, int64_t* live_bytes_per_block);
/* RegionsCoverRange (pool_layout.cc:256-272). */
TS_API int ts_regions_cover_range(const ts_region_spec* regions, int64_t n, uint64_t start,
                                  uint64_t end, int* covered);

/* Output arrays below follow one protocol: *n_out receives the number of
 * results; when it exceeds `cap` nothing is written and the call returns
 * TS_RESOURCE_EXHAUSTED (call again with cap >= *n_out). */

/* ComputePoolBlockCopyExtents (pool_layout.cc:274-374): declared-live byte
 * extents of the given blocks, sorted and merged where they touch. */
TS_API int ts_pool_copy_extents(const ts_pool_spec* pool, const int64_t* block_ids,
                                int64_t n_ids, ts_pool_extent* out, int64_t cap,
                                int64_t* n_out);
/* ExpandPoolLiveSegments (pool_layout.cc:376-472). */
TS_API int ts_pool_live_segments(const ts_pool_spec* pool, ts_live_segment* out, int64_t cap,
                                 int64_t* n_out);
/* PhysicalLiveRangeToLogical (pool_layout.cc:474-493). */
TS_API int ts_pool_physical_to_logical(const ts_live_segment* segments, int64_t n,
                                       int64_t physical_offset, int64_t size,
                                       int64_t* logical_start, int64_t* logical_end);
/* TranslateLiveCopy (pool_layout.cc:554-602). */
TS_API int ts_pool_translate_live_copy(const ts_live_segment* src, int64_t n_src,
                                       const ts_live_segment* dst, int64_t n_dst,
                                       int64_t src_offset, int64_t dst_offset, int64_t size,
                                       ts_live_copy_chunk* out, int64_t cap, int64_t* n_out);

/* Pool reshard planning (prefill -> decode KV hand-off).  Replaces the data
 * part of BuildPoolReshardPlan
 * (tpu_sync/kv_cache/reshard/pool_reshard_planner.cc:132-859) with the span
 * declarations of tpu_sync/kv_cache/reshard/declaration_types.h:17-58. */
typedef struct ts_byte_span {        /* PoolByteSpan */
  int64_t src_block_ordinal;         /* index into the declaration's block_ids */
  int64_t src_offset_bytes;          /* compact-live offset in the source block */
  int64_t dst_block_index;           /* index into the tag's destination block list */
  int64_t dst_offset_bytes;          /* compact-live offset (v1: request-global) */
  int64_t size_bytes;
  int64_t src_stride_bytes;
  int64_t dst_stride_bytes;
  int32_t count;                     /* repeats at the strides */
  int32_t pad_;
} ts_byte_span;

typedef struct ts_span_decl {        /* PoolSpanRegistration of one source unit */
  int64_t src_unit;                  /* index of the declaring source unit */
  const char* tag;
  const int64_t* block_ids;
  int64_t n_block_ids;
  const ts_byte_span* spans;
  int64_t n_spans;
  int64_t declared_bytes;
  int32_t dst_space_version;         /* 0: page-indexed, 1: request-global */
  int32_t pad_;
} ts_span_decl;

typedef struct ts_pool_reshard_request {  /* PlanRequest (data-plane fields) */
  int64_t n_src_units;
  const ts_pool_spec* const* src_pools;   /* per unit: its pool manifest */
  const int64_t* n_src_pools;             /* per unit */
  const ts_pool_spec* dst_pools;          /* the destination unit's manifest */
  int64_t n_dst_pools;
  const int32_t* transfer_ranks;          /* per unit (NULL: unit index) */
  const int32_t* transfer_parallelism;    /* per unit (NULL: the number of units) */
  int32_t parallelism;                    /* 0: the units' admitted value */
  int32_t pad_;
  const char* const* tags;                /* transfer_pool_tags */
  int64_t n_tags;
  const int64_t* dst_block_ids;
  int64_t n_dst_block_ids;
  const int64_t* dst_block_counts;        /* per tag, or n = 0 */
  int64_t n_dst_block_counts;
  const int64_t* dst_skip_bytes;          /* per tag, or n = 0 */
  int64_t n_dst_skip_bytes;
  const ts_span_decl* decls;
  int64_t n_decls;
  const char* const* unit_names;          /* per unit names for messages, or NULL */
} ts_pool_reshard_request;

typedef struct ts_schedule_entry {   /* ScheduleEntry (pool_reshard_planner.h:20-33) */
  int64_t src_block_id;
  int64_t dst_block_id;
  int64_t src_offset_bytes;          /* physical offset inside the source pool block */
  int64_t dst_offset_bytes;          /* physical offset inside the destination pool block */
  int64_t size_bytes;
  int32_t pool_group;
  int32_t pad_;
} ts_schedule_entry;

typedef struct ts_pool_reshard_plan ts_pool_reshard_plan;
typedef struct ts_pool_reshard_program ts_pool_reshard_program;

TS_API int ts_pool_reshard_plan_build(const ts_pool_reshard_request* request,
                                      ts_pool_reshard_plan** out);
TS_API void ts_pool_reshard_plan_destroy(ts_pool_reshard_plan* plan);
/* info[8] = {groups, active source units, expected_block_count, parallelism,
 * expected_pushes_per_pool, transfer pool count, entries (all units), units}. */
TS_API int ts_pool_reshard_plan_info(const ts_pool_reshard_plan* plan, int64_t* info);
/* One source unit's schedule (capacity protocol as above). */
TS_API int ts_pool_reshard_plan_entries(const ts_pool_reshard_plan* plan, int64_t src_unit,
                                        ts_schedule_entry* out, int64_t cap, int64_t* n_out);
/* Active source units in rank order (info[1] of them) and the transfer pool
 * indices (info[5]); either pointer may be NULL. */
TS_API int ts_pool_reshard_plan_units(const ts_pool_reshard_plan* plan, int64_t* units,
                                      int32_t* pool_indices);
/* sizes[4] = {pools, destination blocks, expected pushes, order rank}; the
 * arrays (may be NULL) receive the pool indices, destination block ids and
 * expected extent bytes per destination block. */
TS_API int ts_pool_reshard_plan_group(const ts_pool_reshard_plan* plan, int64_t group,
                                      int64_t* sizes, int32_t* pool_indices, int64_t* dst_ids,
                                      int64_t* extents);

/* Plans that arrive from a controller (the data fields of StartTransferRequest
 * with its ShardPushEntryProto / PoolGroup lists,
 * tpu_sync/rpc/raiden_service.proto).  dst_peer is an id for the entry's
 * destination endpoint (< 0 stands for an empty address); source_rank is the
 * entry's shard_push_schedules key. */
typedef struct ts_received_entry {
  int32_t source_rank;
  int32_t dst_peer;
  int64_t dst_shard_idx;
  int64_t src_block_id;
  int64_t dst_block_id;
  int64_t src_offset_bytes;
  int64_t dst_offset_bytes;
  int64_t size_bytes;
  int64_t src_stride_bytes;
  int64_t dst_stride_bytes;
  int32_t count;
  int32_t pool_group;
} ts_received_entry;

typedef struct ts_received_group {
  const int32_t* pool_indices;
  int64_t n_pool_indices;
  const int64_t* dst_block_ids;
  int64_t n_dst_block_ids;
  const int64_t* extents;            /* dst_expected_extent_bytes */
  int64_t n_extents;
  int32_t expected_pushes;
  int32_t order_rank;
} ts_received_group;

typedef struct ts_received_plan {
  const int32_t* transfer_pool_indices;
  int64_t n_transfer_pools;
  const char* const* pool_dtype_tags;  /* one per pool of the local table */
  int64_t n_pool_dtype_tags;
  const ts_received_group* groups;
  int64_t n_groups;
  const ts_received_entry* entries;    /* all schedules' entries */
  int64_t n_entries;
  int64_t n_schedules;                 /* number of shard_push_schedules keys */
  int32_t parallelism;
  int32_t pad_;
} ts_received_plan;

/* The executor's checks of a received plan against the local pool table:
 * ValidatePoolReshardPlan and, for a receiver, the exact-coverage and push
 * accounting of ValidatePoolReshardReceiverCoverage
 * (tpu_sync/core/kv_cache_manager_with_transfer.cc:742-1150); same codes and
 * messages.  The transport identity fields (req_id, uuid, use_block_chunks)
 * are the control plane's and are not checked here. */
TS_API int ts_pool_reshard_validate(const ts_received_plan* plan,
                                    const ts_pool_spec* local_pools, int64_t n_local_pools,
                                    int64_t num_shards, const int64_t* local_block_ids,
                                    int64_t n_local_block_ids, int is_sender);
/* An executable plan from a received one: runs the sender's checks against
 * src_pools / src_block_ids and the receiver's against dst_pools /
 * dst_block_ids (messages prefixed "sender: " / "receiver: "), so every
 * entry of the result lies inside both sides' declared pool regions. */
TS_API int ts_pool_reshard_plan_from_received(const ts_received_plan* plan,
                                              const ts_pool_spec* src_pools,
                                              const ts_pool_spec* dst_pools, int64_t n_pools,
                                              const int64_t* src_block_ids,
                                              int64_t n_src_block_ids,
                                              const int64_t* dst_block_ids,
                                              int64_t n_dst_block_ids, int64_t dst_num_shards,
                                              ts_pool_reshard_plan** out);

/* Pool reshard execution: replaces PoolReshardPush / StartPoolReshardPush /
 * OnPoolReceived + H2dPoolBlocks (D2H, TCP push, H2D;
 * tpu_sync/core/kv_cache_manager_with_transfer.cc:1152-1335, :2665-2805) by
 * one kernel on the source GPU that stores every entry of `src_unit`, for
 * every pool of its group, into the destination storages.  Storage pointers
 * are indexed by pool storage_index: the source unit's device storages and
 * the destination's storages as this device addresses them (its own memory,
 * a peer pointer with peer access enabled, or a CUDA IPC mapping opened on
 * this device), with their sizes in bytes: every transferred pool must fit
 * its storages (checked), so no copy reaches outside them.  create uploads
 * two small tables per pool group (device allocations owned by the program);
 * launch queues one kernel per group on `stream`. */
TS_API int ts_pool_reshard_program_create(const ts_pool_reshard_plan* plan, int64_t src_unit,
                                          int device, const uint64_t* src_storage_ptrs,
                                          const uint64_t* dst_storage_ptrs,
                                          const uint64_t* src_storage_bytes,
                                          const uint64_t* dst_storage_bytes, int64_t n_storages,
                                          ts_pool_reshard_program** out);
TS_API int ts_pool_reshard_program_info(const ts_pool_reshard_program* prog, int64_t* n_tasks,
                                        uint64_t* bytes);
TS_API int ts_pool_reshard_program_launch(ts_pool_reshard_program* prog, void* stream,
                                          int max_ctas);
TS_API void ts_pool_reshard_program_destroy(ts_pool_reshard_program* prog);

/* ------------------------------------------------------------------------ */
/* Block-movement kernels (manager-free).                                    */
/* ------------------------------------------------------------------------ */

/* One (layer, shard) storage as the kernels see it: a device buffer whose
 * dim-0 slices are blocks of `block_bytes` bytes, and the byte offset of this
 * storage's slot inside one staging block.  Lives in DEVICE memory when passed
 * to the kernels below (an array of n_storages entries, 16-byte aligned). */
typedef struct ts_block_storage {
  uint64_t dev_ptr;      /* device address of block 0 */
  uint64_t block_bytes;  /* bytes of one block of this storage */
  uint64_t dev_bytes;    /* bytes of the storage on the device (bounds check) */
  uint64_t stage_off;    /* byte offset of this storage inside a staging block */
} ts_block_storage;

/* Extract (gather): staging[k*stage_pitch + st[s].stage_off + b] =
 *   storage s block ids[k], byte b; for every k < n_blocks, s < n_storages.
 * `ids` is a device array of n_blocks int64.  The staging layout is
 * block-major: one staging block holds that block of every storage
 * (the "[blocks, layers, K/V, ...]" staging of the reference's configs).
 * Replaces the per-(storage, run) DMA loop of DispatchD2hWork
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:2036-2124) on the device side.
 * `err_flag` (device or host-mapped int, may be 0) receives 1 when an id is
 * out of the storage's bounds (that block is skipped).  The table is read on
 * the device only (the kernel scans it for block sizes and alignment), so
 * the call queues its kernel on `stream` and returns without waiting for the
 * device. */
TS_API int ts_kv_extract(int device, const ts_block_storage* d_storages, int n_storages,
                  const int64_t* d_ids, int64_t n_blocks, void* d_staging,
                  uint64_t stage_pitch, int* err_flag, void* stream);

/* Insert (scatter), the inverse of ts_kv_extract; replaces DispatchH2dWork's
 * per-run copies (tpu_sync/kv_cache/kv_cache_manager_base.cc:1945-2033). */
TS_API int ts_kv_insert(int device, const ts_block_storage* d_storages, int n_storages,
                 const int64_t* d_ids, int64_t n_blocks, const void* d_staging,
                 uint64_t stage_pitch, int* err_flag, void* stream);

/* Fused extract + bf16 -> fp8 e4m3 cast.  Storages hold bf16; per (block,
 * storage) one fp32 scale = absmax/448 (1 if absmax is 0) is written to
 * staging[k*stage_pitch + scale_off + 4*s] and the payload
 * e4m3_rn_satfinite(x / scale) to staging[k*stage_pitch + st[s].stage_off ...]
 * (block_bytes/2 bytes).  No reference counterpart (new in this build).
 * pitch, staging and scale_off alignment is checked on the host
 * (TS_INVALID_ARGUMENT); a storage whose address, block bytes or stage offset
 * is not a multiple of 16 is found by the kernel, which then sets *err_flag
 * to 2 and moves nothing. */
TS_API int ts_kv_extract_fp8(int device, const ts_block_storage* d_storages,
                      int n_storages, const int64_t* d_ids, int64_t n_blocks,
                      void* d_staging, uint64_t stage_pitch, uint64_t scale_off,
                      int* err_flag, void* stream);

/* Inverse of ts_kv_extract_fp8: x = bf16_rn(float(q) * scale). */
TS_API int ts_kv_insert_fp8(int device, const ts_block_storage* d_storages,
                     int n_storages, const int64_t* d_ids, int64_t n_blocks,
                     const void* d_staging, uint64_t stage_pitch,
                     uint64_t scale_off, int* err_flag, void* stream);

/* Offload without device allocation: for callers that cannot cudaMalloc
 * (an engine that has handed nearly all HBM to its own KV pool or
 * allocator, where an extra cudaMalloc fails or fragments that pool, and
 * cudaMalloc / cudaFree may synchronise the device under its running work).
 * No counterpart in the reference.  For k < n_blocks and every storage s:
 *   host_dst[dst_ids[k]*host_pitch + st[s].stage_off + b] = storage s block
 *   src_ids[k], byte b
 * (the block-major layout of the manager's host tier; bytes of a host block
 * that no storage slot covers are written as zeros).  `storages` is a HOST
 * array of at most 512 entries (passed to the gather kernel by value), and
 * src_ids / dst_ids are HOST arrays: every check (slots inside the pitch, ids
 * against the storages and host_blocks) is made on the host before anything
 * is queued, and nothing is read back from the device, so the call returns
 * without waiting for it.  host_dst is pinned (or registered) host memory of
 * host_blocks blocks.  Staging is a file-scope device array of 64 MiB: a
 * host_pitch above that is rejected (TS_OUT_OF_RANGE).  Allocates nothing;
 * everything is queued on `stream` (synchronise it to know the copy landed).
 * Each call looks up the array's device address (the first lookup on a device
 * also loads this library's device code there); the array is shared, so
 * calls that overlap on the GPU (other streams) race on it. */
TS_API int ts_kv_offload_noalloc(int device, const ts_block_storage* storages,
                                 int n_storages, const int64_t* src_ids,
                                 const int64_t* dst_ids, int64_t n_blocks,
                                 void* host_dst, uint64_t host_pitch,
                                 int64_t host_blocks, void* stream);

/* ------------------------------------------------------------------------ */
/* Strided chunk copy (weight-sync reshard executor).                        */
/* ------------------------------------------------------------------------ */

/* One strided chunk of the reshard plan, in ELEMENTS of the source/dest
 * tensors: count rows of `size` elements from src + src_off + c*src_stride to
 * dst + dst_off + c*dst_stride.  The reference's ShardPushEntryProto carries the
 * same six numbers in bytes of one dtype (tpu_sync/rpc/raiden_service.proto:105-131,
 * expansion in tpu_sync/weight_sync/weight_synchronizer_base.cc:606-667);
 * elements are used so a chunk can change dtype on the way. */
typedef struct ts_reshard_chunk {
  uint64_t src_ptr;     /* device address of the source tensor (element 0) */
  uint64_t dst_ptr;     /* device address (local or peer) of the destination */
  int64_t src_off;
  int64_t dst_off;
  int64_t size;
  int64_t src_stride;
  int64_t dst_stride;
  int64_t count;
} ts_reshard_chunk;

typedef enum ts_dtype {
  TS_DTYPE_U8 = 0,   /* raw bytes */
  TS_DTYPE_BF16 = 1,
  TS_DTYPE_F32 = 2,
  TS_DTYPE_F16 = 3
} ts_dtype;

/* Executes n_chunks chunks (device array `d_chunks`) on `device`, converting
 * src_dtype -> dst_dtype (identity, or F32 -> BF16 round-to-nearest-even).
 * Destinations may be peer-GPU addresses (P2P stores over NVLink).
 * `d_row_prefix` is a device int64 array of n_chunks+1 entries: the prefix sum
 * of the per-chunk work items as computed by ts_reshard_work_items(). */
TS_API int ts_reshard_work_items(const ts_reshard_chunk* h_chunks, int64_t n_chunks,
                          int src_dtype, int dst_dtype, int64_t* h_prefix_out);
TS_API int ts_reshard_copy(int device, const ts_reshard_chunk* d_chunks,
                    const int64_t* d_item_prefix, int64_t n_chunks,
                    int64_t n_items, int src_dtype, int dst_dtype, void* stream);

/* Lets kernels running on `device` load and store `peer`'s memory through
 * plain device pointers (NVLink P2P); idempotent.  The in-process
 * counterpart of the reference's peer connection set-up. */
TS_API int ts_enable_peer_access(int device, int peer);

/* Maps another process's device allocation (a 64-byte cudaIpcMemHandle_t)
 * into this process FOR KERNELS RUNNING ON `device`: the handle is opened
 * with `device` current and lazy peer access, so `device`'s kernels can
 * store into the peer GPU's memory over NVLink.  Replaces the TCP push of
 * the reference's cross-host transfers on one NVSwitch box.  Mappings are
 * shared per (device, handle) in a process and reference-counted: every
 * ts_ipc_open is paired with a ts_ipc_close, the last one unmaps. */
TS_API int ts_ipc_open(int device, const void* handle_bytes, void** base_out);
/* The exporting side: the 64-byte handle of the allocation holding dev_ptr and
 * dev_ptr's byte offset inside it (cudaMalloc'ed memory, e.g. torch's default
 * caching allocator; not virtual-memory-mapped segments). */
TS_API int ts_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
TS_API int ts_ipc_close(int device, void* base);

/* Weight-sync reshard pushed by the copy engines: the chunks' fp32 -> bf16
 * cast goes to a local staging buffer (rows packed), and every staged chunk
 * moves to its (local or peer) destination with one cudaMemcpy2DAsync;
 * groups of chunks pipeline the cast against the copies.  Same-dtype chunks
 * are copied from the source directly.  Launches are ordered on `stream`
 * (after its earlier work, before its later work).  Replaces, like
 * ts_reshard_copy, PushWeightsResharded's D2H + TCP push + H2D
 * (weight_synchronizer_base.cc:558-760). */
typedef struct ts_reshard_ce ts_reshard_ce;
TS_API int ts_reshard_ce_create(int device, const ts_reshard_chunk* chunks, int64_t n,
                                int src_dtype, int dst_dtype, int n_groups,
                                ts_reshard_ce** out);
TS_API int ts_reshard_ce_launch(ts_reshard_ce* program, void* stream);
TS_API int ts_reshard_ce_info(ts_reshard_ce* program, int64_t* groups,
                              uint64_t* staging_bytes, int64_t* copies);
TS_API int ts_reshard_ce_destroy(ts_reshard_ce* program);

/* Weight-sync reshard pulled by the receivers ("staged pull").  On this
 * platform a GPU's NVLink loads of a peer's memory run at the peer-copy
 * rate while its stores into a peer stop near 0.92 of it, so this variant
 * moves the bytes with loads: the sender casts its fp32 shard into a local
 * bf16 staging buffer of the same element layout, group by group, and
 * publishes each group's readiness in a /dev/shm mailbox; every receiver
 * maps the staging (CUDA IPC) and, as groups become ready, launches the
 * strided copies of its chunks that need nothing beyond them.  No kernel
 * waits on another GPU: readiness travels through host memory.  Replaces,
 * like ts_reshard_copy, PushWeightsResharded's D2H + TCP push + H2D
 * (weight_synchronizer_base.cc:558-760), with the direction of the data
 * plane's requests reversed (the receiver reads).
 *
 * Sender: `name` is the mailbox (a /dev/shm name; the creator owns and
 * unlinks it).  `src` holds n_elems fp32 values (the shard, as the
 * receivers' chunks address it).  n_groups (1..61) sets the group size,
 * n_elems / n_groups rounded up to 8 elements; the first three groups are
 * 1/8, 1/4 and 1/2 of it, so receivers can start early.  stage() casts every group
 * on the sender's stream ordered after `stream`'s queued work (the caller's
 * stream then waits for the staging to be written) and publishes group g as
 * soon as it is written; before overwriting the staging it waits, at most
 * `timeout_ms`, until every receiver that attached has finished pulling the
 * previous generation (TS_DEADLINE_EXCEEDED otherwise, nothing queued).
 * wait() returns once every group of the last stage() is published.
 * destroy() waits up to 2 s for attached receivers to detach before it
 * frees the staging; destroy the receivers first. */
typedef struct ts_wpull_src ts_wpull_src;
TS_API int ts_wpull_src_create(int device, const char* name, const void* src_f32,
                               int64_t n_elems, int n_groups, ts_wpull_src** out);
TS_API int ts_wpull_src_stage(ts_wpull_src* src, void* stream, int64_t timeout_ms);
TS_API int ts_wpull_src_wait(ts_wpull_src* src, int64_t timeout_ms);
TS_API int ts_wpull_src_info(ts_wpull_src* src, int64_t* generation, int64_t* groups,
                             uint64_t* staging_bytes, int64_t* receivers);
TS_API int ts_wpull_src_destroy(ts_wpull_src* src);

/* Receiver: attaches to the mailboxes `names[0..n_src)`.  Each chunk's
 * src_ptr is the INDEX of its sender in `names` (not an address); src_off,
 * strides and size count bf16 elements of that sender's staging; dst_ptr /
 * dst_off / dst_stride address this GPU's bf16 destination.  Every chunk is
 * checked against its sender's staging before anything is created.  pull()
 * is one generation: it launches, on `stream` and in group order, the
 * copies of every chunk as soon as each sender has published the groups the
 * chunk reads (the host thread waits on the mailboxes, at most timeout_ms in
 * all; TS_DEADLINE_EXCEEDED leaves the copies already queued in place), then
 * tells the senders when the copies have finished, so their next stage()
 * may overwrite the staging.  Later work on `stream` sees the bytes. */
typedef struct ts_wpull_dst ts_wpull_dst;
TS_API int ts_wpull_dst_create(int device, const char* const* names, int n_src,
                               const ts_reshard_chunk* chunks, int64_t n_chunks,
                               ts_wpull_dst** out);
TS_API int ts_wpull_dst_pull(ts_wpull_dst* dst, void* stream, int64_t timeout_ms);
TS_API int ts_wpull_dst_info(ts_wpull_dst* dst, int64_t* generation, int64_t* launches,
                             uint64_t* bytes);
TS_API int ts_wpull_dst_destroy(ts_wpull_dst* dst);

/* ------------------------------------------------------------------------ */
/* Weight synchronizer (resharded push of controller-made schedules).        */
/* ------------------------------------------------------------------------ */

/* Replaces WeightSynchronizerBase's resharded push
 * (tpu_sync/weight_sync/weight_synchronizer_base.cc:558-760): the trainer's
 * [layer][shard] buffers, a registered plan of ShardPushEntry lists, and its
 * execution as one strided-copy kernel per source GPU storing straight into
 * the destinations (no D2H, TCP push, receiver H2D). */
typedef struct ts_wsync ts_wsync;

/* One [layer][shard] buffer of the synchronizer (the reference's host mirror
 * of that buffer is not needed: the kernel reads the device buffer). */
typedef struct ts_wsync_buffer {
  uint64_t dev_ptr;  /* device address */
  uint64_t nbytes;   /* its size (the reference's GetHostSize) */
  int32_t device;    /* CUDA device ordinal */
  int32_t pad_;
} ts_wsync_buffer;

/* ShardPushEntryProto (tpu_sync/rpc/raiden_service.proto:105-131) plus the
 * map key it sits under in StartTransferRequest.shard_push_schedules. */
typedef struct ts_shard_push_entry {
  int32_t src_shard_idx;  /* local shard whose schedule holds the entry */
  int32_t has_layer_idx;  /* 0: the layer named by the request's first source unit */
  int32_t layer_idx;
  int32_t pad_;
  const char* dst_peer;
  int64_t dst_shard_idx;
  uint64_t src_offset_bytes;
  uint64_t dst_offset_bytes;
  uint64_t size_bytes;
  uint64_t src_stride_bytes;
  uint64_t dst_stride_bytes;
  int64_t count;          /* <= 0 means 1, as in the reference */
} ts_shard_push_entry;

/* Where the bytes of (peer, layer, destination shard) go, as the source's
 * kernels address them: its own memory, a peer GPU's memory (device >= 0:
 * peer access is enabled by the registration), or a CUDA IPC mapping opened
 * for the source device (device = -1). */
typedef struct ts_wsync_dest {
  const char* peer;
  int64_t layer_idx;
  int64_t dst_shard_idx;
  uint64_t dst_ptr;
  uint64_t nbytes;
  int32_t device;
  int32_t pad_;
} ts_wsync_dest;

/* num_layers x num_shards buffers, row-major [layer][shard]; layer_names may
 * be NULL (names "0", "1", ...), as WeightSynchronizerBase's layer names. */
TS_API int ts_wsync_create(const ts_wsync_buffer* buffers, int num_layers, int num_shards,
                           const char* const* layer_names, ts_wsync** out);
/* Checks every entry, in the reference's order and words (per local shard in
 * order, its entries in order: layer index or the fallback layer named
 * src_data_name, NULL = no source units -> "src_units list cannot be empty",
 * unknown -> TS_NOT_FOUND "Layer name not found in WeightSynchronizer: <name>";
 * "Layer index out of bounds: <i>"; "Push range out of bounds" per contiguous
 * payload or per repeat), then that its destination is registered and holds
 * its range ("No destination for peer ...", "Push destination range out of
 * bounds"), and replaces the registered plan only if all pass.  Uploads the
 * plan's task tables (device allocations owned by the object; a push still
 * running on the previous plan is waited for first). */
TS_API int ts_wsync_register_plan(ts_wsync* w, const ts_shard_push_entry* entries,
                                  int64_t n_entries, const char* src_data_name,
                                  const ts_wsync_dest* dests, int64_t n_dests);
/* Queues the registered plan, ordered after the work already queued on
 * `stream` (any device of this process; 0 = the current device's default
 * stream): one kernel per source GPU on the object's own streams. */
TS_API int ts_wsync_push(ts_wsync* w, void* stream);
/* TS_OK when the last push has landed, TS_PENDING before. */
TS_API int ts_wsync_query(ts_wsync* w);
/* Waits for the last push (timeout_ms < 0: no limit; TS_DEADLINE_EXCEEDED). */
TS_API int ts_wsync_wait(ts_wsync* w, int64_t timeout_ms);
/* Makes `stream` wait on the device for the last push. */
TS_API int ts_wsync_stream_wait(ts_wsync* w, void* stream);
/* Tasks (one per non-empty entry) and bytes of the registered plan. */
TS_API int ts_wsync_info(ts_wsync* w, int64_t* n_tasks, uint64_t* bytes);
TS_API void ts_wsync_destroy(ts_wsync* w);

/* ------------------------------------------------------------------------ */
/* Paged KV relayout (disaggregated prefill -> decode hand-off).             */
/* ------------------------------------------------------------------------ */

/* Geometry of one paged KV storage.  A block holds `block_tokens` tokens of
 * `heads` heads of `head_bytes` bytes, ordered head-major ([heads][tokens])
 * when head_major != 0 else token-major ([tokens][heads]). */
typedef struct ts_page_geometry {
  int64_t block_tokens;
  int64_t heads;
  int64_t head_bytes;
  int32_t head_major;
  int32_t pad_;
} ts_page_geometry;

/* For every storage s (n_storages pairs of device base addresses, src_bases[s]
 * and dst_bases[s], device arrays of uint64), every sequence q < n_seqs and
 * token t < seq_tokens: copies each head vector of token t from source block
 * src_table[q*src_table_stride + t/src.block_tokens] to destination block
 * dst_table[q*dst_table_stride + t/dst.block_tokens] in the destination order.
 * src.heads == dst.heads and src.head_bytes == dst.head_bytes are required.
 * Destination addresses may be a peer GPU's (P2P stores).  Every storage
 * holds at least src_pages (dst_pages) pages: a table entry outside
 * [0, pages) is skipped and sets *d_err (a device int, may be NULL) to 1. */
TS_API int ts_kv_relayout(int device, const uint64_t* d_src_bases,
                   const uint64_t* d_dst_bases, int n_storages,
                   ts_page_geometry src, ts_page_geometry dst,
                   const int32_t* d_src_table, int64_t src_table_stride,
                   const int32_t* d_dst_table, int64_t dst_table_stride,
                   int64_t n_seqs, int64_t seq_tokens, int64_t src_pages,
                   int64_t dst_pages, int* d_err, void* stream);

/* ------------------------------------------------------------------------ */
/* Pinned host tier.                                                         */
/* ------------------------------------------------------------------------ */

typedef struct ts_host_tier ts_host_tier;

/* Allocates `bytes` of DMA-registered host memory: anonymous mmap, or a
 * /dev/shm segment when shm_name is non-empty, registered with
 * cudaHostRegister (Portable|Mapped).  Replaces XlaHostMemoryAllocator /
 * SharedMemoryHostMemoryAllocator (tpu_sync/core/host_memory_allocator.cc:125-196,
 * :217-407).  `register_with_cuda` = 0 skips the CUDA registration (CPU use).
 * *warm_out = 1 when an existing /dev/shm segment with the same name,
 * model_uid and geometry was attached (warm boot). */
TS_API int ts_host_tier_create(uint64_t bytes, const char* shm_name,
                        const char* model_uid, uint64_t geometry_tag,
                        int register_with_cuda, ts_host_tier** out,
                        int* warm_out);
TS_API void* ts_host_tier_ptr(ts_host_tier* tier);
TS_API uint64_t ts_host_tier_bytes(ts_host_tier* tier);
TS_API int ts_host_tier_destroy(ts_host_tier* tier, int unlink_shm);

/* ------------------------------------------------------------------------ */
/* KV cache manager (replaces KVCacheManagerBase's device path).            */
/* ------------------------------------------------------------------------ */

typedef struct ts_manager ts_manager;
typedef struct ts_event ts_event;

typedef struct ts_storage_desc {
  uint64_t dev_ptr;   /* device address of the (layer, shard) storage */
  uint64_t nbytes;    /* its on-device size in bytes */
  int64_t dim0;       /* its dim-0 extent (number of blocks) */
  int32_t device;     /* CUDA device ordinal */
  int32_t pad_;
} ts_storage_desc;

typedef struct ts_manager_opts {
  int64_t host_blocks;         /* host tier capacity in blocks (reference default 64) */
  int64_t chunk_blocks;        /* blocks per pipelined chunk (0 = default 64) */
  const char* shm_name;        /* "" / NULL = anonymous pinned memory */
  const char* model_uid;       /* stored in the /dev/shm header */
  int32_t fp8;                 /* 1: host tier holds fp8 e4m3 + per-block scales */
  int32_t mode;                /* per direction (bit 0 offload, bit 1 reload):
                                  0 = staged: extract/insert kernels + copy-engine
                                  DMAs via HBM staging slots; 1 = direct: the
                                  kernels read / write the mapped host tier over
                                  PCIe themselves */
  int32_t copy_streams;        /* staged mode: copy streams per direction (1..4) */
  int32_t max_ctas;            /* grid cap of the kernels (0 = every SM) */
  int32_t reload_staged_every; /* direct reloads only: every n-th chunk goes through
                                  the copy engines instead (0 = none), so both
                                  H2D mechanisms run at once */
  int32_t sched;               /* SM scheduling of the two directions, a sum of
                                  TS_SCHED_* flags (0 = neither) */
  int32_t numa_node;           /* NUMA node of the host tier's pages: 0 = the
                                  node of the device's PCI function (the
                                  reference's DetectAndAssignNumaNode), n > 0 =
                                  node n - 1 (its assigned_numa_node_override),
                                  -1 = no placement.  Applied on hosts with
                                  more than one node. */
} ts_manager_opts;

/* ts_manager_opts.sched flags. */
enum {
  /* offload kernels run on a stream of the device's highest priority, so the
   * gather takes SM slots ahead of a long-running reload kernel */
  TS_SCHED_OFFLOAD_PRIORITY = 1,
  /* direct reloads launch one CTA per 16 KiB piece instead of a persistent
   * grid, so their CTAs retire (and free SM slots) as each piece lands */
  TS_SCHED_RELOAD_PER_PIECE = 2,
  /* consecutive direct reload chunks alternate between two kernel streams,
   * so one chunk's last wave overlaps the next chunk's first (not used when
   * a destination block repeats inside the call) */
  TS_SCHED_RELOAD_OVERLAP = 4,
  /* staged (HBM -> HBM) extract and insert kernels move 16 KiB pieces with
   * bulk copies through shared memory: one CTA of 6 warps per SM instead of
   * a full-SM grid of vector loads (plain copies of 16-byte aligned tables;
   * fp8 and direct-mode kernels are unchanged) */
  TS_SCHED_BULK_COPY = 8,
  /* direct reloads read the mapped host tier with 32-byte (256-bit) vector
   * loads instead of 16-byte ones (tables whose storages, slots and tier are
   * all 32-byte aligned; others keep 16-byte vectors) */
  TS_SCHED_WIDE_LOADS = 16,
};

/* Creates a manager over num_layers x num_shards storages (row-major
 * [layer][shard]).  Replaces the device-backed KVCacheManagerBase constructor
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:223-372): block bytes of layer l
 * = nbytes(l) / dim0(layer 0) (layer_block_byte_size, kv_cache_manager_base.h:434-439),
 * host mirror of host_blocks blocks per storage. */
TS_API int ts_mgr_create(const ts_storage_desc* storages, int num_layers,
                  int num_shards, const ts_manager_opts* opts,
                  ts_manager** out);
TS_API int ts_mgr_destroy(ts_manager* mgr);

/* Device -> host tier: KVCacheManagerBase::D2h
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:2616 -> :792 -> :652 -> :2036).
 * n == 0 means "whole storages" as in the reference.  layer_idx / shard_idx
 * = -1 mean all.  The copy is ordered after the work already queued on
 * `stream`.  *out receives an event handle to query/wait/release. */
TS_API int ts_d2h(ts_manager* mgr, const int64_t* src, const int64_t* dst,
           const int64_t* sizes, int64_t n_src, int64_t n_dst, int64_t n_sizes,
           int64_t layer_idx, int64_t shard_idx, void* stream, ts_event** out);

/* Host tier -> device: KVCacheManagerBase::H2d
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:2575 -> :518 -> :1945). */
TS_API int ts_h2d(ts_manager* mgr, const int64_t* src, const int64_t* dst,
           const int64_t* sizes, int64_t n_src, int64_t n_dst, int64_t n_sizes,
           int64_t layer_idx, int64_t shard_idx, void* stream, ts_event** out);

/* Host address of (layer, shard, host block) and the layout of the tier.
 * Replaces GetBlockHostPointerValue (kv_cache/kv_cache_manager_base.h:358-362). */
TS_API int ts_mgr_host_block_ptr(ts_manager* mgr, int64_t layer_idx, int64_t shard_idx,
                          int64_t block_id, uint64_t* ptr_out,
                          uint64_t* bytes_out);
/* RaidenManagerBase::assigned_numa_node (tpu_sync/core/raiden_manager_base.h:102):
 * the node assigned to the manager (-1 = none known) and whether the host
 * tier's pages were placed on it (0 on single-node hosts, or when the kernel
 * refused the memory policy). */
TS_API int ts_mgr_numa_node(ts_manager* mgr, int* node, int* placed);
/* The NUMA node sysfs lists for a PCI bus id ("0000:1b:00.0" or CUDA's
 * 8-digit-domain form), -1 when unknown; sysfs_root NULL = "/sys".  Host
 * logic of GetPjRtDeviceNumaNode's role in DetectAndAssignNumaNode
 * (tpu_sync/core/raiden_manager_base.cc:47-78); no CUDA call. */
TS_API int ts_pci_numa_node(const char* bus_id, const char* sysfs_root, int* node);
TS_API int ts_mgr_info(ts_manager* mgr, int64_t* host_blocks, uint64_t* host_block_pitch,
                int64_t* major_dim, uint64_t* bytes_per_block);

/* Explicit block pools: KVCacheManagerBase::RegisterPools
 * (tpu_sync/kv_cache/kv_cache_manager_base.cc:1653-1712).  Until it is
 * called the manager has implicit pools, one per storage (layer) whose
 * block bytes are positive (EnsureImplicitPools, :1554-1590).  The host
 * mirror of storage s shares its byte offsets: device byte x of the storage
 * lives in host block x / bb(s) at offset x % bb(s) of that storage's slot.
 * Pools whose live extent reaches past host_blocks * bb(s) are rejected
 * (the host tier is one allocation and is not regrown).  Not available on an
 * fp8 host tier. */
TS_API int ts_mgr_register_pools(ts_manager* mgr, const ts_pool_spec* pools, int64_t n);
TS_API int ts_mgr_num_pools(ts_manager* mgr, int64_t* n, int* explicit_pools);
/* Geometry of pool `pool_idx` (strings are not returned: the caller keeps
 * the specs it registered; implicit pools are tagged "opaque" with one region
 * "block"). */
TS_API int ts_mgr_pool_geometry(ts_manager* mgr, int64_t pool_idx, int64_t* storage_index,
                                int64_t* block_stride_bytes, int64_t* num_blocks);

/* CopyPoolBlocks (kv_cache_manager_base.cc:1789-1858): copies the declared-
 * live extents of the given pool blocks between the device storage and its
 * host mirror (same byte offsets); shard_idx = -1 copies every shard.
 * Whole aligned blocks move as strided DMAs, partial regions with one
 * segment-copy kernel over the mapped host tier. */
TS_API int ts_d2h_pool_blocks(ts_manager* mgr, int64_t pool_idx, const int64_t* block_ids,
                              int64_t n_ids, int64_t shard_idx, void* stream, ts_event** out);
TS_API int ts_h2d_pool_blocks(ts_manager* mgr, int64_t pool_idx, const int64_t* block_ids,
                              int64_t n_ids, int64_t shard_idx, void* stream, ts_event** out);
/* GetPoolBlockRef (kv_cache_manager_base.cc:1714-1760): host address of one
 * pool block (the block's live bytes must sit inside one host block of the
 * block-major tier, which holds whenever the pool's blocks are the storage's
 * blocks). */
TS_API int ts_mgr_pool_block_ref(ts_manager* mgr, int64_t pool_idx, int64_t shard_idx,
                                 int64_t block_id, uint64_t* host_ptr);

/* Per-launch timing of the manager's kernels (CUDA events around every
 * extract / insert launch on its kernel streams).  ts_mgr_kernel_stats
 * returns and resets the launches, their device time (the union of the
 * launches' intervals: launches that overlap on two streams count once) and
 * their algorithmic HBM bytes (read + write) for which = 0 (extract) or
 * 1 (insert).
 * Plays the role of the reference's per-op duration telemetry
 * (JoinAndRecordTelemetry, tpu_sync/kv_cache/kv_cache_manager_base.cc:205-219). */
TS_API int ts_mgr_set_profiling(ts_manager* mgr, int on);
TS_API int ts_mgr_kernel_stats(ts_manager* mgr, int which, int64_t* launches,
                               double* total_ms, uint64_t* bytes);

/* Completion handles (replace PjRtCopyFuture / RaidenFuture,
 * tpu_sync/core/raw_transfer_core.h:379-621,
 * tpu_sync/frameworks/torch/tpu_raiden_torch_module.cc:179-211). */
TS_API int ts_event_query(ts_event* ev);               /* TS_OK, TS_PENDING or error */
TS_API int ts_event_wait(ts_event* ev, int64_t timeout_ms); /* <0: no timeout */
TS_API int ts_event_error(ts_event* ev, char* buf, size_t len);
/* Makes `stream` wait for the event on the device (no host synchronisation). */
TS_API int ts_event_stream_wait(ts_event* ev, void* stream);
TS_API int ts_event_elapsed_ms(ts_event* ev, float* ms);
TS_API void ts_event_release(ts_event* ev);

/* ------------------------------------------------------------------------ */
/* Tier-2 prefix cache (KVCacheStore, local paths).                          */
/* ------------------------------------------------------------------------ */

/* BlockStatus of tpu_sync/kv_cache/kv_cache_store_backend.h:39-45. */
enum {
  TS_BLOCK_INIT = 0,
  TS_BLOCK_REMOTE = 1,
  TS_BLOCK_HBM = 2,
  TS_BLOCK_HOST = 3,
  TS_BLOCK_HOST_AND_HBM = 4
};

/* RaidenBlockId without the RaidenId strings (local blocks only). */
typedef struct ts_block_info {
  int32_t host_block_id;
  int32_t device_block_id;
  int32_t status;
  int32_t pad_;
} ts_block_info;

typedef struct ts_store ts_store;

/* Block hashes are byte strings packed back to back in `keys`, key i being
 * keys[offs[i] .. offs[i+1]).  The store's Save / Load move bytes through
 * `mgr` (ts_d2h / ts_h2d); with mgr == NULL transfers complete at once
 * (host-only state machine).  capacity = LRU entries; host_blocks = host
 * tier blocks the allocator hands out.
 * Replaces KVCacheStore + HostOffloadBackend + LRUCache + LogicalBlockManager
 * local paths: tpu_sync/kv_cache/kv_cache_store.h:100-808,
 * tpu_sync/kv_cache/host_offload_backend.cc:154-470,
 * tpu_sync/kv_cache/lru_cache.h:41-364,
 * tpu_sync/kv_cache/logical_block_manager.cc:32-224. */
TS_API int ts_store_create(ts_manager* mgr, int64_t capacity, int64_t host_blocks,
                           ts_store** out);
TS_API int ts_store_destroy(ts_store* store);
/* KVCacheStore::Lookup (kv_cache_store.cc:837-904): hits up to the first miss,
 * pinned when pin_found != 0. */
TS_API int ts_store_lookup(ts_store* store, const uint8_t* keys, const int64_t* offs,
                           int64_t n, int pin_found, ts_block_info* out,
                           int64_t* n_found);
/* KVCacheStore::Insert (kv_cache_store.cc:906-939), all-or-nothing, pins. */
TS_API int ts_store_insert(ts_store* store, const uint8_t* keys, const int64_t* offs,
                           int64_t n, const ts_block_info* slices, int64_t n_slices,
                           int on_host);
TS_API int ts_store_release(ts_store* store, const uint8_t* keys, const int64_t* offs,
                            int64_t n);
TS_API int ts_store_pin_count(ts_store* store, const uint8_t* key, int64_t len, int* out);
/* KVCacheStore::SaveLocal (kv_cache_store.cc:977-1058): HBM -> host tier. */
TS_API int ts_store_save(ts_store* store, const uint8_t* keys, const int64_t* offs,
                         int64_t n, void* stream);
/* KVCacheStore::Load (kv_cache_store.cc:1060-1140): host tier -> HBM. */
TS_API int ts_store_load(ts_store* store, const uint8_t* keys, const int64_t* offs,
                         int64_t n, const int32_t* device_block_ids, int64_t n_ids,
                         void* stream);
/* PollSaveStatus (which = 0: done, failed, pending, existing, unregistered) /
 * PollLoadStatus (which = 1: done, failed, pending), kv_cache_store.cc:1453-1521.
 * counts[] receives the list sizes, the keys are packed into buf / offs.
 * TS_RESOURCE_EXHAUSTED (nothing consumed) when buf_len < *need_bytes or
 * offs_len < *need_keys + 1. */
TS_API int ts_store_poll(ts_store* store, int which, int64_t* counts, uint8_t* buf,
                         int64_t buf_len, int64_t* offs, int64_t offs_len,
                         int64_t* need_bytes, int64_t* need_keys);
/* capacity, size, available space, host blocks total, free, locked. */
TS_API int ts_store_stats(ts_store* store, int64_t* stats6);
/* Test hooks: LRU order (which 0 = active MRU-first, 1 = candidates,
 * 2 = GetEvictableKeys order) and direct allocator operations
 * (op 0 deallocate, 1 allocate_target, 2 unlock, 3 access one id). */
TS_API int ts_store_lru_order(ts_store* store, int which, uint8_t* buf, int64_t buf_len,
                              int64_t* offs, int64_t offs_len, int64_t* need_bytes,
                              int64_t* need_keys);
TS_API int ts_store_allocate_host_blocks(ts_store* store, int n, int lock, int32_t* out);
TS_API int ts_store_host_block_op(ts_store* store, int op, const int32_t* ids, int64_t n);
/* Test hook: one raw operation on the LRU index (0 put, 1 pin, 2 unpin,
 * 3 peek, 4 peek including candidates, 5 pin count, 6 erase, 7 contains,
 * 8 available space, 9 size); put reports a demoted key in out_key. */
TS_API int ts_store_lru_op(ts_store* store, int op, const uint8_t* key, int64_t len,
                           const ts_block_info* in, ts_block_info* out_info,
                           int64_t* out_val, uint8_t* out_key, int64_t out_key_cap,
                           int64_t* out_key_len);

/* The manager's storages (layer-major, then shard): device, address, bytes,
 * blocks (dim 0) and block bytes of storage `index`. */
TS_API int ts_mgr_num_storages(ts_manager* mgr, int* n);
TS_API int ts_mgr_storage(ts_manager* mgr, int index, int* device, uint64_t* dev_ptr,
                          uint64_t* nbytes, int64_t* dim0, uint64_t* block_bytes);

/* ---- Same-node block hand-off between managers (pull protocol) ---------
 * Replaces the reference's NotifyForRead / StartRead / CompleteRead
 * (tpu_sync/core/kv_cache_manager_with_transfer.cc:624-665, :1478-1760)
 * and their TCP control and data planes: the producer publishes a /dev/shm
 * mailbox (its storages' CUDA IPC handles, one entry per registered read
 * with an interprocess event marking the blocks written); the consumer maps
 * the storages, waits on that event on its stream and pulls every storage's
 * bytes of each block pair with one kernel over NVLink.  Producer and
 * consumer storages must match storage for storage (count, block bytes). */
typedef struct ts_xfer_endpoint ts_xfer_endpoint;
typedef struct ts_xfer_reader ts_xfer_reader;
/* Producer: the endpoint `name` (a /dev/shm name; "ipc:" prefix accepted)
 * with max_entries concurrent reads of up to max_blocks blocks each;
 * unclaimed registrations time out after timeout_ms. */
TS_API int ts_xfer_endpoint_create(ts_manager* mgr, const char* name, int max_entries,
                                   int max_blocks, int64_t timeout_ms, ts_xfer_endpoint** out);
TS_API int ts_xfer_endpoint_destroy(ts_xfer_endpoint* ep);
TS_API int ts_xfer_endpoint_name(ts_xfer_endpoint* ep, char* buf, int64_t cap);
/* State of the producer's read `uuid`: 0 none, 2 registered (blocks still
 * being written), 3 ready, 4 being read, 5 consumed, 6 failed. */
TS_API int ts_xfer_read_state(ts_xfer_endpoint* ep, uint64_t uuid, int* state);
/* NotifyForRead: the blocks are readable once the work queued on `stream`
 * so far is done; *registered = 0 for an empty list (nothing to move). */
TS_API int ts_xfer_register_read(ts_xfer_endpoint* ep, const char* req_id, uint64_t uuid,
                                 const int64_t* block_ids, int64_t n, void* stream,
                                 int* registered);
/* Producer half of CompleteRead: req ids whose reads finished (or failed,
 * or were never claimed before the timeout), packed into buf / offs under
 * the capacity protocol (TS_RESOURCE_EXHAUSTED keeps them for a retry). */
TS_API int ts_xfer_poll_sends(ts_xfer_endpoint* ep, uint8_t* buf, int64_t buf_len,
                              int64_t* offs, int64_t offs_len, int64_t* n_out,
                              int64_t* need_bytes);
/* Consumer: reads into `mgr`'s storages; a read whose uuid the producer has
 * not registered within timeout_ms fails. */
TS_API int ts_xfer_reader_create(ts_manager* mgr, int64_t timeout_ms, ts_xfer_reader** out);
TS_API int ts_xfer_reader_destroy(ts_xfer_reader* r);
/* StartRead: remote block remote_ids[i] -> local block local_ids[i], queued
 * on `stream` behind the producer's event (later work on `stream` sees the
 * blocks).  Only blocks the producer registered under `uuid` may be read. */
TS_API int ts_xfer_start_read(ts_xfer_reader* r, const char* req_id, uint64_t uuid,
                              const char* endpoint, const int64_t* remote_ids,
                              const int64_t* local_ids, int64_t n, void* stream);
/* Consumer half of CompleteRead: which = 0 done req ids (polls first),
 * 1 failed req ids; same packing as ts_xfer_poll_sends. */
TS_API int ts_xfer_poll_reads(ts_xfer_reader* r, int which, uint8_t* buf, int64_t buf_len,
                              int64_t* offs, int64_t offs_len, int64_t* n_out,
                              int64_t* need_bytes);
TS_API int ts_xfer_reader_pending(ts_xfer_reader* r, int64_t* n);

/* ---- Crash-persistent KV block metadata --------------------------------
 * KVCacheMetadata (tpu_sync/kv_cache/kv_cache_metadata.h:19-141,
 * kv_cache_metadata.cc:27-188) on the reference's byte layout: a 128-byte
 * header {u64 magic "RAIDENKM", u32 version 1, u32 num_blocks, u32 entry
 * size 128, char model_uid[64] at offset 20} and num_blocks 128-byte entries
 * {u64 seq, u16 hash_len, u8 valid at offset 10, hash[112] at offset 16}. */
typedef struct ts_kv_metadata ts_kv_metadata;
/* KVCacheMetadata::RequiredSizeBytes; 0 for num_blocks <= 0. */
TS_API uint64_t ts_kv_metadata_required_bytes(int num_blocks);
/* KVCacheMetadataShmRegion::AttachOrFormat (kv_cache_metadata_shm.cc:29-130):
 * attach the /dev/shm segment `key` (leading '/' added) when its table
 * validates for (num_blocks, model_uid) -> *warm = 1, else unlink it and
 * format a fresh one -> *warm = 0. */
TS_API int ts_kv_metadata_open(const char* key, int num_blocks, const char* model_uid,
                               ts_kv_metadata** out, int* warm);
/* KVCacheMetadata::Format (attach == 0) / Attach (attach != 0) on caller
 * memory (64-byte aligned, >= required bytes), which must outlive the handle. */
TS_API int ts_kv_metadata_on_region(void* region, uint64_t size, int num_blocks,
                                    const char* model_uid, int attach, ts_kv_metadata** out);
/* KVCacheMetadata::Set / Clear. */
TS_API int ts_kv_metadata_set(ts_kv_metadata* m, int block_id, const uint8_t* hash,
                              int64_t len, uint64_t seq);
TS_API int ts_kv_metadata_clear(ts_kv_metadata* m, int block_id);
/* KVCacheMetadata::ValidEntries in block order: ids, seqs and the hashes
 * packed into buf (hash i = buf[offs[i] .. offs[i+1])).  *n_out / *need_bytes
 * always receive the sizes; TS_RESOURCE_EXHAUSTED (nothing written) when
 * cap < *n_out or buf_len < *need_bytes (offs holds cap + 1 values). */
TS_API int ts_kv_metadata_entries(ts_kv_metadata* m, int32_t* block_ids, uint64_t* seqs,
                                  uint8_t* buf, int64_t buf_len, int64_t* offs, int64_t cap,
                                  int64_t* n_out, int64_t* need_bytes);
/* KVCacheMetadataShmRegion::Reformat (kv_cache_metadata_shm.cc:148-160). */
TS_API int ts_kv_metadata_reformat(ts_kv_metadata* m);
TS_API int ts_kv_metadata_info(ts_kv_metadata* m, int* num_blocks, int* warm);
/* Unmaps (and, with unlink_shm, removes the segment of) an opened table. */
TS_API int ts_kv_metadata_close(ts_kv_metadata* m, int unlink_shm);
/* KVCacheStore::Evict (kv_cache_store.cc:1553-1570): unpinned HOST /
 * HOST_AND_HBM entries among the keys are erased and their host blocks
 * freed; *evicted = how many. */
TS_API int ts_store_evict(ts_store* store, const uint8_t* keys, const int64_t* offs, int64_t n,
                          int64_t* evicted);
/* Attach (or with NULL detach) a table to a store: host-resident entries are
 * recorded on insert / save / load completion and cleared on eviction and
 * rollback (HostOffloadBackend::SetMetadataEntry / ClearMetadataEntry,
 * host_offload_backend.cc:1224-1256).  The table must outlive the store or
 * be detached first. */
TS_API int ts_store_attach_metadata(ts_store* store, ts_kv_metadata* m);
/* KVCacheStore::RecoverFromLocalManifest (kv_cache_store.cc:1541-1551,
 * host_offload_backend.cc:559-617): rebuilds an empty store's LRU from the
 * table's newest entry per hash, in seq order, as HOST blocks. */
TS_API int ts_store_recover(ts_store* store, int64_t* recovered);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* TPUSYNC_B200_H_ */

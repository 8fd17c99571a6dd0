"""ctypes binding of the C ABI in ``include/tpusync_b200.h``.

The library is loaded from ``tpu_sync_b200/_lib/libtpusync_b200.so`` (built
in-tree by ``tpu_sync_b200.build``).  There is no fallback: if the library is
missing every entry point raises, so a missing build can never silently turn
into a CPU path.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libtpusync_b200.so"

# ts_status values
OK = 0
CANCELLED = 1
UNKNOWN = 2
INVALID_ARGUMENT = 3
DEADLINE_EXCEEDED = 4
NOT_FOUND = 5
ALREADY_EXISTS = 6
RESOURCE_EXHAUSTED = 8
FAILED_PRECONDITION = 9
OUT_OF_RANGE = 11
UNIMPLEMENTED = 12
INTERNAL = 13
UNAVAILABLE = 14
PENDING = 100

# ts_manager_opts.sched flags (TS_SCHED_*)
SCHED_OFFLOAD_PRIORITY = 1
SCHED_RELOAD_PER_PIECE = 2
SCHED_RELOAD_OVERLAP = 4
SCHED_BULK_COPY = 8
SCHED_WIDE_LOADS = 16

STATUS_NAMES = {
    OK: "OK", CANCELLED: "CANCELLED", UNKNOWN: "UNKNOWN",
    INVALID_ARGUMENT: "INVALID_ARGUMENT", DEADLINE_EXCEEDED: "DEADLINE_EXCEEDED",
    NOT_FOUND: "NOT_FOUND", ALREADY_EXISTS: "ALREADY_EXISTS",
    RESOURCE_EXHAUSTED: "RESOURCE_EXHAUSTED",
    FAILED_PRECONDITION: "FAILED_PRECONDITION", OUT_OF_RANGE: "OUT_OF_RANGE",
    UNIMPLEMENTED: "UNIMPLEMENTED", INTERNAL: "INTERNAL",
    UNAVAILABLE: "UNAVAILABLE", PENDING: "PENDING",
}

DTYPE_U8, DTYPE_BF16, DTYPE_F32, DTYPE_F16 = 0, 1, 2, 3

c_i64_p = ctypes.POINTER(ctypes.c_int64)
c_u64_p = ctypes.POINTER(ctypes.c_uint64)
c_i32_p = ctypes.POINTER(ctypes.c_int32)


class BlockStorage(ctypes.Structure):
  _fields_ = [("dev_ptr", ctypes.c_uint64), ("block_bytes", ctypes.c_uint64),
              ("dev_bytes", ctypes.c_uint64), ("stage_off", ctypes.c_uint64)]


class WsyncBuffer(ctypes.Structure):
  _fields_ = [("dev_ptr", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
              ("device", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class ShardPushEntry(ctypes.Structure):
  _fields_ = [("src_shard_idx", ctypes.c_int32), ("has_layer_idx", ctypes.c_int32),
              ("layer_idx", ctypes.c_int32), ("pad_", ctypes.c_int32),
              ("dst_peer", ctypes.c_char_p), ("dst_shard_idx", ctypes.c_int64),
              ("src_offset_bytes", ctypes.c_uint64), ("dst_offset_bytes", ctypes.c_uint64),
              ("size_bytes", ctypes.c_uint64), ("src_stride_bytes", ctypes.c_uint64),
              ("dst_stride_bytes", ctypes.c_uint64), ("count", ctypes.c_int64)]


class WsyncDest(ctypes.Structure):
  _fields_ = [("peer", ctypes.c_char_p), ("layer_idx", ctypes.c_int64),
              ("dst_shard_idx", ctypes.c_int64), ("dst_ptr", ctypes.c_uint64),
              ("nbytes", ctypes.c_uint64), ("device", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class ReshardChunk(ctypes.Structure):
  _fields_ = [("src_ptr", ctypes.c_uint64), ("dst_ptr", ctypes.c_uint64),
              ("src_off", ctypes.c_int64), ("dst_off", ctypes.c_int64),
              ("size", ctypes.c_int64), ("src_stride", ctypes.c_int64),
              ("dst_stride", ctypes.c_int64), ("count", ctypes.c_int64)]


class PageGeometry(ctypes.Structure):
  _fields_ = [("block_tokens", ctypes.c_int64), ("heads", ctypes.c_int64),
              ("head_bytes", ctypes.c_int64), ("head_major", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class StorageDesc(ctypes.Structure):
  _fields_ = [("dev_ptr", ctypes.c_uint64), ("nbytes", ctypes.c_uint64),
              ("dim0", ctypes.c_int64), ("device", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class ManagerOpts(ctypes.Structure):
  _fields_ = [("host_blocks", ctypes.c_int64), ("chunk_blocks", ctypes.c_int64),
              ("shm_name", ctypes.c_char_p), ("model_uid", ctypes.c_char_p),
              ("fp8", ctypes.c_int32), ("mode", ctypes.c_int32),
              ("copy_streams", ctypes.c_int32), ("max_ctas", ctypes.c_int32),
              ("reload_staged_every", ctypes.c_int32), ("sched", ctypes.c_int32),
              ("numa_node", ctypes.c_int32)]


class BlockInfo(ctypes.Structure):
  _fields_ = [("host_block_id", ctypes.c_int32), ("device_block_id", ctypes.c_int32),
              ("status", ctypes.c_int32), ("pad_", ctypes.c_int32)]


class RegionSpecC(ctypes.Structure):
  _fields_ = [("name", ctypes.c_char_p), ("offset_bytes", ctypes.c_int64),
              ("stride_bytes", ctypes.c_int64), ("unit_bytes", ctypes.c_int64),
              ("num_units", ctypes.c_int64), ("units_per_stride", ctypes.c_int64)]


class PoolSpecC(ctypes.Structure):
  _fields_ = [("tag", ctypes.c_char_p), ("storage_index", ctypes.c_int64),
              ("base_offset_bytes", ctypes.c_int64), ("block_stride_bytes", ctypes.c_int64),
              ("num_blocks", ctypes.c_int64), ("regions", ctypes.POINTER(RegionSpecC)),
              ("num_regions", ctypes.c_int64), ("dtype_tag", ctypes.c_char_p)]


class PoolExtent(ctypes.Structure):
  _fields_ = [("offset_bytes", ctypes.c_int64), ("size_bytes", ctypes.c_int64)]


class LiveSegmentC(ctypes.Structure):
  _fields_ = [("logical_offset", ctypes.c_int64), ("physical_offset", ctypes.c_int64),
              ("size", ctypes.c_int64)]


class LiveCopyChunkC(ctypes.Structure):
  _fields_ = [("src_physical", ctypes.c_int64), ("dst_physical", ctypes.c_int64),
              ("size", ctypes.c_int64)]


class ByteSpanC(ctypes.Structure):
  _fields_ = [("src_block_ordinal", ctypes.c_int64), ("src_offset_bytes", ctypes.c_int64),
              ("dst_block_index", ctypes.c_int64), ("dst_offset_bytes", ctypes.c_int64),
              ("size_bytes", ctypes.c_int64), ("src_stride_bytes", ctypes.c_int64),
              ("dst_stride_bytes", ctypes.c_int64), ("count", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class SpanDeclC(ctypes.Structure):
  _fields_ = [("src_unit", ctypes.c_int64), ("tag", ctypes.c_char_p),
              ("block_ids", c_i64_p), ("n_block_ids", ctypes.c_int64),
              ("spans", ctypes.POINTER(ByteSpanC)), ("n_spans", ctypes.c_int64),
              ("declared_bytes", ctypes.c_int64), ("dst_space_version", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class PoolReshardRequestC(ctypes.Structure):
  _fields_ = [("n_src_units", ctypes.c_int64),
              ("src_pools", ctypes.POINTER(ctypes.POINTER(PoolSpecC))),
              ("n_src_pools", c_i64_p), ("dst_pools", ctypes.POINTER(PoolSpecC)),
              ("n_dst_pools", ctypes.c_int64), ("transfer_ranks", c_i32_p),
              ("transfer_parallelism", c_i32_p), ("parallelism", ctypes.c_int32),
              ("pad_", ctypes.c_int32), ("tags", ctypes.POINTER(ctypes.c_char_p)),
              ("n_tags", ctypes.c_int64), ("dst_block_ids", c_i64_p),
              ("n_dst_block_ids", ctypes.c_int64), ("dst_block_counts", c_i64_p),
              ("n_dst_block_counts", ctypes.c_int64), ("dst_skip_bytes", c_i64_p),
              ("n_dst_skip_bytes", ctypes.c_int64), ("decls", ctypes.POINTER(SpanDeclC)),
              ("n_decls", ctypes.c_int64), ("unit_names", ctypes.POINTER(ctypes.c_char_p))]


class ScheduleEntryC(ctypes.Structure):
  _fields_ = [("src_block_id", ctypes.c_int64), ("dst_block_id", ctypes.c_int64),
              ("src_offset_bytes", ctypes.c_int64), ("dst_offset_bytes", ctypes.c_int64),
              ("size_bytes", ctypes.c_int64), ("pool_group", ctypes.c_int32),
              ("pad_", ctypes.c_int32)]


class ReceivedEntryC(ctypes.Structure):
  _fields_ = [("source_rank", ctypes.c_int32), ("dst_peer", ctypes.c_int32),
              ("dst_shard_idx", ctypes.c_int64), ("src_block_id", ctypes.c_int64),
              ("dst_block_id", ctypes.c_int64), ("src_offset_bytes", ctypes.c_int64),
              ("dst_offset_bytes", ctypes.c_int64), ("size_bytes", ctypes.c_int64),
              ("src_stride_bytes", ctypes.c_int64), ("dst_stride_bytes", ctypes.c_int64),
              ("count", ctypes.c_int32), ("pool_group", ctypes.c_int32)]


class ReceivedGroupC(ctypes.Structure):
  _fields_ = [("pool_indices", c_i32_p), ("n_pool_indices", ctypes.c_int64),
              ("dst_block_ids", c_i64_p), ("n_dst_block_ids", ctypes.c_int64),
              ("extents", c_i64_p), ("n_extents", ctypes.c_int64),
              ("expected_pushes", ctypes.c_int32), ("order_rank", ctypes.c_int32)]


class ReceivedPlanC(ctypes.Structure):
  _fields_ = [("transfer_pool_indices", c_i32_p), ("n_transfer_pools", ctypes.c_int64),
              ("pool_dtype_tags", ctypes.POINTER(ctypes.c_char_p)),
              ("n_pool_dtype_tags", ctypes.c_int64), ("groups", ctypes.POINTER(ReceivedGroupC)),
              ("n_groups", ctypes.c_int64), ("entries", ctypes.POINTER(ReceivedEntryC)),
              ("n_entries", ctypes.c_int64), ("n_schedules", ctypes.c_int64),
              ("parallelism", ctypes.c_int32), ("pad_", ctypes.c_int32)]


# name -> (restype, argtypes); every symbol declared in include/tpusync_b200.h
_V = ctypes.c_void_p
_SIGS = {
    "ts_last_error": (ctypes.c_char_p, []),
    "ts_version": (ctypes.c_char_p, []),
    "ts_validate_copy_spec": (ctypes.c_int, [c_i64_p, ctypes.c_int64, c_i64_p,
                                             ctypes.c_int64, c_i64_p, ctypes.c_int64]),
    "ts_coalesce_runs": (ctypes.c_int, [c_i64_p, c_i64_p, c_i64_p, ctypes.c_int64,
                                        c_i64_p, c_i64_p, c_i64_p, c_i64_p]),
    "ts_region_validate": (ctypes.c_int, [ctypes.POINTER(RegionSpecC), ctypes.c_int64]),
    "ts_pool_validate": (ctypes.c_int, [ctypes.POINTER(PoolSpecC), ctypes.c_int64]),
    "ts_pool_geometry": (ctypes.c_int, [ctypes.POINTER(PoolSpecC), c_i64_p, c_i64_p, c_i64_p]),
    "ts_regions_cover_range": (ctypes.c_int, [ctypes.POINTER(RegionSpecC), ctypes.c_int64,
                                              ctypes.c_uint64, ctypes.c_uint64,
                                              ctypes.POINTER(ctypes.c_int)]),
    "ts_pool_copy_extents": (ctypes.c_int, [ctypes.POINTER(PoolSpecC), c_i64_p, ctypes.c_int64,
                                            ctypes.POINTER(PoolExtent), ctypes.c_int64, c_i64_p]),
    "ts_pool_live_segments": (ctypes.c_int, [ctypes.POINTER(PoolSpecC),
                                             ctypes.POINTER(LiveSegmentC), ctypes.c_int64,
                                             c_i64_p]),
    "ts_pool_physical_to_logical": (ctypes.c_int, [ctypes.POINTER(LiveSegmentC), ctypes.c_int64,
                                                   ctypes.c_int64, ctypes.c_int64, c_i64_p,
                                                   c_i64_p]),
    "ts_pool_translate_live_copy": (ctypes.c_int, [ctypes.POINTER(LiveSegmentC), ctypes.c_int64,
                                                   ctypes.POINTER(LiveSegmentC), ctypes.c_int64,
                                                   ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                   ctypes.POINTER(LiveCopyChunkC),
                                                   ctypes.c_int64, c_i64_p]),
    "ts_pool_reshard_plan_build": (ctypes.c_int, [ctypes.POINTER(PoolReshardRequestC),
                                                  ctypes.POINTER(_V)]),
    "ts_pool_reshard_plan_destroy": (None, [_V]),
    "ts_pool_reshard_plan_info": (ctypes.c_int, [_V, c_i64_p]),
    "ts_pool_reshard_plan_entries": (ctypes.c_int, [_V, ctypes.c_int64,
                                                    ctypes.POINTER(ScheduleEntryC),
                                                    ctypes.c_int64, c_i64_p]),
    "ts_pool_reshard_plan_units": (ctypes.c_int, [_V, c_i64_p, c_i32_p]),
    "ts_pool_reshard_plan_group": (ctypes.c_int, [_V, ctypes.c_int64, c_i64_p, c_i32_p, c_i64_p,
                                                  c_i64_p]),
    "ts_pool_reshard_validate": (ctypes.c_int, [ctypes.POINTER(ReceivedPlanC),
                                                ctypes.POINTER(PoolSpecC), ctypes.c_int64,
                                                ctypes.c_int64, c_i64_p, ctypes.c_int64,
                                                ctypes.c_int]),
    "ts_pool_reshard_plan_from_received": (ctypes.c_int, [ctypes.POINTER(ReceivedPlanC),
                                                          ctypes.POINTER(PoolSpecC),
                                                          ctypes.POINTER(PoolSpecC),
                                                          ctypes.c_int64, c_i64_p, ctypes.c_int64,
                                                          c_i64_p, ctypes.c_int64, ctypes.c_int64,
                                                          ctypes.POINTER(_V)]),
    "ts_pool_reshard_program_create": (ctypes.c_int, [_V, ctypes.c_int64, ctypes.c_int, c_u64_p,
                                                      c_u64_p, c_u64_p, c_u64_p, ctypes.c_int64,
                                                      ctypes.POINTER(_V)]),
    "ts_pool_reshard_program_info": (ctypes.c_int, [_V, c_i64_p, c_u64_p]),
    "ts_pool_reshard_program_launch": (ctypes.c_int, [_V, _V, ctypes.c_int]),
    "ts_pool_reshard_program_destroy": (None, [_V]),
    "ts_kv_extract": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int, _V,
                                     ctypes.c_int64, _V, ctypes.c_uint64, _V, _V]),
    "ts_kv_insert": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int, _V,
                                    ctypes.c_int64, _V, ctypes.c_uint64, _V, _V]),
    "ts_kv_extract_fp8": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int, _V,
                                         ctypes.c_int64, _V, ctypes.c_uint64,
                                         ctypes.c_uint64, _V, _V]),
    "ts_kv_insert_fp8": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int, _V,
                                        ctypes.c_int64, _V, ctypes.c_uint64,
                                        ctypes.c_uint64, _V, _V]),
    "ts_kv_offload_noalloc": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int, c_i64_p,
                                             c_i64_p, ctypes.c_int64, _V, ctypes.c_uint64,
                                             ctypes.c_int64, _V]),
    "ts_reshard_work_items": (ctypes.c_int, [ctypes.POINTER(ReshardChunk),
                                             ctypes.c_int64, ctypes.c_int,
                                             ctypes.c_int, c_i64_p]),
    "ts_reshard_copy": (ctypes.c_int, [ctypes.c_int, _V, _V, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int, ctypes.c_int, _V]),
    "ts_wsync_create": (ctypes.c_int, [ctypes.POINTER(WsyncBuffer), ctypes.c_int, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_V)]),
    "ts_wsync_register_plan": (ctypes.c_int, [_V, ctypes.POINTER(ShardPushEntry),
                                              ctypes.c_int64, ctypes.c_char_p,
                                              ctypes.POINTER(WsyncDest), ctypes.c_int64]),
    "ts_wsync_push": (ctypes.c_int, [_V, _V]),
    "ts_wsync_query": (ctypes.c_int, [_V]),
    "ts_wsync_wait": (ctypes.c_int, [_V, ctypes.c_int64]),
    "ts_wsync_stream_wait": (ctypes.c_int, [_V, _V]),
    "ts_wsync_info": (ctypes.c_int, [_V, c_i64_p, c_u64_p]),
    "ts_wsync_destroy": (None, [_V]),
    "ts_enable_peer_access": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "ts_ipc_open": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(_V)]),
    "ts_ipc_close": (ctypes.c_int, [ctypes.c_int, _V]),
    "ts_ipc_export": (ctypes.c_int, [_V, ctypes.c_char_p, c_u64_p]),
    "ts_kv_relayout": (ctypes.c_int, [ctypes.c_int, _V, _V, ctypes.c_int,
                                      PageGeometry, PageGeometry, _V, ctypes.c_int64,
                                      _V, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _V,
                                      _V]),
    "ts_host_tier_create": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_char_p,
                                           ctypes.c_char_p, ctypes.c_uint64,
                                           ctypes.c_int, ctypes.POINTER(_V),
                                           ctypes.POINTER(ctypes.c_int)]),
    "ts_host_tier_ptr": (_V, [_V]),
    "ts_host_tier_bytes": (ctypes.c_uint64, [_V]),
    "ts_host_tier_destroy": (ctypes.c_int, [_V, ctypes.c_int]),
    "ts_mgr_create": (ctypes.c_int, [ctypes.POINTER(StorageDesc), ctypes.c_int,
                                     ctypes.c_int, ctypes.POINTER(ManagerOpts),
                                     ctypes.POINTER(_V)]),
    "ts_mgr_destroy": (ctypes.c_int, [_V]),
    "ts_d2h": (ctypes.c_int, [_V, c_i64_p, c_i64_p, c_i64_p, ctypes.c_int64,
                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_int64, _V, ctypes.POINTER(_V)]),
    "ts_h2d": (ctypes.c_int, [_V, c_i64_p, c_i64_p, c_i64_p, ctypes.c_int64,
                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                              ctypes.c_int64, _V, ctypes.POINTER(_V)]),
    "ts_mgr_host_block_ptr": (ctypes.c_int, [_V, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int64, c_u64_p, c_u64_p]),
    "ts_mgr_info": (ctypes.c_int, [_V, c_i64_p, c_u64_p, c_i64_p, c_u64_p]),
    "ts_mgr_register_pools": (ctypes.c_int, [_V, ctypes.POINTER(PoolSpecC), ctypes.c_int64]),
    "ts_mgr_num_pools": (ctypes.c_int, [_V, c_i64_p, ctypes.POINTER(ctypes.c_int)]),
    "ts_mgr_pool_geometry": (ctypes.c_int, [_V, ctypes.c_int64, c_i64_p, c_i64_p, c_i64_p]),
    "ts_d2h_pool_blocks": (ctypes.c_int, [_V, ctypes.c_int64, c_i64_p, ctypes.c_int64,
                                          ctypes.c_int64, _V, ctypes.POINTER(_V)]),
    "ts_h2d_pool_blocks": (ctypes.c_int, [_V, ctypes.c_int64, c_i64_p, ctypes.c_int64,
                                          ctypes.c_int64, _V, ctypes.POINTER(_V)]),
    "ts_mgr_pool_block_ref": (ctypes.c_int, [_V, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             c_u64_p]),
    "ts_mgr_set_profiling": (ctypes.c_int, [_V, ctypes.c_int]),
    "ts_mgr_kernel_stats": (ctypes.c_int, [_V, ctypes.c_int, c_i64_p,
                                           ctypes.POINTER(ctypes.c_double), c_u64_p]),
    "ts_store_create": (ctypes.c_int, [_V, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(_V)]),
    "ts_store_destroy": (ctypes.c_int, [_V]),
    "ts_store_lookup": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64, ctypes.c_int,
                                       ctypes.POINTER(BlockInfo), c_i64_p]),
    "ts_store_insert": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64,
                                       ctypes.POINTER(BlockInfo), ctypes.c_int64, ctypes.c_int]),
    "ts_store_release": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64]),
    "ts_store_pin_count": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_int64,
                                          ctypes.POINTER(ctypes.c_int)]),
    "ts_store_save": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64, _V]),
    "ts_store_load": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64, c_i32_p,
                                     ctypes.c_int64, _V]),
    "ts_store_poll": (ctypes.c_int, [_V, ctypes.c_int, c_i64_p, ctypes.c_char_p, ctypes.c_int64,
                                     c_i64_p, ctypes.c_int64, c_i64_p, c_i64_p]),
    "ts_store_stats": (ctypes.c_int, [_V, c_i64_p]),
    "ts_store_lru_order": (ctypes.c_int, [_V, ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                          c_i64_p, ctypes.c_int64, c_i64_p, c_i64_p]),
    "ts_store_allocate_host_blocks": (ctypes.c_int, [_V, ctypes.c_int, ctypes.c_int, c_i32_p]),
    "ts_store_host_block_op": (ctypes.c_int, [_V, ctypes.c_int, c_i32_p, ctypes.c_int64]),
    "ts_store_lru_op": (ctypes.c_int, [_V, ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                       ctypes.POINTER(BlockInfo), ctypes.POINTER(BlockInfo),
                                       c_i64_p, ctypes.c_char_p, ctypes.c_int64, c_i64_p]),
    "ts_mgr_num_storages": (ctypes.c_int, [_V, ctypes.POINTER(ctypes.c_int)]),
    "ts_mgr_storage": (ctypes.c_int, [_V, ctypes.c_int, ctypes.POINTER(ctypes.c_int), c_u64_p,
                                      c_u64_p, c_i64_p, c_u64_p]),
    "ts_xfer_endpoint_create": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_int64, ctypes.POINTER(_V)]),
    "ts_xfer_endpoint_destroy": (ctypes.c_int, [_V]),
    "ts_xfer_endpoint_name": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_int64]),
    "ts_xfer_read_state": (ctypes.c_int, [_V, ctypes.c_uint64, ctypes.POINTER(ctypes.c_int)]),
    "ts_xfer_register_read": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_uint64, c_i64_p,
                                             ctypes.c_int64, _V, ctypes.POINTER(ctypes.c_int)]),
    "ts_xfer_poll_sends": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_int64, c_i64_p,
                                          ctypes.c_int64, c_i64_p, c_i64_p]),
    "ts_xfer_reader_create": (ctypes.c_int, [_V, ctypes.c_int64, ctypes.POINTER(_V)]),
    "ts_xfer_reader_destroy": (ctypes.c_int, [_V]),
    "ts_xfer_start_read": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_char_p,
                                          c_i64_p, c_i64_p, ctypes.c_int64, _V]),
    "ts_xfer_poll_reads": (ctypes.c_int, [_V, ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                          c_i64_p, ctypes.c_int64, c_i64_p, c_i64_p]),
    "ts_xfer_reader_pending": (ctypes.c_int, [_V, c_i64_p]),
    "ts_reshard_ce_create": (ctypes.c_int, [ctypes.c_int, _V, ctypes.c_int64, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, ctypes.POINTER(_V)]),
    "ts_reshard_ce_launch": (ctypes.c_int, [_V, _V]),
    "ts_reshard_ce_info": (ctypes.c_int, [_V, c_i64_p, c_u64_p, c_i64_p]),
    "ts_reshard_ce_destroy": (ctypes.c_int, [_V]),
    "ts_mgr_numa_node": (ctypes.c_int, [_V, ctypes.POINTER(ctypes.c_int),
                                        ctypes.POINTER(ctypes.c_int)]),
    "ts_pci_numa_node": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p,
                                        ctypes.POINTER(ctypes.c_int)]),
    "ts_wpull_src_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, _V, ctypes.c_int64,
                                           ctypes.c_int, ctypes.POINTER(_V)]),
    "ts_wpull_src_stage": (ctypes.c_int, [_V, _V, ctypes.c_int64]),
    "ts_wpull_src_wait": (ctypes.c_int, [_V, ctypes.c_int64]),
    "ts_wpull_src_info": (ctypes.c_int, [_V, c_i64_p, c_i64_p, c_u64_p, c_i64_p]),
    "ts_wpull_src_destroy": (ctypes.c_int, [_V]),
    "ts_wpull_dst_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(ctypes.c_char_p),
                                           ctypes.c_int, _V, ctypes.c_int64,
                                           ctypes.POINTER(_V)]),
    "ts_wpull_dst_pull": (ctypes.c_int, [_V, _V, ctypes.c_int64]),
    "ts_wpull_dst_info": (ctypes.c_int, [_V, c_i64_p, c_i64_p, c_u64_p]),
    "ts_wpull_dst_destroy": (ctypes.c_int, [_V]),
    "ts_kv_metadata_required_bytes": (ctypes.c_uint64, [ctypes.c_int]),
    "ts_kv_metadata_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p,
                                           ctypes.POINTER(_V), ctypes.POINTER(ctypes.c_int)]),
    "ts_kv_metadata_on_region": (ctypes.c_int, [_V, ctypes.c_uint64, ctypes.c_int,
                                                ctypes.c_char_p, ctypes.c_int,
                                                ctypes.POINTER(_V)]),
    "ts_kv_metadata_set": (ctypes.c_int, [_V, ctypes.c_int, ctypes.c_char_p, ctypes.c_int64,
                                          ctypes.c_uint64]),
    "ts_kv_metadata_clear": (ctypes.c_int, [_V, ctypes.c_int]),
    "ts_kv_metadata_entries": (ctypes.c_int, [_V, c_i32_p, c_u64_p, ctypes.c_char_p,
                                              ctypes.c_int64, c_i64_p, ctypes.c_int64, c_i64_p,
                                              c_i64_p]),
    "ts_kv_metadata_reformat": (ctypes.c_int, [_V]),
    "ts_kv_metadata_info": (ctypes.c_int, [_V, ctypes.POINTER(ctypes.c_int),
                                           ctypes.POINTER(ctypes.c_int)]),
    "ts_kv_metadata_close": (ctypes.c_int, [_V, ctypes.c_int]),
    "ts_store_attach_metadata": (ctypes.c_int, [_V, _V]),
    "ts_store_recover": (ctypes.c_int, [_V, c_i64_p]),
    "ts_store_evict": (ctypes.c_int, [_V, ctypes.c_char_p, c_i64_p, ctypes.c_int64, c_i64_p]),
    "ts_event_query": (ctypes.c_int, [_V]),
    "ts_event_wait": (ctypes.c_int, [_V, ctypes.c_int64]),
    "ts_event_error": (ctypes.c_int, [_V, ctypes.c_char_p, ctypes.c_size_t]),
    "ts_event_stream_wait": (ctypes.c_int, [_V, _V]),
    "ts_event_elapsed_ms": (ctypes.c_int, [_V, ctypes.POINTER(ctypes.c_float)]),
    "ts_event_release": (None, [_V]),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
  """A ts_status error from the native library."""

  def __init__(self, code: int, message: str):
    super().__init__(message)
    self.code = code
    self.status = STATUS_NAMES.get(code, str(code))


def lib() -> ctypes.CDLL:
  """Returns the loaded library (loads it on first use; raises if missing)."""
  global _lib
  if _lib is not None:
    return _lib
  with _lock:
    if _lib is None:
      if not LIB_PATH.exists():
        raise ImportError(
            f"tpu_sync_b200 native library not built: {LIB_PATH} is missing. "
            "Run `python -m tpu_sync_b200.build` (nvcc required).")
      l = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | ctypes.RTLD_LOCAL)
      for name, (res, args) in _SIGS.items():
        fn = getattr(l, name)
        fn.restype = res
        fn.argtypes = args
      _lib = l
  return _lib


def last_error() -> str:
  msg = lib().ts_last_error()
  return msg.decode(errors="replace") if msg else ""


def check(rc: int, prefix: str = "") -> None:
  if rc != OK:
    msg = last_error()
    raise NativeError(rc, f"{prefix}{msg}" if prefix else msg)


def i64_array(values) -> np.ndarray:
  return np.ascontiguousarray(np.asarray(values, dtype=np.int64).reshape(-1))


def i64_ptr(arr: np.ndarray):
  return arr.ctypes.data_as(c_i64_p) if arr.size else None


def declared_symbols() -> list[str]:
  return sorted(_SIGS)

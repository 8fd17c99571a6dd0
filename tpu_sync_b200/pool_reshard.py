"""Pool reshard: plan and execute the prefill -> decode KV hand-off.

Planning restates BuildPoolReshardPlan's data part
(tpu_sync/kv_cache/reshard/pool_reshard_planner.cc:132-859) in the native
library: source units declare byte spans over their pool blocks
(``PoolSpanRegistration`` / ``PoolByteSpan``,
tpu_sync/kv_cache/reshard/declaration_types.h:17-58); the planner splits
request-global spans at destination pages, checks exactly-once coverage of
every destination block and emits (src block, dst block, src offset, dst
offset, size) entries per source unit, one group per transfer tag.

Execution replaces the reference's D2H -> TCP push -> receiver H2D with one
kernel per source GPU (``PoolReshardProgram``) that stores straight into the
destination GPU's pool storages over NVLink (peer pointers within a process,
CUDA IPC mappings across processes -- see weight_synchronizer.PeerBuffer).
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import Any, Dict, List, Optional, Sequence, Tuple

from tpu_sync_b200 import _native
from tpu_sync_b200.pool_layout import PoolSpec, coerce_pool_spec, _pool_c


@dataclasses.dataclass(frozen=True)
class PoolByteSpan:
  src_block_ordinal: int
  src_offset_bytes: int
  dst_block_index: int
  dst_offset_bytes: int
  size_bytes: int
  src_stride_bytes: int = 0
  dst_stride_bytes: int = 0
  count: int = 1


@dataclasses.dataclass
class PoolSpanRegistration:
  tag: str
  block_ids: Sequence[int]
  spans: Sequence[PoolByteSpan]
  declared_bytes: Optional[int] = None  # default: sum of size x count
  dst_space_version: int = 0

  def declared(self) -> int:
    if self.declared_bytes is not None:
      return int(self.declared_bytes)
    return sum(s.size_bytes * max(s.count, 1) for s in self.spans)


@dataclasses.dataclass(frozen=True)
class ScheduleEntry:
  src_block_id: int
  dst_block_id: int
  src_offset_bytes: int
  dst_offset_bytes: int
  size_bytes: int
  pool_group: int


@dataclasses.dataclass(frozen=True)
class PlanPoolGroup:
  pool_indices: Tuple[int, ...]
  dst_device_block_ids: Tuple[int, ...]
  expected_pushes: int
  dst_expected_extent_bytes: Tuple[int, ...]
  order_rank: int


class PoolReshardPlan:
  """A built plan: per-source-unit schedules and per-tag pool groups."""

  def __init__(self, handle, n_units: int, keep):
    self._h = handle
    self._keep = keep  # pool specs referenced by programs (geometry lives natively)
    info = (ctypes.c_int64 * 8)()
    _native.check(_native.lib().ts_pool_reshard_plan_info(self._h, info))
    n_groups, n_active, self.expected_block_count, self.parallelism = info[0], info[1], info[2], info[3]
    self.expected_pushes_per_pool = info[4]
    n_pools = info[5]
    units = (ctypes.c_int64 * max(n_active, 1))()
    pools = (ctypes.c_int32 * max(n_pools, 1))()
    _native.check(_native.lib().ts_pool_reshard_plan_units(self._h, units, pools))
    self.src_units = [units[i] for i in range(n_active)]
    self.transfer_pool_indices = [pools[i] for i in range(n_pools)]
    self.schedules: Dict[int, List[ScheduleEntry]] = {}
    for u in range(n_units):
      n = ctypes.c_int64()
      _native.lib().ts_pool_reshard_plan_entries(self._h, u, None, 0, ctypes.byref(n))
      out = (_native.ScheduleEntryC * max(n.value, 1))()
      _native.check(_native.lib().ts_pool_reshard_plan_entries(self._h, u, out, n.value,
                                                               ctypes.byref(n)))
      if n.value:
        self.schedules[u] = [ScheduleEntry(e.src_block_id, e.dst_block_id, e.src_offset_bytes,
                                           e.dst_offset_bytes, e.size_bytes, e.pool_group)
                             for e in out[:n.value]]
    self.pool_groups: List[PlanPoolGroup] = []
    for g in range(n_groups):
      sizes = (ctypes.c_int64 * 4)()
      _native.check(_native.lib().ts_pool_reshard_plan_group(self._h, g, sizes, None, None, None))
      pi = (ctypes.c_int32 * max(sizes[0], 1))()
      ids = (ctypes.c_int64 * max(sizes[1], 1))()
      ext = (ctypes.c_int64 * max(sizes[1], 1))()
      _native.check(_native.lib().ts_pool_reshard_plan_group(self._h, g, sizes, pi, ids, ext))
      self.pool_groups.append(PlanPoolGroup(tuple(pi[:sizes[0]]), tuple(ids[:sizes[1]]),
                                            sizes[2], tuple(ext[:sizes[1]]), sizes[3]))
    self.dst_expected_extent_bytes = [x for g in self.pool_groups
                                      for x in g.dst_expected_extent_bytes]

  def close(self) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_pool_reshard_plan_destroy(self._h)
      self._h = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass


def build_pool_reshard_plan(
    src_pools: Sequence[Sequence[Any]],
    dst_pools: Sequence[Any],
    transfer_pool_tags: Sequence[str],
    dst_device_block_ids: Sequence[int],
    declarations: Sequence[Tuple[int, PoolSpanRegistration]],
    *,
    dst_block_counts: Optional[Sequence[int]] = None,
    dst_skip_bytes: Optional[Sequence[int]] = None,
    parallelism: Optional[int] = None,
    transfer_ranks: Optional[Sequence[int]] = None,
    transfer_parallelism: Optional[Sequence[int]] = None,
    unit_names: Optional[Sequence[str]] = None,
) -> PoolReshardPlan:
  """Plans a hand-off from len(src_pools) source units to one destination.

  src_pools[u]: source unit u's pool manifest; dst_pools: the destination's.
  declarations: (source unit index, PoolSpanRegistration) pairs.
  transfer_parallelism / transfer_ranks: each unit's registration (default:
  the number of units / the unit's index).
  Raises ValueError with the reference's messages: the checks its unit and
  span registration make (work_unit_directory.cc:66-86,
  request_block_registry.cc:142-245), then the planner's.
  """
  nu = len(src_pools)
  src = [[coerce_pool_spec(p) for p in unit] for unit in src_pools]
  dst = [coerce_pool_spec(p) for p in dst_pools]
  keep: List[Any] = []
  src_arrays = []
  for unit in src:
    cs = [_pool_c(p) for p in unit]
    keep.append(cs)
    arr = (_native.PoolSpecC * max(len(cs), 1))(*[c[0] for c in cs])
    src_arrays.append(arr)
  src_ptrs = (ctypes.POINTER(_native.PoolSpecC) * max(nu, 1))(
      *[ctypes.cast(a, ctypes.POINTER(_native.PoolSpecC)) for a in src_arrays])
  n_src = (ctypes.c_int64 * max(nu, 1))(*[len(u) for u in src])
  dcs = [_pool_c(p) for p in dst]
  keep.append(dcs)
  dst_arr = (_native.PoolSpecC * max(len(dcs), 1))(*[c[0] for c in dcs])
  i32 = lambda v: (ctypes.c_int32 * max(len(v), 1))(*[int(x) for x in v]) if v is not None else None
  i64 = lambda v: (ctypes.c_int64 * max(len(v), 1))(*[int(x) for x in v])
  tag_bytes = [t.encode() for t in transfer_pool_tags]
  tags = (ctypes.c_char_p * max(len(tag_bytes), 1))(*tag_bytes)
  decl_arr = (_native.SpanDeclC * max(len(declarations), 1))()
  for i, (u, reg) in enumerate(declarations):
    spans = (_native.ByteSpanC * max(len(reg.spans), 1))(*[
        _native.ByteSpanC(s.src_block_ordinal, s.src_offset_bytes, s.dst_block_index,
                          s.dst_offset_bytes, s.size_bytes, s.src_stride_bytes,
                          s.dst_stride_bytes, s.count, 0) for s in reg.spans])
    ids = i64(reg.block_ids)
    tb = reg.tag.encode()
    keep.append((spans, ids, tb))
    decl_arr[i] = _native.SpanDeclC(int(u), tb, ids, len(reg.block_ids), spans, len(reg.spans),
                                    reg.declared(), int(reg.dst_space_version), 0)
  names = None
  if unit_names is not None:
    nb = [n.encode() for n in unit_names]
    keep.append(nb)
    names = (ctypes.c_char_p * max(nu, 1))(*nb)
  counts = list(dst_block_counts or [])
  skips = list(dst_skip_bytes or [])
  dst_ids = list(dst_device_block_ids)
  req = _native.PoolReshardRequestC(
      nu, src_ptrs, n_src, dst_arr, len(dst), i32(transfer_ranks), i32(transfer_parallelism),
      int(parallelism or 0), 0, tags, len(tag_bytes), i64(dst_ids), len(dst_ids),
      i64(counts), len(counts), i64(skips), len(skips), decl_arr, len(declarations), names)
  h = ctypes.c_void_p()
  rc = _native.lib().ts_pool_reshard_plan_build(ctypes.byref(req), ctypes.byref(h))
  if rc != _native.OK:
    raise ValueError(_native.last_error())
  return PoolReshardPlan(h, nu, keep)


# -- plans that arrive from a controller ---------------------------------------
#
# A received plan is a dict with the data fields of StartTransferRequest
# (tpu_sync/rpc/raiden_service.proto): "transfer_pool_indices",
# "pool_dtype_tags", "parallelism", "pool_groups" (dicts with pool_indices,
# dst_device_block_ids, dst_expected_extent_bytes, expected_pushes,
# order_rank) and "shard_push_schedules" ({source rank: [entry dicts with the
# ShardPushEntryProto fields dst_peer, dst_shard_idx, src_block_id,
# dst_block_id, src_offset_bytes, dst_offset_bytes, size_bytes,
# src_stride_bytes, dst_stride_bytes, count, pool_group]}).

def _received_c(plan: Dict[str, Any]):
  keep: List[Any] = []
  i32 = lambda v: (ctypes.c_int32 * max(len(v), 1))(*[int(x) for x in v])
  i64 = lambda v: (ctypes.c_int64 * max(len(v), 1))(*[int(x) for x in v])
  tpi = list(plan.get("transfer_pool_indices", []))
  tags = [str(t).encode() for t in plan.get("pool_dtype_tags", [])]
  tag_arr = (ctypes.c_char_p * max(len(tags), 1))(*tags)
  groups = plan.get("pool_groups", [])
  garr = (_native.ReceivedGroupC * max(len(groups), 1))()
  for i, g in enumerate(groups):
    pi, ids, ext = (i32(g.get("pool_indices", [])), i64(g.get("dst_device_block_ids", [])),
                    i64(g.get("dst_expected_extent_bytes", [])))
    keep.append((pi, ids, ext))
    garr[i] = _native.ReceivedGroupC(pi, len(g.get("pool_indices", [])), ids,
                                     len(g.get("dst_device_block_ids", [])), ext,
                                     len(g.get("dst_expected_extent_bytes", [])),
                                     int(g.get("expected_pushes", 0)), int(g.get("order_rank", 0)))
  peers: Dict[str, int] = {}
  rows = []
  scheds = plan.get("shard_push_schedules", {})
  for rank, entries in scheds.items():
    for e in entries:
      peer = str(e.get("dst_peer", ""))
      pid = -1 if not peer else peers.setdefault(peer, len(peers))
      rows.append(_native.ReceivedEntryC(
          int(rank), pid, int(e.get("dst_shard_idx", 0)), int(e.get("src_block_id", 0)),
          int(e.get("dst_block_id", 0)), int(e.get("src_offset_bytes", 0)),
          int(e.get("dst_offset_bytes", 0)), int(e.get("size_bytes", 0)),
          int(e.get("src_stride_bytes", 0)), int(e.get("dst_stride_bytes", 0)),
          int(e.get("count", 1)), int(e.get("pool_group", 0))))
  earr = (_native.ReceivedEntryC * max(len(rows), 1))(*rows)
  tarr = i32(tpi)
  keep += [tag_arr, tags, garr, earr, tarr]
  c = _native.ReceivedPlanC(tarr, len(tpi), tag_arr, len(tags), garr, len(groups), earr,
                            len(rows), len(scheds), int(plan.get("parallelism", 0)), 0)
  return c, keep


def _pool_array(pools):
  specs = [coerce_pool_spec(p) for p in pools]
  cs = [_pool_c(p) for p in specs]
  arr = (_native.PoolSpecC * max(len(cs), 1))(*[c[0] for c in cs])
  return arr, cs


def validate_pool_reshard_plan(plan: Dict[str, Any], local_pools: Sequence[Any],
                               local_block_ids: Sequence[int], is_sender: bool,
                               num_shards: int = 1) -> None:
  """The executor's checks of a received plan; raises ValueError with the
  reference's messages (kv_cache_manager_with_transfer.cc:742-1150)."""
  c, keep = _received_c(plan)
  parr, pkeep = _pool_array(local_pools)
  ids = _native.i64_array(list(local_block_ids))
  rc = _native.lib().ts_pool_reshard_validate(ctypes.byref(c), parr, len(pkeep), int(num_shards),
                                              _native.i64_ptr(ids), ids.size, int(bool(is_sender)))
  del keep
  if rc != _native.OK:
    raise ValueError(_native.last_error())


def plan_from_received(plan: Dict[str, Any], src_pools: Sequence[Any], dst_pools: Sequence[Any],
                       src_block_ids: Sequence[int], dst_block_ids: Sequence[int],
                       dst_num_shards: int = 1) -> PoolReshardPlan:
  """An executable plan from a received one, checked on both ends first."""
  c, keep = _received_c(plan)
  sarr, skeep = _pool_array(src_pools)
  darr, dkeep = _pool_array(dst_pools)
  if len(skeep) != len(dkeep):
    raise ValueError("source and destination pool tables must have the same length")
  sids = _native.i64_array(list(src_block_ids))
  dids = _native.i64_array(list(dst_block_ids))
  h = ctypes.c_void_p()
  rc = _native.lib().ts_pool_reshard_plan_from_received(
      ctypes.byref(c), sarr, darr, len(skeep), _native.i64_ptr(sids), sids.size,
      _native.i64_ptr(dids), dids.size, int(dst_num_shards), ctypes.byref(h))
  if rc != _native.OK:
    raise ValueError(_native.last_error())
  info = (ctypes.c_int64 * 8)()
  _native.check(_native.lib().ts_pool_reshard_plan_info(h, info))
  return PoolReshardPlan(h, info[7], [keep, skeep, dkeep])


def _ptr(t) -> int:
  return int(t.data_ptr())


def _nbytes(t) -> int:
  """Bytes of a storage: a tensor, or a PeerBuffer (dtype and shape)."""
  import math
  import torch
  if isinstance(t, torch.Tensor):
    return t.numel() * t.element_size()
  return math.prod(t.shape) * torch.empty((), dtype=t.dtype).element_size()


class PoolReshardProgram:
  """One source unit's share of a plan, ready to launch on a GPU.

  src_storages / dst_storages are indexed by pool storage_index, each as the
  launching GPU reaches it: tensors on this or a peer GPU, or PeerBuffer
  mappings of another process's memory.  The program runs on the source
  unit's GPU by default (stores cross NVLink); with `device` set to the
  destination's GPU it pulls instead (loads cross NVLink).
  """

  def __init__(self, plan: PoolReshardPlan, src_unit: int, src_storages: Sequence[Any],
               dst_storages: Sequence[Any], device: Optional[int] = None):
    import torch
    if len(src_storages) != len(dst_storages):
      raise ValueError("src_storages and dst_storages must have the same length")
    dev = src_storages[0].device.index if device is None else int(device)
    for t in list(src_storages) + list(dst_storages):
      if isinstance(t, torch.Tensor) and t.device.index != dev:
        from tpu_sync_b200.weight_synchronizer import enable_peer_access
        enable_peer_access(dev, t.device.index)
    sp = (ctypes.c_uint64 * len(src_storages))(*[_ptr(t) for t in src_storages])
    dp = (ctypes.c_uint64 * len(dst_storages))(*[_ptr(t) for t in dst_storages])
    sb = (ctypes.c_uint64 * len(src_storages))(*[_nbytes(t) for t in src_storages])
    db = (ctypes.c_uint64 * len(dst_storages))(*[_nbytes(t) for t in dst_storages])
    h = ctypes.c_void_p()
    _native.check(_native.lib().ts_pool_reshard_program_create(
        plan._h, int(src_unit), dev, sp, dp, sb, db, len(src_storages), ctypes.byref(h)),
        "pool reshard program: ")
    self._h = h
    self.device = torch.device("cuda", dev)
    self._refs = (list(src_storages), list(dst_storages))
    n, b = ctypes.c_int64(), ctypes.c_uint64()
    _native.check(_native.lib().ts_pool_reshard_program_info(self._h, ctypes.byref(n),
                                                             ctypes.byref(b)))
    self.n_tasks, self.bytes = n.value, b.value

  def launch(self, stream=None, max_ctas: int = 0) -> None:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream(self.device)
    _native.check(_native.lib().ts_pool_reshard_program_launch(
        self._h, ctypes.c_void_p(s.cuda_stream), int(max_ctas)), "pool reshard launch: ")

  def close(self) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_pool_reshard_program_destroy(self._h)
      self._h = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass

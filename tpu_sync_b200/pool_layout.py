"""Storage / pool / region descriptors and their byte geometry.

Keeps the reference's Python surface (tpu_sync/api/torch/pool_layout.py:33-199):
``RegionSpec`` / ``PoolSpec`` frozen dataclasses with ``live_bytes``,
``extent_end_bytes``, ``storage_extent_end_bytes``, ``live_bytes_per_block``,
``validate``, ``to_dict``, ``to_native_tuple`` and the ``coerce_*`` helpers.
A *storage* is one wrapped allocation (constructor order gives
``storage_index``), a *pool* an array of equally strided blocks inside it,
*regions* the live bytes inside one block.  ``tag`` / ``dtype_tag`` are
opaque.

Validation and the geometry functions of tpu_sync/kv_cache/pool_layout.cc
(ComputePoolBlockCopyExtents, ExpandPoolLiveSegments,
PhysicalLiveRangeToLogical, TranslateLiveCopy, RegionsCoverRange) run in the
native library, so Python and the manager's copies share one implementation
and the C++ messages ("region key exceeds slot bytes: end=... slot=...").
"""

from __future__ import annotations

import ctypes
import dataclasses
from typing import List, Mapping, Optional, Sequence, Tuple

from tpu_sync_b200 import _native


class PoolLayoutError(ValueError):
  """A rejected pool geometry; ``code`` is the absl status code."""

  def __init__(self, code: int, message: str):
    super().__init__(message)
    self.code = code


def _raise(rc: int):
  raise PoolLayoutError(rc, _native.last_error())


@dataclasses.dataclass(frozen=True)
class RegionSpec:
  name: str
  offset_bytes: int
  stride_bytes: int
  unit_bytes: int
  num_units: int
  units_per_stride: int = 1

  @property
  def live_bytes(self) -> int:
    return self.unit_bytes * self.num_units * self.units_per_stride

  @property
  def extent_end_bytes(self) -> int:
    if self.num_units == 0:
      return self.offset_bytes
    return (self.offset_bytes + (self.num_units - 1) * self.stride_bytes +
            self.units_per_stride * self.unit_bytes)

  def validate(self, slot_bytes: int) -> None:
    c = _region_c(self)
    rc = _native.lib().ts_region_validate(ctypes.byref(c), int(slot_bytes))
    if rc != _native.OK:
      _raise(rc)

  def to_dict(self) -> dict:
    return dataclasses.asdict(self)

  def to_native_tuple(self) -> tuple:
    return (self.name, int(self.offset_bytes), int(self.stride_bytes), int(self.unit_bytes),
            int(self.num_units), int(self.units_per_stride))


@dataclasses.dataclass(frozen=True)
class PoolSpec:
  tag: str
  storage_index: int
  base_offset_bytes: int
  block_stride_bytes: int
  num_blocks: int
  regions: Tuple[RegionSpec, ...]
  dtype_tag: str = ""

  @property
  def storage_extent_end_bytes(self) -> int:
    """Absolute end of the last declared live byte in the storage."""
    block_live_end = max((r.extent_end_bytes for r in self.regions), default=0)
    return (self.base_offset_bytes + (self.num_blocks - 1) * self.block_stride_bytes +
            block_live_end)

  @property
  def live_bytes_per_block(self) -> int:
    return sum(r.live_bytes for r in self.regions)

  def validate(self, storage_bytes: Optional[int] = None) -> None:
    if self.storage_index < 0:
      raise PoolLayoutError(_native.INVALID_ARGUMENT, f"pool {self.tag} storage_index must be >= 0")
    keep = _pool_c(self)
    rc = _native.lib().ts_pool_validate(ctypes.byref(keep[0]),
                                        -1 if storage_bytes is None else int(storage_bytes))
    if rc != _native.OK:
      _raise(rc)

  def to_dict(self) -> dict:
    return {"tag": self.tag, "storage_index": self.storage_index,
            "base_offset_bytes": self.base_offset_bytes,
            "block_stride_bytes": self.block_stride_bytes, "num_blocks": self.num_blocks,
            "regions": [r.to_dict() for r in self.regions], "dtype_tag": self.dtype_tag}

  def to_native_tuple(self) -> tuple:
    return (self.tag, int(self.storage_index), int(self.base_offset_bytes),
            int(self.block_stride_bytes), int(self.num_blocks),
            [r.to_native_tuple() for r in self.regions], self.dtype_tag)


def coerce_region_spec(value) -> RegionSpec:
  if isinstance(value, RegionSpec):
    return value
  return RegionSpec(name=str(value["name"]), offset_bytes=int(value["offset_bytes"]),
                    stride_bytes=int(value["stride_bytes"]), unit_bytes=int(value["unit_bytes"]),
                    num_units=int(value["num_units"]),
                    units_per_stride=int(value.get("units_per_stride", 1)))


def coerce_pool_spec(value) -> PoolSpec:
  if isinstance(value, PoolSpec):
    return value
  regions = value["regions"]
  if not isinstance(regions, Sequence):
    raise TypeError("pool regions must be a sequence")
  return PoolSpec(tag=str(value["tag"]), storage_index=int(value["storage_index"]),
                  base_offset_bytes=int(value.get("base_offset_bytes", 0)),
                  block_stride_bytes=int(value["block_stride_bytes"]),
                  num_blocks=int(value["num_blocks"]),
                  regions=tuple(coerce_region_spec(r) for r in regions),
                  dtype_tag=str(value.get("dtype_tag", "")))


# -- native marshalling -------------------------------------------------------

def _region_c(r: RegionSpec) -> _native.RegionSpecC:
  return _native.RegionSpecC(r.name.encode(), int(r.offset_bytes), int(r.stride_bytes),
                             int(r.unit_bytes), int(r.num_units), int(r.units_per_stride))


def _pool_c(p: PoolSpec):
  """(PoolSpecC, region array) -- keep both alive while the native call runs."""
  arr = (_native.RegionSpecC * max(len(p.regions), 1))(*[_region_c(r) for r in p.regions])
  c = _native.PoolSpecC(p.tag.encode(), int(p.storage_index), int(p.base_offset_bytes),
                        int(p.block_stride_bytes), int(p.num_blocks), arr, len(p.regions),
                        p.dtype_tag.encode())
  return c, arr


def pools_c(pools: Sequence[PoolSpec]):
  """A ts_pool_spec array for ts_mgr_register_pools (plus what it points to)."""
  keep = [_pool_c(p) for p in pools]
  arr = (_native.PoolSpecC * max(len(keep), 1))(*[k[0] for k in keep])
  return arr, keep


def _grow(call, ctype):
  """Runs a native call under the capacity protocol; returns the results."""
  cap = 64
  while True:
    out = (ctype * cap)()
    n = ctypes.c_int64()
    rc = call(out, cap, ctypes.byref(n))
    if rc == _native.OK:
      return [out[i] for i in range(n.value)]
    if rc != _native.RESOURCE_EXHAUSTED:
      _raise(rc)
    cap = max(cap * 2, n.value)


# -- geometry (pool_layout.cc) -------------------------------------------------

def compute_pool_block_copy_extents(pool: PoolSpec, block_ids: Sequence[int]) -> List[Tuple[int, int]]:
  """[(offset_bytes, size_bytes)]: live extents of the blocks, sorted, merged."""
  keep = _pool_c(pool)
  ids = _native.i64_array(list(block_ids))
  res = _grow(lambda out, cap, n: _native.lib().ts_pool_copy_extents(
      ctypes.byref(keep[0]), _native.i64_ptr(ids), ids.size, out, cap, n), _native.PoolExtent)
  return [(e.offset_bytes, e.size_bytes) for e in res]


def expand_pool_live_segments(pool: PoolSpec) -> List[Tuple[int, int, int]]:
  """[(logical_offset, physical_offset, size)] of the pool's live runs."""
  keep = _pool_c(pool)
  res = _grow(lambda out, cap, n: _native.lib().ts_pool_live_segments(
      ctypes.byref(keep[0]), out, cap, n), _native.LiveSegmentC)
  return [(s.logical_offset, s.physical_offset, s.size) for s in res]


def _segs_c(segments):
  arr = (_native.LiveSegmentC * max(len(segments), 1))(
      *[_native.LiveSegmentC(int(a), int(b), int(c)) for a, b, c in segments])
  return arr


def physical_live_range_to_logical(segments, physical_offset: int, size: int) -> Tuple[int, int]:
  arr = _segs_c(segments)
  a, b = ctypes.c_int64(), ctypes.c_int64()
  rc = _native.lib().ts_pool_physical_to_logical(arr, len(segments), int(physical_offset),
                                                 int(size), ctypes.byref(a), ctypes.byref(b))
  if rc != _native.OK:
    _raise(rc)
  return a.value, b.value


def translate_live_copy(src_segments, dst_segments, src_offset: int, dst_offset: int,
                        size: int) -> List[Tuple[int, int, int]]:
  """[(src_physical, dst_physical, size)] chunks of one compact-live copy."""
  sa, da = _segs_c(src_segments), _segs_c(dst_segments)
  res = _grow(lambda out, cap, n: _native.lib().ts_pool_translate_live_copy(
      sa, len(src_segments), da, len(dst_segments), int(src_offset), int(dst_offset),
      int(size), out, cap, n), _native.LiveCopyChunkC)
  return [(c.src_physical, c.dst_physical, c.size) for c in res]


def regions_cover_range(regions: Sequence[RegionSpec], start: int, end: int) -> bool:
  arr = (_native.RegionSpecC * max(len(regions), 1))(*[_region_c(r) for r in regions])
  out = ctypes.c_int()
  _native.check(_native.lib().ts_regions_cover_range(arr, len(regions), int(start), int(end),
                                                     ctypes.byref(out)))
  return bool(out.value)

"""CPU oracle for pool byte geometry -- TEST INFRASTRUCTURE ONLY.

Only tests/ (and the fixture script under tests/golden/) import this module,
as the checker; the product (tpu_sync_b200) never calls it.

Pure-Python restatement of tpu_sync/kv_cache/pool_layout.cc:

* RegionSpec::Validate / extent_end_bytes        :89-185
* PoolSpec::Validate / storage_extent_end_bytes   :187-254
* RegionsCoverRange (+ RegionCoversOffset)        :65-87, :256-272
* ComputePoolBlockCopyExtents                     :274-374
* ExpandPoolLiveSegments                          :376-472
* PhysicalLiveRangeToLogical                      :474-493
* TranslateLiveCopy                               :554-602

and of the manager's pool copy (KVCacheManagerBase::CopyPoolBlocks,
tpu_sync/kv_cache/kv_cache_manager_base.cc:1789-1858) on the per-storage host
mirrors of oracle.kv_blocks.RefKVManager.

Parity pinning: the known answers of tpu_sync/kv_cache/pool_layout_test.cc
(:35-307) and, where the reference compiles here (oracle/build_ref.py),
random cases run through the reference's own pool_layout.cc are committed
in tests/golden/pool_layout.json; tests/test_cpu_pool.py checks this module
and the product against both.

Errors are (code, message) tuples with the reference's absl codes and texts.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

OK, INVALID_ARGUMENT, OUT_OF_RANGE = 0, 3, 11
INT64_MAX = (1 << 63) - 1
MAX_LIVE_SEGMENTS = 1 << 20


class PoolError(Exception):
  def __init__(self, code: int, message: str):
    super().__init__(message)
    self.code = code
    self.message = message


def _mul_overflows(a: int, b: int) -> bool:
  return a != 0 and b != 0 and a > INT64_MAX // b


def _checked_mul(a, b, what):
  if a < 0 or b < 0:
    raise PoolError(INVALID_ARGUMENT, f"{what} operands must be non-negative")
  if _mul_overflows(a, b):
    raise PoolError(INVALID_ARGUMENT, f"{what} overflows int64")
  return a * b


def _checked_add(a, b, what):
  if a < 0 or b < 0:
    raise PoolError(INVALID_ARGUMENT, f"{what} operands must be non-negative")
  if a > INT64_MAX - b:
    raise PoolError(INVALID_ARGUMENT, f"{what} overflows int64")
  return a + b


# A region is a dict with name, offset_bytes, stride_bytes, unit_bytes,
# num_units, units_per_stride; a pool a dict with tag, storage_index,
# base_offset_bytes, block_stride_bytes, num_blocks, regions, dtype_tag.

def region_extent_end(r) -> int:
  n, st, ub, ups, off = (r["num_units"], r["stride_bytes"], r["unit_bytes"],
                         r["units_per_stride"], r["offset_bytes"])
  if n == 0:
    return off
  if min(n, st, ub, ups, off) < 0:
    return INT64_MAX
  if _mul_overflows(n - 1, st) or _mul_overflows(ups, ub):
    return INT64_MAX
  strided, packed = (n - 1) * st, ups * ub
  if off > INT64_MAX - strided or off + strided > INT64_MAX - packed:
    return INT64_MAX
  return off + strided + packed


def validate_region(r, slot_bytes: int) -> None:
  name = r["name"]
  p = f"region {name}"
  if not name:
    raise PoolError(INVALID_ARGUMENT, "region name must be non-empty")
  if slot_bytes <= 0:
    raise PoolError(INVALID_ARGUMENT, "slot_bytes must be positive")
  for field in ("offset_bytes", "stride_bytes", "unit_bytes", "num_units"):
    if r[field] < 0:
      raise PoolError(INVALID_ARGUMENT, f"{p} {field} must be >= 0")
  if r["units_per_stride"] <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} units_per_stride must be positive")
  if r["num_units"] > 0 and r["unit_bytes"] <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} unit_bytes must be positive")
  if r["num_units"] > 1 and r["stride_bytes"] <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} stride_bytes must be positive")
  packed = _checked_mul(r["units_per_stride"], r["unit_bytes"], f"{p} packed unit bytes")
  if r["num_units"] > 0 and r["stride_bytes"] < packed:
    raise PoolError(INVALID_ARGUMENT, f"{p} stride_bytes is smaller than packed units")
  strided = _checked_mul(max(r["num_units"] - 1, 0), r["stride_bytes"], f"{p} stride extent")
  start = _checked_add(r["offset_bytes"], strided, f"{p} extent start")
  end = _checked_add(start, packed, f"{p} extent end")
  if end > slot_bytes:
    raise PoolError(INVALID_ARGUMENT, f"{p} exceeds slot bytes: end={end} slot={slot_bytes}")


def storage_extent_end(pool) -> int:
  base, stride, nb = pool["base_offset_bytes"], pool["block_stride_bytes"], pool["num_blocks"]
  if base < 0 or stride < 0 or nb <= 0 or _mul_overflows(nb - 1, stride):
    return INT64_MAX
  block_off = (nb - 1) * stride
  live = max([region_extent_end(r) for r in pool["regions"]] + [0])
  if base > INT64_MAX - block_off:
    return INT64_MAX
  last = base + block_off
  if live < 0 or last > INT64_MAX - live:
    return INT64_MAX
  return last + live


def validate_pool(pool, storage_bytes: int = -1) -> None:
  tag = pool["tag"]
  if not tag:
    raise PoolError(INVALID_ARGUMENT, "pool tag must be non-empty")
  p = f"pool {tag}"
  if pool["block_stride_bytes"] <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} block_stride_bytes must be positive")
  if pool["num_blocks"] <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} num_blocks must be positive")
  if pool["base_offset_bytes"] < 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} base_offset_bytes must be >= 0")
  if not pool["regions"]:
    raise PoolError(INVALID_ARGUMENT, f"{p} must contain at least one region")
  for r in pool["regions"]:
    try:
      validate_region(r, pool["block_stride_bytes"])
    except PoolError as e:
      raise PoolError(INVALID_ARGUMENT, f"{p}: {e.message}") from None
  if storage_bytes >= 0:
    end = storage_extent_end(pool)
    if end == INT64_MAX:
      raise PoolError(INVALID_ARGUMENT, f"{p} live storage extent overflows int64")
    if end > storage_bytes:
      raise PoolError(INVALID_ARGUMENT,
                      f"{p} exceeds storage bytes (live regions): end={end} storage={storage_bytes}")


def _region_covers(r, offset: int) -> Optional[int]:
  n = r["num_units"]
  if n <= 0:
    return None
  base, stride = r["offset_bytes"], r["stride_bytes"]
  packed = r["unit_bytes"] * r["units_per_stride"]
  if offset < base or packed == 0:
    return None
  unit = 0
  if n > 1:
    if stride == 0:
      return None
    unit = (offset - base) // stride
    if unit >= n:
      return None
  start = base + unit * stride
  end = start + packed
  return end if start <= offset < end else None


def regions_cover_range(regions, start: int, end: int) -> bool:
  cursor = start
  while cursor < end:
    nxt = cursor
    for r in regions:
      ce = _region_covers(r, cursor)
      if ce is not None:
        nxt = max(nxt, min(ce, end))
    if nxt == cursor:
      return False
    cursor = nxt
  return True


def copy_extents(pool, block_ids: Sequence[int]) -> List[Tuple[int, int]]:
  p = f"pool {pool['tag']}"
  ext = []
  for bid in block_ids:
    if bid < 0 or bid >= pool["num_blocks"]:
      raise PoolError(OUT_OF_RANGE, f"{p} block_id {bid} out of range [0, {pool['num_blocks']})")
    delta = _checked_mul(bid, pool["block_stride_bytes"], f"{p} block offset")
    base = _checked_add(pool["base_offset_bytes"], delta, f"{p} block base")
    for r in pool["regions"]:
      pr = f"{p} region {r['name']}"
      packed = _checked_mul(r["unit_bytes"], r["units_per_stride"], f"{pr} packed bytes")
      if r["num_units"] == 0 or packed == 0:
        continue
      if r["stride_bytes"] == packed:
        nbytes = _checked_mul(r["num_units"], packed, f"{pr} live bytes")
        ext.append((_checked_add(base, r["offset_bytes"], f"{pr} offset"), nbytes))
        continue
      for u in range(r["num_units"]):
        ud = _checked_mul(u, r["stride_bytes"], f"{pr} unit offset")
        rb = _checked_add(base, r["offset_bytes"], f"{pr} base")
        ext.append((_checked_add(rb, ud, f"{pr} unit address"), packed))
  ext.sort()
  merged: List[List[int]] = []
  for off, size in ext:
    end = _checked_add(off, size, f"{p} copy extent end")
    if not merged:
      merged.append([off, size])
      continue
    prev = merged[-1]
    prev_end = _checked_add(prev[0], prev[1], f"{p} previous copy extent end")
    if off > prev_end:
      merged.append([off, size])
      continue
    prev[1] = max(prev_end, end) - prev[0]
  return [(a, b) for a, b in merged]


def live_segments(pool) -> List[Tuple[int, int, int]]:
  p = f"pool {pool['tag']}"
  stride = pool["block_stride_bytes"]
  if stride <= 0:
    raise PoolError(INVALID_ARGUMENT, f"{p} has non-positive block stride")
  iv = []
  for r in pool["regions"]:
    if min(r["offset_bytes"], r["stride_bytes"], r["unit_bytes"], r["num_units"]) < 0:
      raise PoolError(INVALID_ARGUMENT, f"{p} has negative region geometry")
    if r["units_per_stride"] <= 0:
      raise PoolError(INVALID_ARGUMENT, f"{p} has non-positive units_per_stride")
    if _mul_overflows(r["unit_bytes"], r["units_per_stride"]):
      raise PoolError(INVALID_ARGUMENT, f"{p} region byte geometry overflows")
    packed = r["unit_bytes"] * r["units_per_stride"]
    n = r["num_units"]
    if n > 0 and packed <= 0:
      raise PoolError(INVALID_ARGUMENT, f"{p} has an empty live region")
    if n > 1 and r["stride_bytes"] <= 0:
      raise PoolError(INVALID_ARGUMENT, f"{p} has a non-positive region stride")
    if n > 0 and r["stride_bytes"] < packed:
      raise PoolError(INVALID_ARGUMENT, f"{p} has overlapping units within one region")
    if len(iv) + n > MAX_LIVE_SEGMENTS:
      raise PoolError(INVALID_ARGUMENT, f"{p} exceeds the live-region expansion bound")
    if n > 0 and r["stride_bytes"] == packed:
      if _mul_overflows(n, packed):
        raise PoolError(INVALID_ARGUMENT, f"{p} region byte geometry overflows")
      end = r["offset_bytes"] + n * packed
      if end > stride:
        raise PoolError(INVALID_ARGUMENT,
                        f"{p} live region exceeds its block stride: end={end}, stride={stride}")
      iv.append((r["offset_bytes"], end))
      continue
    for u in range(n):
      if _mul_overflows(u, r["stride_bytes"]):
        raise PoolError(INVALID_ARGUMENT, f"{p} region byte geometry overflows")
      s = r["offset_bytes"] + u * r["stride_bytes"]
      e = s + packed
      if e > stride:
        raise PoolError(INVALID_ARGUMENT,
                        f"{p} live region exceeds its block stride: end={e}, stride={stride}")
      iv.append((s, e))
  iv.sort()
  phys: List[List[int]] = []
  for s, e in iv:
    if phys and s < phys[-1][1]:
      raise PoolError(INVALID_ARGUMENT, f"{p} has overlapping live regions at byte {s}")
    if phys and s == phys[-1][1]:
      phys[-1][1] = e
    else:
      phys.append([s, e])
  out, logical = [], 0
  for s, e in phys:
    out.append((logical, s, e - s))
    logical += e - s
  return out


def physical_to_logical(segments, phys: int, size: int) -> Tuple[int, int]:
  if phys < 0 or size <= 0:
    raise PoolError(INVALID_ARGUMENT, "physical live range offset/size is invalid")
  pend = phys + size
  for lo, po, sz in segments:
    if po <= phys and pend <= po + sz:
      start = lo + phys - po
      return start, start + size
  raise PoolError(INVALID_ARGUMENT, f"physical range [{phys}, {pend}) crosses padding or lies "
                                    "outside declared live regions")


def translate_live_copy(src_segments, dst_segments, src_off: int, dst_off: int,
                        size: int) -> List[Tuple[int, int, int]]:
  if src_off < 0 or dst_off < 0 or size <= 0:
    raise PoolError(INVALID_ARGUMENT, "Compact-live copy offsets/size are invalid")

  def locate(segs, logical):
    for lo, po, sz in segs:
      if lo <= logical < lo + sz:
        return po + logical - lo, lo + sz - logical
    raise PoolError(INVALID_ARGUMENT, f"Compact-live offset {logical} is out of range")

  out = []
  left, sc, dc = size, src_off, dst_off
  while left > 0:
    sp, sa = locate(src_segments, sc)
    dp, da = locate(dst_segments, dc)
    take = min(left, sa, da)
    out.append((sp, dp, take))
    if len(out) > MAX_LIVE_SEGMENTS:
      raise PoolError(INVALID_ARGUMENT, "Compact-live copy exceeds the segment expansion bound")
    sc += take
    dc += take
    left -= take
  return out


def copy_pool_blocks(mgr, pool, block_ids, shard_idx=None, to_host=True):
  """CopyPoolBlocks on an oracle.kv_blocks.RefKVManager (per-storage mirrors).

  Returns (code, message); on OK the bytes of every extent are copied between
  mgr.device[storage][shard] and mgr.host[storage][shard] at equal offsets.
  """
  try:
    ext = copy_extents(pool, block_ids)
  except PoolError as e:
    return e.code, e.message
  l = pool["storage_index"]
  for s in range(mgr.num_shards):
    if shard_idx is not None and s != shard_idx:
      continue
    dev, host = mgr.device[l][s], mgr.host[l][s]
    for off, size in ext:
      if off + size > host.size:
        return OUT_OF_RANGE, "pool block copy exceeds host buffer size"
      if off + size > dev.size:
        return OUT_OF_RANGE, "pool block copy exceeds device buffer size"
    for off, size in ext:
      if to_host:
        host[off:off + size] = dev[off:off + size]
      else:
        dev[off:off + size] = host[off:off + size]
  return OK, ""

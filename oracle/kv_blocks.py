"""CPU oracle for KV block movement -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this module, and only as the checker or the timed CPU
baseline; the product (tpu_sync_b200) never calls it.

Restates, on host byte arrays, what the reference's host path does on its own
fake device (the XLA CPU PJRT client, where D2H/H2D are memcpys):

* ValidateOffsetsAndSizes      tpu_sync/kv_cache/kv_cache_manager_base.cc:72-102
* CoalesceMajorDimCopies       tpu_sync/kv_cache/kv_cache_manager_base.cc:121-141
* DispatchD2hWork (per storage, per run, bounds checks)
                               tpu_sync/kv_cache/kv_cache_manager_base.cc:2036-2124
* DispatchH2dWork              tpu_sync/kv_cache/kv_cache_manager_base.cc:1945-2033
* layer/shard range check      tpu_sync/kv_cache/kv_cache_manager_base.cc:540-545
* host mirror = host_blocks * bytes_per_block() per storage, zero-filled
                               tpu_sync/kv_cache/kv_cache_manager_base.cc:309-352
* bytes_per_block() = slice byte size of layer 0; layer block bytes =
  physical_size(l) / dim0(layer 0)
                               tpu_sync/kv_cache/kv_cache_manager_base.cc:1468,
                               tpu_sync/kv_cache/kv_cache_manager_base.h:434-439
* compact staging slot (request block k -> slot block k)
                               tpu_sync/core/kv_cache_manager_with_transfer.cc:326-355

Parity pinning: the reference's own tests that fix this behaviour are ported
as fixtures and cases in tests/ (validation messages from
tpu_sync/kv_cache/kv_cache_manager_test.cc:579-636, heterogeneous block sizes
from tpu_sync/frameworks/torch/kv_cache_manager_test.py:206-275, the
round-trip check of tpu_sync/benchmarks/perf_core.py:112-142).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

# absl status codes used by the reference
OK, INVALID_ARGUMENT, FAILED_PRECONDITION, OUT_OF_RANGE = 0, 3, 9, 11

SAME_LENGTH = "src_offsets, dst_offsets, and sizes must have the same length"
NON_NEGATIVE = "copy offsets and sizes must be non-negative"
LAYER_RANGE = "layer or shard index out of range"


def validate_offsets_and_sizes(src: Sequence[int], dst: Sequence[int],
                               sizes: Sequence[int]) -> Tuple[int, str]:
  """kv_cache_manager_base.cc:72-102 (empty dst / sizes = not given)."""
  if len(dst) and len(src) != len(dst):
    return INVALID_ARGUMENT, SAME_LENGTH
  if len(sizes) and len(src) != len(sizes):
    return INVALID_ARGUMENT, SAME_LENGTH
  for lst in (src, dst, sizes):
    for v in lst:
      if v < 0:
        return INVALID_ARGUMENT, NON_NEGATIVE
  return OK, ""


def coalesce_major_dim_copies(src, dst, sizes):
  """kv_cache_manager_base.cc:121-141: merge copies continuing the last run."""
  out_s, out_d, out_n = [], [], []
  for s, d, n in zip(src, dst, sizes):
    if out_s and s == out_s[-1] + out_n[-1] and d == out_d[-1] + out_n[-1]:
      out_n[-1] += n
    else:
      out_s.append(int(s))
      out_d.append(int(d))
      out_n.append(int(n))
  return out_s, out_d, out_n


@dataclass
class RefKVManager:
  """Byte-level model of KVCacheManagerBase over a [layer][shard] grid.

  device[l][s]: uint8 arrays (the storages); host[l][s]: uint8 arrays of
  host_blocks * bytes_per_block bytes (zero-filled, as posix_memalign+memset).
  """

  device: List[List[np.ndarray]]
  dim0: int
  host_blocks: int = 64
  host: List[List[np.ndarray]] = field(default_factory=list)

  def __post_init__(self):
    self.num_layers = len(self.device)
    self.num_shards = len(self.device[0])
    self.bytes_per_block = self.device[0][0].size // self.dim0
    self.host = [[np.zeros(self.host_blocks * self.bytes_per_block, np.uint8)
                  for _ in range(self.num_shards)] for _ in range(self.num_layers)]

  def layer_block_bytes(self, layer: int) -> int:
    # physical_size of the layer (shard 0's buffer) / major dim of layer 0
    return self.device[layer][0].size // self.dim0

  def _works(self, layer_idx, shard_idx):
    for l in range(self.num_layers):
      if layer_idx is not None and l != layer_idx:
        continue
      for s in range(self.num_shards):
        if shard_idx is not None and s != shard_idx:
          continue
        yield l, s

  def _prepare(self, src, dst, sizes, layer_idx, shard_idx):
    code, msg = validate_offsets_and_sizes(src, dst, sizes)
    if code != OK:
      return code, msg, None
    if (layer_idx is not None and layer_idx >= self.num_layers) or (
        shard_idx is not None and shard_idx >= self.num_shards):
      return OUT_OF_RANGE, LAYER_RANGE, None
    if len(src) and not len(sizes):
      sizes = [1] * len(src)
    return OK, "", coalesce_major_dim_copies(src, dst, sizes)

  def d2h(self, src, dst, sizes=None, layer_idx=None, shard_idx=None):
    """DispatchD2hWork: host[dst*bb, +n*bb) = device[src*bb, +n*bb)."""
    if sizes is None:
      sizes = [1] * len(src)
    code, msg, runs = self._prepare(list(src), list(dst), list(sizes), layer_idx,
                                    shard_idx)
    if code != OK:
      return code, msg
    cs, cd, cn = runs
    partial = len(cs) > 0
    copies = []
    for l, s in self._works(layer_idx, shard_idx):
      dev, host = self.device[l][s], self.host[l][s]
      bb = self.layer_block_bytes(l)
      phys = self.device[l][0].size
      if not partial:
        if phys > host.size:
          return OUT_OF_RANGE, "Copy range exceeds destination host buffer size"
        copies.append((host, 0, dev, 0, phys))
        continue
      for so_b, do_b, n_b in zip(cs, cd, cn):
        so, do, n = so_b * bb, do_b * bb, n_b * bb
        if so + n > dev.size:
          return INVALID_ARGUMENT, "Copy range exceeds source device buffer size"
        if do + n > host.size:
          return INVALID_ARGUMENT, "Copy range exceeds destination host buffer size"
        copies.append((host, do, dev, so, n))
    for dst_arr, do, src_arr, so, n in copies:
      dst_arr[do:do + n] = src_arr[so:so + n]
    return OK, ""

  def h2d(self, src, dst, sizes=None, layer_idx=None, shard_idx=None):
    """DispatchH2dWork: device[dst*bb, +n*bb) = host[src*bb, +n*bb)."""
    if sizes is None:
      sizes = [1] * len(src)
    code, msg, runs = self._prepare(list(src), list(dst), list(sizes), layer_idx,
                                    shard_idx)
    if code != OK:
      return code, msg
    cs, cd, cn = runs
    partial = len(cs) > 0
    copies = []
    for l, s in self._works(layer_idx, shard_idx):
      dev, host = self.device[l][s], self.host[l][s]
      bb = self.layer_block_bytes(l)
      phys = self.device[l][0].size
      if not partial:
        if phys > host.size:
          return INVALID_ARGUMENT, "Source host buffer is too small"
        copies.append((dev, 0, host, 0, phys))
        continue
      for so_b, do_b, n_b in zip(cs, cd, cn):
        so, do, n = so_b * bb, do_b * bb, n_b * bb
        if so + n > host.size:
          return INVALID_ARGUMENT, "Copy range exceeds source host buffer size"
        if do + n > dev.size:
          return INVALID_ARGUMENT, "Copy range exceeds destination device buffer size"
        copies.append((dev, do, host, so, n))
    for dst_arr, do, src_arr, so, n in copies:
      dst_arr[do:do + n] = src_arr[so:so + n]
    return OK, ""

  def host_block(self, layer: int, block_id: int, shard: int = 0) -> bytes:
    bb = self.layer_block_bytes(layer)
    return self.host[layer][shard][block_id * bb:(block_id + 1) * bb].tobytes()


def extract_to_staging(storages: Sequence[np.ndarray], ids: Sequence[int]) -> np.ndarray:
  """Compact staging slot, block-major: staging[k] = [storage s block ids[k]]_s.

  Each storage is a uint8 array [num_blocks, block_bytes]; the slot layout is
  block k of the request -> slot block k (kv_cache_manager_with_transfer.cc:326-355)
  with the storages of one block side by side ([blocks, layers, K/V, ...]).
  """
  ids = np.asarray(ids, dtype=np.int64)
  parts = [np.asarray(st).reshape(st.shape[0], -1)[ids] for st in storages]
  return np.concatenate(parts, axis=1) if parts else np.zeros((len(ids), 0), np.uint8)


def insert_from_staging(storages: Sequence[np.ndarray], ids: Sequence[int],
                        staging: np.ndarray) -> None:
  """Inverse of extract_to_staging (in place on the storages)."""
  off = 0
  for st in storages:
    flat = st.reshape(st.shape[0], -1)
    bb = flat.shape[1]
    flat[np.asarray(ids, dtype=np.int64)] = staging[:, off:off + bb]
    off += bb


def staging_layout(block_bytes: Sequence[int], fp8: bool = False):
  """Slot offsets / pitch of the 16-byte aligned block-major staging."""
  offs, off = [], 0
  for bb in block_bytes:
    offs.append(off)
    slot = bb // 2 if fp8 else bb
    off += (slot + 15) // 16 * 16
  scale_off = off if fp8 else 0
  if fp8:
    off += (4 * len(block_bytes) + 15) // 16 * 16
  return offs, scale_off, (off + 15) // 16 * 16


def extract_to_padded_staging(storages, ids, offs=None, pitch=None) -> np.ndarray:
  """extract_to_staging with the kernel's 16-byte aligned slot layout, or
  with the given slot offsets and pitch; bytes no slot covers are zero."""
  bbs = [st.reshape(st.shape[0], -1).shape[1] for st in storages]
  if offs is None:
    offs, _, pitch = staging_layout(bbs)
  out = np.zeros((len(ids), pitch), np.uint8)
  ids = np.asarray(ids, dtype=np.int64)
  for st, off, bb in zip(storages, offs, bbs):
    out[:, off:off + bb] = st.reshape(st.shape[0], -1)[ids]
  return out

"""KVCacheStore: tier-2 prefix cache over the pinned host tier.

Mirrors the reference's Python surface (tpu_sync/api/torch/kv_cache_store.py:154-594):
``lookup(block_hashes, enable_global=False, pin_found=True)`` ->
``[(hash, RaidenBlockId)]``, ``insert(hashes, slices, on_host) -> bool``,
``release(hashes)``, ``save(hashes, dst_raiden_id=None) -> bool``,
``load(hashes, device_block_ids, slices=None) -> bool``,
``poll_save_status() -> (done, failed, pending, existing, unregistered)``,
``poll_load_status() -> (done, failed, pending)``, ``capacity()`` and the
pin contract (lookup -> load, insert -> save; a failed operation keeps its
pin).  Only the local paths exist: no global registry, no remote peers, so
``enable_global`` finds nothing more and a REMOTE ``dst_raiden_id`` /
``slices`` load is refused.

Save and Load move bytes through a KVCacheManager (HBM pages <-> host tier)
on the GPU; the index, the pins and the host block allocator are C++
(tpu_sync_b200/csrc/kv_store.cu).
"""

from __future__ import annotations

import ctypes
import enum
import logging
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

from tpu_sync_b200 import _native


class BlockStatus(enum.IntEnum):
  INIT = 0
  REMOTE = 1
  HBM = 2
  HOST = 3
  HOST_AND_HBM = 4


@dataclass(frozen=True)
class RaidenId:
  """RaidenId (tpu_sync/api/torch/kv_cache_store.py:38-86): a value type here
  (no native object behind it), so `impl`, the reference's handle to one,
  is accepted and ignored."""
  job_name: str = ""
  job_replica_id: str = ""
  data_name: str = ""
  data_replica_idx: int = 0
  impl: object = field(default=None, repr=False, compare=False)


@dataclass
class RaidenBlockId:
  """RaidenBlockId (tpu_sync/api/torch/kv_cache_store.py:89-151), with the
  reference's positional order (raiden_id, host_block_id, status,
  device_block_id) and its accessors of the owning RaidenId's fields."""
  raiden_id: Optional[RaidenId] = None  # None: an empty RaidenId, as in the reference
  host_block_id: int = -1
  status: BlockStatus = BlockStatus.INIT
  device_block_id: int = -1
  impl: object = field(default=None, repr=False, compare=False)

  def __post_init__(self):
    if self.raiden_id is None:
      self.raiden_id = RaidenId()

  @property
  def job_name(self) -> str:
    return self.raiden_id.job_name

  @property
  def job_replica_id(self) -> str:
    return self.raiden_id.job_replica_id

  @property
  def data_name(self) -> str:
    return self.raiden_id.data_name

  @property
  def data_replica_idx(self) -> int:
    return self.raiden_id.data_replica_idx


def _pack(hashes: Sequence[bytes]):
  hs = [bytes(h) for h in hashes]
  offs = np.zeros(len(hs) + 1, dtype=np.int64)
  if hs:
    offs[1:] = np.cumsum([len(h) for h in hs])
  return b"".join(hs), offs


class KVCacheStore:
  """Local tier-2 prefix cache (see the module docstring for the contract)."""

  def __init__(self, capacity: int, global_registry_address: str = "",
               raiden_id: Optional[RaidenId] = None, *, num_shards: int = 1,
               store_server_ip: str = "127.0.0.1", shard_size_bytes: int = 0,
               raiden_controller_port: int = 0, expected_worker_count: int = 0,
               kv_pool_group: str = "", manager=None, host_blocks: Optional[int] = None,
               metadata=None):
    if num_shards < 1:
      raise ValueError("num_shards must be >= 1")
    if global_registry_address:
      raise ValueError("the global registry is not supported (local store only)")
    self._raiden_id = raiden_id or RaidenId()
    self._mgr = manager
    if host_blocks is None:
      host_blocks = manager.host_blocks if manager is not None else capacity
    h = ctypes.c_void_p()
    _native.check(_native.lib().ts_store_create(
        manager._mgr if manager is not None else None, int(capacity), int(host_blocks),
        ctypes.byref(h)), "KVCacheStore: ")
    self._impl = h
    # KVCacheStoreWrapper (kv_cache_store_wrapper.cc:111-185): with
    # RAIDEN_SHM_KEY set, the table lives in /dev/shm beside the host tier's
    # data segment; a table that survived a crash (warm) rebuilds the LRU, and
    # a failed recovery falls back to a cold start over a reformatted table.
    self._meta_region = None
    self._metadata = None
    self.recovered_blocks = 0
    if metadata is None and num_shards > 0:
      from tpu_sync_b200 import kv_metadata
      key = kv_metadata.metadata_shm_key()
      if key:
        try:
          self._meta_region = kv_metadata.KVCacheMetadataShmRegion.attach_or_format(
              key, int(capacity), kv_metadata.model_uid_from_env())
          metadata = self._meta_region.metadata
        except (ValueError, RuntimeError) as e:
          logging.warning("KV metadata table unavailable, serving without crash "
                          "recovery: %s", e)
    if metadata is not None:
      self._metadata = metadata
      _native.check(_native.lib().ts_store_attach_metadata(self._impl, metadata._h),
                    "KVCacheStore: ")
    if self._meta_region is not None and self._meta_region.warm:
      try:
        self.recovered_blocks = self.recover_from_local_manifest()
        logging.info("Recovered %d blocks from the local KV metadata table",
                     self.recovered_blocks)
      except RuntimeError as e:
        logging.warning("KV metadata recovery failed, falling back to a cold start: %s", e)
        try:
          self._meta_region.reformat()
        except RuntimeError as e2:
          logging.warning("Failed to reformat the KV metadata table: %s", e2)

  @property
  def raiden_id(self) -> RaidenId:
    """The RaidenId of this store (tpu_sync/api/torch/kv_cache_store.py:260-263)."""
    return self._raiden_id

  def close(self) -> None:
    if getattr(self, "_impl", None):
      _native.lib().ts_store_destroy(self._impl)
      self._impl = None
    # the store is gone, so its own table can be unmapped; the segment stays
    # in /dev/shm for the next start
    if getattr(self, "_meta_region", None) is not None:
      self._meta_region.close()
      self._meta_region = None
    self._metadata = None

  def evict(self, block_hashes: List[bytes]) -> int:
    """KVCacheStore::Evict (kv_cache_store.cc:1553-1570): drop unpinned
    host-resident entries and free their host blocks; returns how many."""
    keys, offs = _pack(block_hashes)
    n = ctypes.c_int64()
    _native.check(_native.lib().ts_store_evict(self._impl, keys, _native.i64_ptr(offs),
                                               len(block_hashes), ctypes.byref(n)),
                  "KVCacheStore evict: ")
    return n.value

  def recover_from_local_manifest(self) -> int:
    """KVCacheStore::RecoverFromLocalManifest (kv_cache_store.cc:1541-1551):
    rebuild an empty store's index from the metadata table's newest entry per
    hash (HOST blocks at their recorded host block ids, LRU order by seq);
    returns the number of recovered blocks."""
    n = ctypes.c_int64()
    _native.check(_native.lib().ts_store_recover(self._impl, ctypes.byref(n)),
                  "RecoverFromLocalManifest: ")
    return n.value

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass

  # -- index ----------------------------------------------------------------
  def lookup(self, block_hashes: List[bytes], enable_global: bool = False,
             pin_found: bool = True) -> List[Tuple[bytes, RaidenBlockId]]:
    keys, offs = _pack(block_hashes)
    out = (_native.BlockInfo * max(len(block_hashes), 1))()
    n = ctypes.c_int64()
    _native.check(_native.lib().ts_store_lookup(self._impl, keys, _native.i64_ptr(offs),
                                                len(block_hashes), int(pin_found), out,
                                                ctypes.byref(n)), "KVCacheStore lookup: ")
    return [(bytes(block_hashes[i]),
             RaidenBlockId(raiden_id=self.raiden_id, host_block_id=out[i].host_block_id,
                           device_block_id=out[i].device_block_id,
                           status=BlockStatus(out[i].status))) for i in range(n.value)]

  def insert(self, block_hashes: List[bytes], slices: Sequence, on_host: bool = False) -> bool:
    infos = (_native.BlockInfo * max(len(slices), 1))()
    for i, s in enumerate(slices):
      if isinstance(s, RaidenId):
        s = RaidenBlockId(raiden_id=s)
      if s.status == BlockStatus.REMOTE:
        raise ValueError(f"Insert only takes LOCAL entries; slice {i} has status REMOTE")
      infos[i] = _native.BlockInfo(int(s.host_block_id), int(s.device_block_id), int(s.status), 0)
    keys, offs = _pack(block_hashes)
    rc = _native.lib().ts_store_insert(self._impl, keys, _native.i64_ptr(offs),
                                       len(block_hashes), infos, len(slices), int(on_host))
    if rc == _native.INVALID_ARGUMENT:
      raise ValueError(_native.last_error())
    return rc == _native.OK

  def release(self, block_hashes: List[bytes]) -> None:
    keys, offs = _pack(block_hashes)
    _native.check(_native.lib().ts_store_release(self._impl, keys, _native.i64_ptr(offs),
                                                 len(block_hashes)))

  def get_pin_count(self, block_hash: bytes) -> int:
    out = ctypes.c_int()
    _native.check(_native.lib().ts_store_pin_count(self._impl, bytes(block_hash),
                                                   len(block_hash), ctypes.byref(out)))
    return out.value

  def capacity(self) -> int:
    return self.stats()["capacity"]

  def stats(self) -> dict:
    a = np.zeros(6, dtype=np.int64)
    _native.check(_native.lib().ts_store_stats(self._impl, _native.i64_ptr(a)))
    return dict(zip(["capacity", "size", "available", "host_blocks", "host_free",
                     "host_locked"], (int(x) for x in a)))

  # -- transfers --------------------------------------------------------------
  def save(self, block_hashes: List[bytes], dst_raiden_id: Optional[RaidenId] = None,
           stream=None) -> bool:
    """HBM -> host tier for inserted (pinned, HBM) blocks; True if launched."""
    if dst_raiden_id is not None:
      raise ValueError("remote save is not supported (local store only)")
    keys, offs = _pack(block_hashes)
    rc = _native.lib().ts_store_save(self._impl, keys, _native.i64_ptr(offs), len(block_hashes),
                                     self._stream(stream))
    self.last_error = _native.last_error() if rc else ""
    return rc == _native.OK

  def load(self, block_hashes: List[bytes], device_block_ids: Sequence[int],
           slices: Optional[Sequence] = None, stream=None) -> bool:
    """Host tier -> HBM for looked-up (pinned, host) blocks; True if launched."""
    if slices is not None:
      raise ValueError("peer loads with slices are not supported (local store only)")
    keys, offs = _pack(block_hashes)
    ids = np.ascontiguousarray(np.asarray(device_block_ids, dtype=np.int32))
    rc = _native.lib().ts_store_load(self._impl, keys, _native.i64_ptr(offs), len(block_hashes),
                                     ids.ctypes.data_as(_native.c_i32_p), ids.size,
                                     self._stream(stream))
    self.last_error = _native.last_error() if rc else ""
    if rc == _native.INVALID_ARGUMENT and "size mismatch" in self.last_error:
      raise ValueError(self.last_error)
    return rc == _native.OK

  def read_remote(self, block_hashes: List[bytes], slices: Sequence,
                  device_block_ids: Sequence[int]) -> bool:
    """Reads REMOTE blocks from their owning peers (api/torch/kv_cache_store.py:536-581).

    The owning peer's controller is found through the global registry, which
    this local store does not have, so every read is refused (False, with
    `last_error`), as the reference's store refuses without a registry."""
    if len(slices) != len(block_hashes) or len(device_block_ids) != len(block_hashes):
      raise ValueError("block_hashes, slices and device_block_ids must have the same length")
    self.last_error = ("read_remote needs a global registry to reach the owning peer; "
                       "this store is local only")
    return False

  def poll_remote_read_status(self):
    """(done, failed, pending) of remote reads: none are ever issued."""
    return [], [], []

  @property
  def raiden_controller_address(self) -> str:
    """No controller endpoint: transfers are driven in-process."""
    return ""

  @property
  def store_server_address(self) -> str:
    """Not published to a registry ("" = undiscoverable)."""
    return ""

  def _stream(self, stream):
    if self._mgr is None:
      return None
    import torch
    s = stream if stream is not None else torch.cuda.current_stream(self._mgr.device)
    return ctypes.c_void_p(s.cuda_stream)

  def _poll(self, which: int, n_lists: int):
    counts = np.zeros(5, dtype=np.int64)
    need_b, need_k = ctypes.c_int64(), ctypes.c_int64()
    size_b, size_k = 1 << 16, 1024
    while True:
      buf = ctypes.create_string_buffer(size_b)
      offs = np.zeros(size_k + 1, dtype=np.int64)
      rc = _native.lib().ts_store_poll(self._impl, which, _native.i64_ptr(counts), buf, size_b,
                                       _native.i64_ptr(offs), size_k + 1, ctypes.byref(need_b),
                                       ctypes.byref(need_k))
      if rc == _native.OK:
        break
      if rc != _native.RESOURCE_EXHAUSTED:
        _native.check(rc)
      size_b, size_k = max(size_b, 2 * need_b.value), max(size_k, 2 * need_k.value)
    raw = buf.raw
    keys = [raw[offs[i]:offs[i + 1]] for i in range(int(need_k.value))]
    out, pos = [], 0
    for c in range(n_lists):
      out.append(keys[pos:pos + int(counts[c])])
      pos += int(counts[c])
    return tuple(out)

  def poll_save_status(self):
    """(done, failed, pending, existing, unregistered) hash lists."""
    return self._poll(0, 5)

  def poll_load_status(self):
    """(done, failed, pending) hash lists."""
    return self._poll(1, 3)

  # -- test hooks -------------------------------------------------------------
  def _order(self, which: int) -> List[bytes]:
    need_b, need_k = ctypes.c_int64(), ctypes.c_int64()
    size_b, size_k = 1 << 16, 1024
    while True:
      buf = ctypes.create_string_buffer(size_b)
      offs = np.zeros(size_k + 1, dtype=np.int64)
      rc = _native.lib().ts_store_lru_order(self._impl, which, buf, size_b,
                                            _native.i64_ptr(offs), size_k + 1,
                                            ctypes.byref(need_b), ctypes.byref(need_k))
      if rc == _native.OK:
        raw = buf.raw
        return [raw[offs[i]:offs[i + 1]] for i in range(int(need_k.value))]
      size_b, size_k = max(size_b, 2 * need_b.value), max(size_k, 2 * need_k.value)

  def active_order(self) -> List[bytes]:
    return self._order(0)

  def candidate_order(self) -> List[bytes]:
    return self._order(1)

  def evictable_order(self) -> List[bytes]:
    return self._order(2)

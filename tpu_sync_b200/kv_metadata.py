"""Crash-persistent KV block metadata (which host block holds which hash).

Mirrors KVCacheMetadata (tpu_sync/kv_cache/kv_cache_metadata.h:19-141) and
KVCacheMetadataShmRegion (tpu_sync/kv_cache/kv_cache_metadata_shm.h:19-86):
``KVCacheMetadata.format(region, num_blocks, model_uid)`` /
``KVCacheMetadata.attach(...)`` over caller memory (a numpy buffer here),
``set(block_id, hash, seq)``, ``clear(block_id)``, ``valid_entries()`` ->
``[Entry(block_id, hash, seq)]`` in block order, and
``KVCacheMetadataShmRegion.attach_or_format(shm_key, num_blocks, model_uid)``
with ``.metadata``, ``.warm`` and ``.reformat()``.  The bytes are the
reference's on-memory format (tpu_sync_b200/csrc/kv_metadata.cu), so a
table one side wrote attaches on the other.  Errors raise ValueError for
invalid arguments and RuntimeError for failed preconditions (a table that
does not validate), as absl statuses surface through the reference's
bindings.
"""

from __future__ import annotations

import ctypes
from typing import List, NamedTuple, Optional

import numpy as np

from tpu_sync_b200 import _native

HEADER_BYTES = 128
ENTRY_BYTES = 128
MAX_HASH_LENGTH = 112
MAX_MODEL_UID_LENGTH = 63


class Entry(NamedTuple):
  """KVCacheMetadata::Entry (kv_cache_metadata.h:118-123)."""
  block_id: int
  hash: bytes
  seq: int


def _raise(rc: int) -> None:
  if rc == _native.OK:
    return
  msg = _native.last_error()
  if rc == _native.INVALID_ARGUMENT:
    raise ValueError(msg)
  raise _native.NativeError(rc, msg)


def required_size_bytes(num_blocks: int) -> int:
  """KVCacheMetadata::RequiredSizeBytes (kv_cache_metadata.cc:55-57)."""
  return HEADER_BYTES + int(num_blocks) * ENTRY_BYTES


def aligned_region(num_blocks: int) -> np.ndarray:
  """A zeroed, 64-byte aligned uint8 buffer sized for a table (the test
  fixture's MetadataRegion)."""
  n = required_size_bytes(num_blocks)
  raw = np.zeros(n + 64, np.uint8)
  off = (-raw.ctypes.data) % 64
  return raw[off:off + n]


class KVCacheMetadata:
  """A table handle.  Over caller memory it keeps that buffer alive; over a
  /dev/shm segment it owns the mapping, so a store holding the table keeps
  it mapped even after the KVCacheMetadataShmRegion object is gone."""

  def __init__(self, handle, owner=None):
    self._h = handle
    self._owner = owner  # the caller buffer of a region table, else None

  @classmethod
  def _on_region(cls, region: np.ndarray, num_blocks: int, model_uid: str, attach: bool):
    if not isinstance(region, np.ndarray) or region.dtype != np.uint8 or \
        not region.flags["C_CONTIGUOUS"]:
      raise ValueError("region must be a C-contiguous uint8 numpy array")
    h = ctypes.c_void_p()
    _raise(_native.lib().ts_kv_metadata_on_region(
        ctypes.c_void_p(region.ctypes.data), region.nbytes, int(num_blocks),
        model_uid.encode(), int(attach), ctypes.byref(h)))
    return cls(h, owner=region)

  @classmethod
  def format(cls, region: np.ndarray, num_blocks: int, model_uid: str = "") -> "KVCacheMetadata":
    """KVCacheMetadata::Format: zero the table and write a fresh header."""
    return cls._on_region(region, num_blocks, model_uid, attach=False)

  @classmethod
  def attach(cls, region: np.ndarray, num_blocks: int, model_uid: str = "") -> "KVCacheMetadata":
    """KVCacheMetadata::Attach: validate an existing header."""
    return cls._on_region(region, num_blocks, model_uid, attach=True)

  @property
  def num_blocks(self) -> int:
    n = ctypes.c_int()
    _raise(_native.lib().ts_kv_metadata_info(self._h, ctypes.byref(n), None))
    return n.value

  def set(self, block_id: int, block_hash: bytes, seq: int) -> None:
    h = bytes(block_hash)
    _raise(_native.lib().ts_kv_metadata_set(self._h, int(block_id), h, len(h), int(seq)))

  def clear(self, block_id: int) -> None:
    _raise(_native.lib().ts_kv_metadata_clear(self._h, int(block_id)))

  def valid_entries(self) -> List[Entry]:
    n, need = ctypes.c_int64(), ctypes.c_int64()
    rc = _native.lib().ts_kv_metadata_entries(self._h, None, None, None, 0, None, 0,
                                              ctypes.byref(n), ctypes.byref(need))
    if rc != _native.RESOURCE_EXHAUSTED:  # the size query of a non-empty table
      _raise(rc)
    if n.value == 0:
      return []
    ids = np.zeros(n.value, np.int32)
    seqs = np.zeros(n.value, np.uint64)
    offs = np.zeros(n.value + 1, np.int64)
    buf = ctypes.create_string_buffer(max(need.value, 1))
    _raise(_native.lib().ts_kv_metadata_entries(
        self._h, ids.ctypes.data_as(_native.c_i32_p), seqs.ctypes.data_as(_native.c_u64_p),
        buf, need.value, offs.ctypes.data_as(_native.c_i64_p), n.value, ctypes.byref(n),
        ctypes.byref(need)))
    raw = buf.raw
    return [Entry(int(ids[i]), raw[offs[i]:offs[i + 1]], int(seqs[i])) for i in range(len(ids))]

  def _close(self, unlink: bool = False) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_kv_metadata_close(self._h, int(unlink))
      self._h = None

  def __del__(self):
    try:
      self._close()
    except Exception:
      pass


class KVCacheMetadataShmRegion:
  """A table in a /dev/shm segment that outlives the process (a crash)."""

  def __init__(self, meta: KVCacheMetadata, warm: bool, key: str):
    self._meta = meta
    self._warm = warm
    self.key = key

  @classmethod
  def attach_or_format(cls, shm_key: str, num_blocks: int,
                       model_uid: str = "") -> "KVCacheMetadataShmRegion":
    """AttachOrFormat (kv_cache_metadata_shm.cc:29-130): a surviving segment
    whose table validates is attached (warm), anything else is replaced by
    a freshly formatted one (cold)."""
    h = ctypes.c_void_p()
    warm = ctypes.c_int()
    _raise(_native.lib().ts_kv_metadata_open(shm_key.encode(), int(num_blocks),
                                             model_uid.encode(), ctypes.byref(h),
                                             ctypes.byref(warm)))
    key = shm_key if shm_key.startswith("/") else "/" + shm_key
    return cls(KVCacheMetadata(h), bool(warm.value), key)

  @property
  def metadata(self) -> KVCacheMetadata:
    return self._meta

  @property
  def warm(self) -> bool:
    return self._warm

  def reformat(self) -> None:
    """Reformat (kv_cache_metadata_shm.cc:148-160): erase every entry."""
    _raise(_native.lib().ts_kv_metadata_reformat(self._meta._h))
    self._warm = False

  def close(self, unlink: bool = False) -> None:
    """Unmap the segment now (no store may still use the table); it stays
    in /dev/shm unless ``unlink``.  Without an explicit close the mapping
    lives as long as the table object does."""
    self._meta._close(unlink)


def metadata_shm_key(environ=None) -> str:
  """MetadataShmKey (kv_cache_store_wrapper.cc:43-57): RAIDEN_SHM_KEY +
  "_metadata" [+ "_" + RAIDEN_SHM_SERVER_NAME], or "" when unset."""
  import os
  env = os.environ if environ is None else environ
  key = env.get("RAIDEN_SHM_KEY", "")
  if not key:
    return ""
  key += "_metadata"
  server = env.get("RAIDEN_SHM_SERVER_NAME", "")
  if server:
    key += "_" + server
  return key


def model_uid_from_env(environ=None) -> str:
  import os
  env = os.environ if environ is None else environ
  uid = env.get("RAIDEN_SHM_MODEL_UID")
  return "default_model" if uid is None else uid


__all__ = ["aligned_region", "Entry", "KVCacheMetadata", "KVCacheMetadataShmRegion",
           "required_size_bytes", "metadata_shm_key", "model_uid_from_env", "HEADER_BYTES", "ENTRY_BYTES",
           "MAX_HASH_LENGTH"]

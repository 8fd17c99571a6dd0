"""CPU restatement of KVCacheMetadata over a bytearray (test oracle).

Test infrastructure only: tests/ compare the product's table
(tpu_sync_b200/csrc/kv_metadata.cu through tpu_sync_b200/kv_metadata.py)
with this and with the fixtures of tests/golden/kv_metadata.json, which the
reference's own kv_cache_metadata.cc produced (oracle/_ref/meta_ref).

Follows tpu_sync/kv_cache/kv_cache_metadata.h:31-70 (layout) and
kv_cache_metadata.cc:34-186 (ValidateRegion, Format, Attach, Set, Clear,
ValidEntries).  Statuses are (code, message) with absl's numeric codes:
3 invalid argument, 9 failed precondition.  `addr_mod64` stands for the
region's address modulo 64 (the alignment check), None for a null region.
"""

from __future__ import annotations

import struct

MAGIC = 0x52414944454E4B4D
VERSION = 1
HEADER = 128
ENTRY = 128
UID_FIELD = 64
MAX_HASH = 112
OK = (0, "")


def required_size_bytes(num_blocks):
  return HEADER + num_blocks * ENTRY


def _validate(size, addr_mod64, num_blocks, uid):
  """ValidateRegion (kv_cache_metadata.cc:34-62)."""
  if num_blocks <= 0:
    return (3, f"num_blocks must be positive, got {num_blocks}")
  if len(uid) >= UID_FIELD:
    return (3, f"model_uid length {len(uid)} exceeds the maximum of {UID_FIELD - 1}")
  if addr_mod64 is None:
    return (3, "Metadata region is null")
  if addr_mod64 % 64:
    return (3, "Metadata region must be 64-byte aligned")
  need = required_size_bytes(num_blocks)
  if size < need:
    return (3, f"Metadata region too small: {size} bytes, need {need}")
  return OK


class Table:
  """A view of `buf[off:off+size]` holding a formatted / attached table."""

  def __init__(self, buf, off, num_blocks):
    self.buf, self.off, self.n = buf, off, num_blocks

  def _e(self, i):
    return self.off + HEADER + i * ENTRY

  def set(self, block_id, h: bytes, seq):
    """KVCacheMetadata::Set (kv_cache_metadata.cc:135-160)."""
    if block_id < 0 or block_id >= self.n:
      return (3, f"Block ID out of range: {block_id}")
    if not h:
      return (3, "Hash must not be empty")
    if len(h) > MAX_HASH:
      return (3, f"Hash length {len(h)} exceeds the maximum of {MAX_HASH}")
    e = self._e(block_id)
    self.buf[e + 10] = 0
    struct.pack_into("<QH", self.buf, e, seq, len(h))
    self.buf[e + 16:e + 16 + len(h)] = h
    self.buf[e + 10] = 1
    return OK

  def clear(self, block_id):
    """KVCacheMetadata::Clear (kv_cache_metadata.cc:162-169)."""
    if block_id < 0 or block_id >= self.n:
      return (3, f"Block ID out of range: {block_id}")
    self.buf[self._e(block_id) + 10] = 0
    return OK

  def valid_entries(self):
    """ValidEntries (kv_cache_metadata.cc:171-186): (block_id, hash, seq)."""
    out = []
    for i in range(self.n):
      e = self._e(i)
      if self.buf[e + 10] == 0:
        continue
      seq, hl = struct.unpack_from("<QH", self.buf, e)
      if hl == 0 or hl > MAX_HASH:
        continue
      out.append((i, bytes(self.buf[e + 16:e + 16 + hl]), seq))
    return out


def format_table(buf, off, size, addr_mod64, num_blocks, uid: bytes):
  """KVCacheMetadata::Format (kv_cache_metadata.cc:71-89) -> (status, Table)."""
  st = _validate(size, addr_mod64, num_blocks, uid)
  if st != OK:
    return st, None
  buf[off:off + required_size_bytes(num_blocks)] = bytes(required_size_bytes(num_blocks))
  struct.pack_into("<QIII", buf, off, MAGIC, VERSION, num_blocks, ENTRY)
  buf[off + 20:off + 20 + len(uid)] = uid
  return OK, Table(buf, off, num_blocks)


def attach_table(buf, off, size, addr_mod64, num_blocks, uid: bytes):
  """KVCacheMetadata::Attach (kv_cache_metadata.cc:91-129) -> (status, Table)."""
  st = _validate(size, addr_mod64, num_blocks, uid)
  if st != OK:
    return st, None
  magic, version, nb, esz = struct.unpack_from("<QIII", buf, off)
  if magic != MAGIC:
    return (9, "Metadata region magic mismatch"), None
  if version != VERSION:
    return (9, f"Metadata region version mismatch: {version} vs {VERSION}"), None
  if esz != ENTRY:
    return (9, f"Metadata entry size mismatch: {esz} vs {ENTRY}"), None
  if nb != num_blocks:
    return (9, f"Metadata num_blocks mismatch: {nb} vs {num_blocks}"), None
  raw = bytes(buf[off + 20:off + 20 + UID_FIELD])
  rec = raw.split(b"\0", 1)[0]
  if rec != uid:
    return (9, f'Metadata model_uid mismatch: "{rec.decode("latin-1")}" vs '
               f'"{uid.decode("latin-1")}"'), None
  return OK, Table(buf, off, num_blocks)

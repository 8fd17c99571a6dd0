"""CPU oracle of the host block allocator -- TEST INFRASTRUCTURE ONLY.

Restates LogicalBlockManager (tpu_sync/kv_cache/logical_block_manager.cc:32-224)
as written: Allocate scans every block, takes free ids in increasing order,
then evictable (allocated, unlocked) ids sorted by (last_access_counter, id);
one access-counter tick per Allocate / AllocateTarget / AccessBlock call.
Used to check the product allocator's order, which reaches the same result
from ordered sets instead of a full scan.  Pinned, with the product, to the
answers of the reference's own logical_block_manager.cc (compiled by
oracle/build_ref.py; tests/golden/block_manager.json).
"""

from __future__ import annotations

OK, INVALID_ARGUMENT, RESOURCE_EXHAUSTED, FAILED_PRECONDITION = 0, 3, 8, 9


class LogicalBlockManager:
  def __init__(self, n: int):
    self.total = n
    self.allocated = [False] * n
    self.locked = [False] * n
    self.counter = [0] * n
    self.access_counter = 0

  def allocate(self, k: int, lock: bool = False):
    if k <= 0:
      return INVALID_ARGUMENT, None
    if k > self.total:
      return INVALID_ARGUMENT, None
    free = [i for i in range(self.total) if not self.allocated[i]]
    evictable = [i for i in range(self.total) if self.allocated[i] and not self.locked[i]]
    if len(free) + len(evictable) < k:
      return RESOURCE_EXHAUSTED, None
    out = free[:k]
    need = k - len(out)
    if need > 0:
      evictable.sort(key=lambda i: (self.counter[i], i))
      out += evictable[:need]
    self.access_counter += 1
    for i in out:
      self.allocated[i] = True
      self.locked[i] = lock
      self.counter[i] = self.access_counter
    return OK, out

  def deallocate(self, ids):
    for i in ids:
      if i < 0 or i >= self.total or not self.allocated[i]:
        return INVALID_ARGUMENT
    for i in ids:
      self.allocated[i] = False
      self.locked[i] = False
    return OK

  def allocate_target(self, ids):
    seen = set()
    for i in ids:
      if i < 0 or i >= self.total:
        return INVALID_ARGUMENT
      if self.allocated[i]:
        return FAILED_PRECONDITION
      if i in seen:
        return INVALID_ARGUMENT
      seen.add(i)
    self.access_counter += 1
    for i in ids:
      self.allocated[i] = True
      self.locked[i] = True
      self.counter[i] = self.access_counter
    return OK

  def unlock(self, ids):
    for i in ids:
      if i < 0 or i >= self.total or not self.allocated[i]:
        return INVALID_ARGUMENT
    for i in ids:
      self.locked[i] = False
    return OK

  def access(self, i):
    if i < 0 or i >= self.total or not self.allocated[i]:
      return INVALID_ARGUMENT
    self.access_counter += 1
    self.counter[i] = self.access_counter
    return OK

  def num_free(self):
    return sum(1 for a in self.allocated if not a)

  def num_locked(self):
    return sum(1 for a in self.locked if a)

"""GPU test of the tier-2 store driving real transfers: insert -> save moves
HBM blocks to the host tier, lookup -> load moves them back into other device
blocks; bytes checked against the CPU copy, pins and statuses against the
reference's contract."""

import time

import numpy as np
import pytest
import torch

from tpu_sync_b200 import KVCacheManager, workloads
from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId

pytestmark = pytest.mark.gpu


def poll_until(fn, n, timeout=30.0):
  done, t0 = [], time.time()
  while len(done) < n and time.time() - t0 < timeout:
    res = fn()
    done += res[0]
    assert res[1] == []
  return done


def test_store_save_load_moves_blocks(cuda):
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=8, head_dim=128)
  pool = workloads.kv_pool(geom, 64, 7, cuda)
  before = [t.clone() for t in pool]
  mgr = KVCacheManager([[t] for t in pool], host_blocks_to_allocate=16)
  store = KVCacheStore(capacity=16, manager=mgr)
  hs = [f"blk{i}".encode() for i in range(6)]
  dev = [3, 9, 10, 11, 40, 63]
  assert store.insert(hs, [RaidenBlockId(device_block_id=d, status=BlockStatus.HBM) for d in dev])
  assert store.save(hs)
  assert sorted(poll_until(store.poll_save_status, 6)) == sorted(hs)
  found = store.lookup(hs)
  assert len(found) == 6 and all(b.status == BlockStatus.HOST_AND_HBM for _, b in found)
  for (h, b), d in zip(found, dev):
    for l in range(len(pool)):
      assert mgr.read_block_bytes(l, b.host_block_id) == \
          before[l][d].contiguous().view(torch.uint8).cpu().numpy().tobytes()
  targets = [0, 1, 2, 20, 21, 22]
  assert store.load(hs, targets)
  assert sorted(poll_until(store.poll_load_status, 6)) == sorted(hs)
  torch.cuda.synchronize()
  for d_src, d_dst in zip(dev, targets):
    for l in range(len(pool)):
      assert torch.equal(pool[l][d_dst], before[l][d_src])
  assert all(store.get_pin_count(h) == 0 for h in hs)
  store.close()
  mgr.close()

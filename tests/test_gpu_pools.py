"""GPU parity of pool copies (RegisterPools / D2hPoolBlocks / H2dPoolBlocks).

Every case runs the product through KVCacheManager (C ABI) and the oracle's
CopyPoolBlocks model (oracle/pool_layout.py on oracle.kv_blocks.RefKVManager's
per-storage host mirrors) on the same seeded bytes, then compares every byte
of every host mirror and device storage -- bit-exact.

Covered: implicit pools (whole blocks, strided DMAs); explicit pools with
sparse units (units_per_stride > 1), tight regions, 4-byte and 1-byte
aligned units, a pool whose block stride is 1.5 storage blocks so its
extents straddle host blocks of the block-major tier, shard-restricted
copies, ordering after a block-unit d2h, and the error paths.
"""

import random

import numpy as np
import pytest
import torch

from oracle import kv_blocks as ref
from oracle import pool_layout as opl
from tpu_sync_b200.kv_cache_manager import KVCacheManager
from tpu_sync_b200.pool_layout import PoolSpec, RegionSpec

pytestmark = pytest.mark.gpu

DIM0, HOST_BLOCKS = 24, 32


def gpu():
  if not torch.cuda.is_available():
    pytest.skip("needs a GPU")
  return torch.device("cuda", 0)


def make(bb, layers=3, shards=2, seed=0):
  dev = gpu()
  g = torch.Generator().manual_seed(seed)
  grid = [[torch.randint(0, 256, (DIM0, bb), generator=g, dtype=torch.uint8).to(dev)
           for _ in range(shards)] for _ in range(layers)]
  mgr = KVCacheManager(grid, host_blocks_to_allocate=HOST_BLOCKS)
  oracle = ref.RefKVManager([[t.cpu().numpy().reshape(-1).copy() for t in layer] for layer in grid],
                            dim0=DIM0, host_blocks=HOST_BLOCKS)
  return grid, mgr, oracle


def as_dict(p: PoolSpec):
  return p.to_dict()


def check_all(grid, mgr, oracle, bb):
  for l, layer in enumerate(grid):
    for s, t in enumerate(layer):
      np.testing.assert_array_equal(t.cpu().numpy().reshape(-1), oracle.device[l][s],
                                    err_msg=f"device storage {l}/{s}")
      got = np.frombuffer(mgr.read_storage_bytes(l, 0, HOST_BLOCKS * bb, s), np.uint8)
      np.testing.assert_array_equal(got, oracle.host[l][s], err_msg=f"host mirror {l}/{s}")


def run_both(mgr, oracle, pool_idx, pool_dict, ids, shard=None, to_host=True):
  fn = mgr.d2h_pool_blocks if to_host else mgr.h2d_pool_blocks
  fn(pool_idx, ids, shard).Await()
  torch.cuda.synchronize()
  code, msg = opl.copy_pool_blocks(oracle, pool_dict, ids, shard, to_host)
  assert code == 0, msg


def explicit_pools(bb):
  return [
      # sparse: 8 units of 2 x 64 B every 256 B, then a tight 1 KiB region
      PoolSpec("fa", 0, 0, bb, DIM0, (RegionSpec("k", 0, 256, 64, 8, 2),
                                       RegionSpec("v", bb // 2, 128, 128, 8, 1)), "bf16"),
      # block stride of 1.5 storage blocks: extents straddle host blocks;
      # 500-byte units (4-byte path) and one ragged 7-byte region (byte path)
      PoolSpec("ssm", 1, 512, bb * 3 // 2, 15, (RegionSpec("a", 0, 1000, 500, 4, 1),
                                                 RegionSpec("b", bb * 3 // 2 - 7, 7, 7, 1, 1))),
      # whole blocks: strided DMAs
      PoolSpec("whole", 2, 0, bb, DIM0, (RegionSpec("block", 0, bb, bb, 1, 1),)),
  ]


def test_implicit_pools_match_oracle():
  bb = 4096
  grid, mgr, oracle = make(bb, seed=1)
  assert mgr.num_pools() == 3 and not mgr.has_explicit_pools()
  spec = mgr.pool_spec(1)
  assert spec["tag"] == "opaque" and spec["block_stride_bytes"] == bb
  assert spec["num_blocks"] == HOST_BLOCKS  # host mirror bytes / block bytes
  ids = [5, 6, 7, 0, 23, 12]
  for p in range(3):
    run_both(mgr, oracle, p, spec | {"storage_index": p}, ids)
  check_all(grid, mgr, oracle, bb)
  for layer in grid:
    for t in layer:
      t.zero_()
  for l in range(3):
    for s in range(2):
      oracle.device[l][s][:] = 0
  for p in range(3):
    run_both(mgr, oracle, p, spec | {"storage_index": p}, [6, 0, 23], to_host=False)
  check_all(grid, mgr, oracle, bb)
  with pytest.raises(RuntimeError, match=r"pool opaque block_id 32 out of range \[0, 32\)"):
    mgr.d2h_pool_blocks(0, [32])
  # ids beyond the device storage (but inside the mirror) are rejected
  with pytest.raises(RuntimeError, match="pool block copy exceeds device buffer size"):
    mgr.d2h_pool_blocks(0, [24])
  with pytest.raises(RuntimeError, match="pool index 3 out of range: 3 pools"):
    mgr.h2d_pool_blocks(3, [0])
  mgr.close()


@pytest.mark.parametrize("bb", [4096, 3000])
def test_explicit_pools_partial_regions_match_oracle(bb):
  grid, mgr, oracle = make(bb, seed=2 + bb)
  pools = explicit_pools(bb)
  summary = mgr.register_pools(pools)
  assert summary == {"admitted": True, "pools": 3, "storages": 3,
                     "tags": {"fa": 1, "ssm": 1, "whole": 1}}
  assert mgr.has_explicit_pools() and mgr.num_pools() == 3
  assert mgr.pool_ids_with_tag("ssm") == [1]
  rng = random.Random(bb)
  for rnd in range(3):
    for i, p in enumerate(pools):
      ids = rng.sample(range(p.num_blocks), k=min(p.num_blocks, rng.randint(1, 9)))
      shard = None if rnd != 1 else rng.randrange(2)
      run_both(mgr, oracle, i, as_dict(p), ids, shard, to_host=True)
  check_all(grid, mgr, oracle, bb)
  # reload into fresh device contents
  g = torch.Generator().manual_seed(99)
  for l, layer in enumerate(grid):
    for s, t in enumerate(layer):
      t.copy_(torch.randint(0, 256, t.shape, generator=g, dtype=torch.uint8))
      oracle.device[l][s][:] = t.cpu().numpy().reshape(-1)
  for i, p in enumerate(pools):
    ids = rng.sample(range(p.num_blocks), k=min(p.num_blocks, 7))
    run_both(mgr, oracle, i, as_dict(p), ids, None, to_host=False)
  check_all(grid, mgr, oracle, bb)
  mgr.close()


def test_pool_copy_orders_after_block_transfer():
  bb = 4096
  grid, mgr, oracle = make(bb, seed=5)
  pools = explicit_pools(bb)
  mgr.register_pools(pools)
  # block-unit offload of storage blocks 3, 4 (every storage) into host 3, 4 ...
  f = mgr.d2h([3], [3], [2])
  oracle.d2h([3], [3], [2])
  # ... then immediately reload those host blocks through a pool (no host
  # sync).  Read before the offload lands, the host blocks would still be
  # zero and the reload would zero the device blocks.
  g = mgr.h2d_pool_blocks(2, [3, 4])
  opl.copy_pool_blocks(oracle, as_dict(pools[2]), [3, 4], None, False)
  f.Await()
  g.Await()
  torch.cuda.synchronize()
  check_all(grid, mgr, oracle, bb)
  mgr.close()


def test_pool_registration_and_block_ref_errors():
  bb = 4096
  grid, mgr, oracle = make(bb, seed=6)
  with pytest.raises(ValueError, match="pool table must be non-empty"):
    mgr.register_pools([])
  with pytest.raises(ValueError, match="invalid pool 0: pool x: region k exceeds slot bytes"):
    mgr.register_pools([PoolSpec("x", 0, 0, 128, 2, (RegionSpec("k", 0, 64, 64, 3),))])
  with pytest.raises(ValueError, match="storage_index 7 out of range: manager wraps 3 storages"):
    mgr.register_pools([PoolSpec("x", 7, 0, bb, 2, (RegionSpec("k", 0, bb, bb, 1),))])
  with pytest.raises(RuntimeError, match="register_pools failed: invalid pool 0: pool x exceeds "
                                         "storage bytes"):
    mgr.register_pools([PoolSpec("x", 0, 0, bb, DIM0 + 1, (RegionSpec("k", 0, bb, bb, 1),))])
  assert not mgr.has_explicit_pools()
  pools = explicit_pools(bb)
  mgr.register_pools(pools)
  ref0 = mgr.get_block_ref(0, 5, 1)
  assert ref0["tag"] == "fa" and ref0["dtype_tag"] == "bf16" and ref0["block_id"] == 5
  # pointer = host block 5 of storage (0, shard 1): write through it, read back
  import ctypes
  ctypes.memmove(ref0["ptr"], b"\x5a" * 16, 16)
  assert mgr.read_block_bytes(0, 5, 1)[:16] == b"\x5a" * 16
  with pytest.raises(RuntimeError, match="spans several host blocks"):
    mgr.get_block_ref(1, 1)
  with pytest.raises(RuntimeError, match=r"block_id 24 out of range for pool 0 \(fa\)"):
    mgr.get_block_ref(0, 24)
  with pytest.raises(RuntimeError, match="block_id must be non-negative"):
    mgr.get_block_ref(0, -1)
  with pytest.raises(RuntimeError, match="shard index out of range"):
    mgr.d2h_pool_blocks(0, [1], 2)
  mgr.close()
  # a pool reaching past the host tier's mirror of its storage
  dev = gpu()
  big = [[torch.zeros((64, bb), dtype=torch.uint8, device=dev)]]
  m2 = KVCacheManager(big, host_blocks_to_allocate=8)
  with pytest.raises(RuntimeError, match="host tier mirrors 32768 bytes"):
    m2.register_pools([PoolSpec("x", 0, 0, bb, 9, (RegionSpec("k", 0, bb, bb, 1),))])
  m2.close()
  m3 = KVCacheManager([[torch.zeros((8, 1024), dtype=torch.bfloat16, device=dev)]],
                      host_blocks_to_allocate=8, fp8=True)
  with pytest.raises(RuntimeError, match="not supported on an fp8 host tier"):
    m3.register_pools([PoolSpec("x", 0, 0, 2048, 8, (RegionSpec("k", 0, 2048, 2048, 1),))])
  m3.close()

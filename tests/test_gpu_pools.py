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


# ---------------------------------------------------------------------------
# The reference's manager pool tests (tpu_sync/kv_cache/kv_cache_manager_test.cc
# :120-556), one counterpart per TEST, on device-backed managers.  The
# reference's TestKVCacheManager(num_layers, num_shards, slice_byte_size,
# host_blocks) holds storages of host_blocks x slice bytes; here those are
# device tensors of [host_blocks, slice] bytes (or [dim0, slice] where the
# reference sets a device physical size).  Host addresses: byte x of storage
# s lives at host block x // bb of that storage's slot, offset x % bb (the
# block-major tier); with one storage that is the reference's base + x.
# ---------------------------------------------------------------------------

import ctypes

from tpu_sync_b200 import _native


def ref_manager(num_layers, slice_bytes, host_blocks, dim0=None, num_shards=1):
  dev = gpu()
  dim0 = host_blocks if dim0 is None else dim0
  grid = [[torch.zeros((dim0, slice_bytes), dtype=torch.uint8, device=dev)
           for _ in range(num_shards)] for _ in range(num_layers)]
  return grid, KVCacheManager(grid, host_blocks_to_allocate=host_blocks)


def dense_pool(tag, storage_index, base, stride, num_blocks, dtype_tag="dtype_a"):
  """DensePool (kv_cache_manager_test.cc:89-115): one region covering the block."""
  return PoolSpec(tag, storage_index, base, stride, num_blocks,
                  (RegionSpec("block", 0, stride, stride, 1),), dtype_tag=dtype_tag)


def strided_pool(tag, storage_index, base, stride, num_blocks):
  """StridedPool (:68-87): live [0, 32) and [64, 96) of every block."""
  return PoolSpec(tag, storage_index, base, stride, num_blocks,
                  (RegionSpec("payload", 0, 64, 32, 2),), dtype_tag="dtype_a")


def host_addr(mgr, layer, x, shard=0):
  rc, ptr, _ = mgr._host_block(layer, x // mgr.block_bytes(layer), shard)
  assert rc == _native.OK
  return ptr + x % mgr.block_bytes(layer)


def block_ref_rc(mgr, pool_idx, shard_idx, block_id):
  ptr = ctypes.c_uint64()
  rc = _native.lib().ts_mgr_pool_block_ref(mgr._mgr, pool_idx, shard_idx, block_id,
                                           ctypes.byref(ptr))
  return rc, ptr.value


def host_bytes(mgr, layer, x, n):
  return np.frombuffer(mgr.read_storage_bytes(layer, x, n), np.uint8)


def test_register_pools_validates_against_storage():
  """RegisterPoolsValidatesAgainstStorage (:120-153)."""
  _, mgr = ref_manager(2, 128, 2)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 128, 2), strided_pool("kind_b", 0, 0, 128, 2),
                      dense_pool("kind_a", 1, 64, 64, 3)])  # overlapping pools are allowed
  assert mgr.has_explicit_pools() and mgr.num_pools() == 3
  with pytest.raises(ValueError, match="storage_index"):
    mgr.register_pools([dense_pool("kind_a", 5, 0, 128, 2)])
  with pytest.raises(RuntimeError, match="exceeds storage bytes"):  # 64 + 2 x 128 > 256
    mgr.register_pools([dense_pool("kind_a", 0, 64, 128, 2)])
  # the device's physical size, not the host mirror's, bounds a pool
  _, dev_backed = ref_manager(1, 128, 2, dim0=1)
  dev_backed.register_pools([dense_pool("kind_a", 0, 0, 128, 1)])
  with pytest.raises(RuntimeError, match="exceeds storage bytes"):
    dev_backed.register_pools([dense_pool("kind_a", 0, 0, 128, 2)])
  mgr.close()
  dev_backed.close()


def test_get_pool_block_ref_pointer_math():
  """GetPoolBlockRefPointerMath (:155-195), and the same pools on the second
  storage of a two-storage tier (addresses restated for the block-major
  layout)."""
  _, mgr = ref_manager(1, 128, 4)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 128, 2), dense_pool("kind_b", 0, 256, 64, 4)])
  base = host_addr(mgr, 0, 0)
  r = mgr.get_block_ref(0, 1)
  assert r["ptr"] == base + 128 and r["block_stride_bytes"] == 128
  assert r["tag"] == "kind_a" and r["pool_idx"] == 0 and r["block_id"] == 1
  assert mgr.get_block_ref(1, 0)["ptr"] == base + 256
  assert mgr.get_block_ref(1, 3)["ptr"] == base + 256 + 3 * 64
  for pool, shard, block in ((0, 0, 2), (1, 0, 4), (2, 0, 0), (0, 1, 0)):
    assert block_ref_rc(mgr, pool, shard, block)[0] == _native.OUT_OF_RANGE
  mgr.close()
  _, two = ref_manager(2, 128, 4)
  two.register_pools([dense_pool("kind_a", 1, 0, 128, 2), dense_pool("kind_b", 1, 256, 64, 4)])
  assert two.get_block_ref(0, 1)["ptr"] == host_addr(two, 1, 128)
  assert two.get_block_ref(1, 3)["ptr"] == host_addr(two, 1, 256 + 3 * 64)
  assert host_addr(two, 1, 128) - host_addr(two, 1, 0) == two.host_block_pitch
  two.close()


def test_register_pools_grows_device_backed_host_mirror():
  """RegisterPoolsGrowsDeviceBackedHostMirror (:197-225).  The tier here is
  one block-major allocation of host_blocks x the sum of the storages'
  block bytes, sized at creation: where it already mirrors the storage the
  pool is admitted and its last block sits at base + 3 x 64, as in the
  reference after it grew; a pool reaching past the bytes the tier mirrors
  is refused (FAILED_PRECONDITION) instead of regrowing the tier, and the
  bytes already there are kept."""
  _, mgr = ref_manager(1, 256, 1, dim0=1)
  mgr.write_block_bytes(0, 0, bytes(range(64)))
  mgr.register_pools([dense_pool("kind_a", 0, 0, 64, 4)])
  assert mgr.get_block_ref(0, 3)["ptr"] == host_addr(mgr, 0, 0) + 3 * 64
  assert mgr.read_block_bytes(0, 0)[:64] == bytes(range(64))
  mgr.close()
  _, short = ref_manager(1, 64, 1, dim0=4)  # 256 device bytes, the tier mirrors 64
  short.write_block_bytes(0, 0, bytes(range(64)))
  rc = _native.lib().ts_mgr_register_pools(short._mgr, *_pools_c([dense_pool("kind_a", 0, 0,
                                                                              64, 4)]))
  assert rc == _native.FAILED_PRECONDITION
  assert "tier mirrors 64 bytes of storage 0" in _native.last_error()
  assert short.read_block_bytes(0, 0) == bytes(range(64))
  short.close()


def _pools_c(pools):
  from tpu_sync_b200 import pool_layout
  arr, keep = pool_layout.pools_c(tuple(pools))
  _pools_c.keep = keep
  return arr, len(pools)


def test_register_pools_fails_after_active_plan_registered():
  """RegisterPoolsFailsAfterActivePlanRegistered (:227-243).  Active plans
  are the TCP push protocol's state, which this build does not have
  (register_active_plan names the on-node alternatives), so nothing
  freezes the pool table: a later registration replaces it."""
  _, mgr = ref_manager(1, 128, 1)
  with pytest.raises(NotImplementedError, match="PoolReshardProgram"):
    mgr.register_active_plan(445566, None, True)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 128, 1)])
  mgr.register_pools([dense_pool("kind_b", 0, 0, 64, 2)])
  assert mgr.num_pools() == 1 and mgr.pool_spec(0)["tag"] == "kind_b"
  mgr.close()


def test_pool_indices_with_tag():
  """PoolIndicesWithTag (:245-263)."""
  _, mgr = ref_manager(2, 128, 2)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 128, 2),
                      dense_pool("kind_b", 1, 0, 128, 2, dtype_tag="dtype_b"),
                      strided_pool("kind_a", 1, 0, 128, 2)])
  assert mgr.pool_ids_with_tag("kind_a") == [0, 2]
  assert mgr.pool_ids_with_tag("kind_b") == [1]
  assert mgr.pool_ids_with_tag("missing") == []
  mgr.close()


def test_register_active_plan_checks_pool_dtype_tags():
  """RegisterActivePlanChecksPoolDtypeTags (:265-297).  The dtype tags are
  kept per pool (pool_spec) for the on-node hand-off; the TCP plan
  registration that compares them against a request is not built."""
  _, mgr = ref_manager(2, 128, 2)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 128, 2),
                      dense_pool("kind_b", 1, 0, 128, 2, dtype_tag="dtype_b"),
                      strided_pool("kind_a", 1, 0, 128, 2)])
  assert [mgr.pool_spec(i)["dtype_tag"] for i in range(3)] == ["dtype_a", "dtype_b", "dtype_a"]
  with pytest.raises(NotImplementedError):
    mgr.register_active_plan(777, None, True)
  mgr.close()


def test_explicit_pool_addressing_uses_pool_base_and_stride():
  """ExplicitPoolAddressingUsesPoolBaseAndStride (:299-324): pool 0 on
  storage 1 at base 128, stride 64; block 2 lives at storage byte 256.  The
  reference's GetBlockChunks (TCP chunking) has no counterpart; the pool's
  blocks 0, 2, 3 move between device and host at those addresses and
  nothing else does."""
  grid, mgr = ref_manager(2, 128, 4)
  mgr.register_pools([dense_pool("kind_a", 1, 128, 64, 4)])
  assert mgr.get_block_ref(0, 2)["ptr"] == host_addr(mgr, 1, 128 + 2 * 64)
  pattern = torch.arange(512, dtype=torch.int32).remainder(251).to(torch.uint8)
  grid[1][0].view(-1).copy_(pattern.to(grid[1][0].device))
  mgr.d2h_pool_blocks(0, [0, 2, 3]).Await()
  want = np.zeros(512, np.uint8)
  p = pattern.numpy()
  for b in (0, 2, 3):
    want[128 + 64 * b:192 + 64 * b] = p[128 + 64 * b:192 + 64 * b]
  np.testing.assert_array_equal(host_bytes(mgr, 1, 0, 512), want)
  assert not host_bytes(mgr, 0, 0, 512).any()
  mgr.close()


def test_explicit_pool_transport_uses_backing_storage_base_and_pool_stride():
  """ExplicitPoolTransportUsesBackingStorageBaseAndPoolStride (:326-392):
  pool 0 on storage 1 at base 64, stride 128, 2 blocks.  A pattern written
  at the pool's block 0 (storage 1 bytes [64, 192) of the host tier) reaches
  the device at storage 1 bytes
  [64, 192) and storage 0 stays zero; block 2 lies outside the pool (though
  inside storage 1), so a copy of it is refused and its bytes, host and
  device, stay as they were."""
  grid, mgr = ref_manager(2, 64, 8)
  mgr.register_pools([dense_pool("kind_a", 1, 64, 128, 2)])
  pattern = bytes((i * 17 + 3) % 251 for i in range(128))
  # the 128-byte pool block spans two 64-byte host blocks, which are not
  # adjacent on the block-major tier: no single host pointer covers it
  with pytest.raises(RuntimeError, match="spans several host blocks"):
    mgr.get_block_ref(0, 0)
  for i in range(0, 128, 64):
    ctypes.memmove(host_addr(mgr, 1, 64 + i), pattern[i:i + 64], 64)
  mgr.h2d_pool_blocks(0, [0]).Await()
  dev1 = grid[1][0].view(-1).cpu().numpy()
  assert dev1[64:192].tobytes() == pattern
  assert not dev1[:64].any() and not dev1[192:].any()
  assert not grid[0][0].any()
  grid[1][0].view(-1)[64 + 2 * 128:64 + 3 * 128].fill_(0xD4)
  with pytest.raises(RuntimeError, match="out of range"):
    mgr.d2h_pool_blocks(0, [2])
  with pytest.raises(RuntimeError, match="out of range"):
    mgr.h2d_pool_blocks(0, [2])
  torch.cuda.synchronize()
  assert not host_bytes(mgr, 1, 64 + 2 * 128, 128).any()
  assert (grid[1][0].view(-1)[64 + 2 * 128:64 + 3 * 128] == 0xD4).all()
  mgr.close()


def test_aliased_pool_transport_copies_only_live_regions_and_preserves_padding():
  """AliasedPoolTransportCopiesOnlyLiveRegionsAndPreservesPadding (:394-440):
  strided pool at base 32, stride 128, 2 blocks on a 256-byte storage.  Its
  logical end (288) passes the storage but its last live byte is 256, so it
  is admitted and block 1 sits at byte 160.  Copying block 1 moves the live
  [160, 192) and [224, 256) and leaves the padding [192, 224) alone."""
  grid, mgr = ref_manager(1, 128, 2)
  mgr.register_pools([strided_pool("aliased", 0, 32, 128, 2)])
  assert mgr.get_block_ref(0, 1)["ptr"] == host_addr(mgr, 0, 160)
  dev = grid[0][0].view(-1)
  dev.fill_(0xA5)
  dev[160:192].fill_(0x11)
  dev[224:256].fill_(0x22)
  tier = mgr.host_tier_view()
  tier[:] = 0xEE
  mgr.d2h_pool_blocks(0, [1]).Await()
  h = host_bytes(mgr, 0, 0, 256)
  assert (h[160:192] == 0x11).all() and (h[192:224] == 0xEE).all() and (h[224:256] == 0x22).all()
  assert (h[:160] == 0xEE).all()
  dev.zero_()
  mgr.h2d_pool_blocks(0, [1]).Await()
  torch.cuda.synchronize()
  d = dev.cpu().numpy()
  assert (d[160:192] == 0x11).all() and (d[224:256] == 0x22).all()
  assert not d[:160].any() and not d[192:224].any()
  mgr.close()


def test_explicit_pool_transport_enumerates_all_pools():
  """ExplicitPoolTransportEnumeratesAllPools (:442-520): two pools on one
  storage (kind_a at 0, kind_b at 256, 64-byte blocks); each pool's copy of
  its block 1 moves that pool's bytes only, both ways."""
  grid, mgr = ref_manager(1, 64, 8)
  mgr.register_pools([dense_pool("kind_a", 0, 0, 64, 2), dense_pool("kind_b", 0, 256, 64, 2)])
  assert mgr.num_pools() == 2
  dev = grid[0][0].view(-1)
  dev[64:128].fill_(0xA1)
  dev[256 + 64:256 + 128].fill_(0xB2)
  mgr.d2h_pool_blocks(0, [1]).Await()
  h = host_bytes(mgr, 0, 0, 512)
  assert (h[64:128] == 0xA1).all() and not h[256:].any()
  mgr.d2h_pool_blocks(1, [1]).Await()
  h = host_bytes(mgr, 0, 0, 512)
  assert (h[320:384] == 0xB2).all() and not h[:64].any() and not h[128:320].any()
  dev.zero_()
  mgr.h2d_pool_blocks(0, [1]).Await()
  mgr.h2d_pool_blocks(1, [1]).Await()
  torch.cuda.synchronize()
  d = dev.cpu().numpy()
  assert (d[64:128] == 0xA1).all() and (d[320:384] == 0xB2).all()
  assert not d[:64].any() and not d[128:320].any() and not d[384:].any()
  mgr.close()


def test_pool_block_copies_reject_host_only_manager():
  """PoolBlockCopiesRejectHostOnlyManager (:522-538): this build has no
  host-only manager to refuse (blocks live in HBM); asking for one says so."""
  with pytest.raises(NotImplementedError, match="no host-only manager"):
    KVCacheManager.create_host_only_for_testing(num_layers=1, slice_byte_size=64, node_id=0,
                                                host_blocks=2)


def test_implicit_pools_mirror_storages():
  """ImplicitPoolsMirrorStorages (:540-556)."""
  _, mgr = ref_manager(2, 128, 2)
  assert not mgr.has_explicit_pools() and mgr.num_pools() == 2
  p = mgr.pool_spec(0)
  assert (p["tag"], p["storage_index"], p["base_offset_bytes"], p["block_stride_bytes"],
          p["num_blocks"]) == ("opaque", 0, 0, 128, 2)
  assert mgr.get_block_ref(1, 1)["ptr"] == host_addr(mgr, 1, 128)
  mgr.close()

"""GPU parity of the block extract/insert kernels and the KVCacheManager
offload/reload path against the CPU oracle (bit-exact)."""

import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import kv_blocks as ref
from tpu_sync_b200 import KVCacheManager, ops, workloads

pytestmark = pytest.mark.gpu


def u8(t: torch.Tensor) -> np.ndarray:
  return t.contiguous().view(torch.uint8).cpu().numpy().reshape(t.shape[0], -1)


def small_pool(geom, blocks, seed, device):
  return workloads.kv_pool(geom, blocks, seed, device)


def test_c0_extract_insert_round_trip(cuda):
  """Config 0: extract 128 ids (seed 1) into block-major staging, insert at 128
  other ids (seed 2); bit-exact against the oracle, round trip exact."""
  g = workloads.C0
  pool = small_pool(g, workloads.C0_BLOCKS, 0, cuda)
  ids_x = workloads.distinct_ids(workloads.C0_IDS, workloads.C0_BLOCKS, 1)
  ids_i = workloads.distinct_ids(workloads.C0_IDS, workloads.C0_BLOCKS, 2)
  host_pool = [u8(t) for t in pool]
  table = ops.StorageTable(pool)
  staging = table.new_staging(len(ids_x))
  err = torch.zeros(1, dtype=torch.int32, device=cuda)
  ops.kv_extract(table, ids_x, staging, err_flag=err)
  torch.cuda.synchronize()
  want = ref.extract_to_padded_staging(host_pool, ids_x)
  np.testing.assert_array_equal(staging.cpu().numpy(), want)
  # contiguous staging [128, 4, 2, 16, 8, 128] bf16 (no padding at these sizes)
  assert table.pitch == g.block_bytes
  st6 = staging.view(torch.bfloat16).view(len(ids_x), g.layers, g.kv, g.block_tokens,
                                          g.heads, g.head_dim)
  full = torch.stack([torch.stack(pool[l * 2:l * 2 + 2]) for l in range(g.layers)])
  torch.testing.assert_close(st6[5], full[:, :, int(ids_x[5])], rtol=0, atol=0)
  ops.kv_insert(table, ids_i, staging, err_flag=err)
  torch.cuda.synchronize()
  ref.insert_from_staging(host_pool, ids_i, want)
  for t, h in zip(pool, host_pool):
    np.testing.assert_array_equal(u8(t), h)
  assert int(err.item()) == 0


@pytest.mark.parametrize("block_tokens,heads,head_dim,n_st", [
    (16, 8, 128, 3),   # 32 KiB blocks: two 16 KiB pieces
    (1, 1, 8, 5),      # 16-byte blocks
    (3, 1, 40, 2),     # 240-byte blocks: 16-aligned, single partial piece
    (64, 1, 136, 2),   # 17 KiB blocks: partial second piece
])
def test_extract_insert_shapes(cuda, block_tokens, heads, head_dim, n_st):
  geom = workloads.KVGeometry(layers=n_st, kv=1, block_tokens=block_tokens, heads=heads,
                              head_dim=head_dim)
  pool = small_pool(geom, 37, 11, cuda)
  ids = [36, 0, 5, 5, 17]
  table = ops.StorageTable(pool)
  staging = table.new_staging(len(ids))
  ops.kv_extract(table, ids, staging)
  torch.cuda.synchronize()
  want = ref.extract_to_padded_staging([u8(t) for t in pool], ids)
  np.testing.assert_array_equal(staging.cpu().numpy(), want)


def test_unaligned_block_bytes_use_byte_path(cuda):
  # 6-byte blocks (3 x bf16): vector path impossible, byte kernel must be exact
  pool = [torch.arange(30 * 3, dtype=torch.int16, device=cuda).view(30, 3) + 100 * s
          for s in range(3)]
  ids = [29, 3, 0, 14]
  table = ops.StorageTable(pool)
  staging = table.new_staging(len(ids))
  staging.zero_()
  ops.kv_extract(table, ids, staging)
  torch.cuda.synchronize()
  want = ref.extract_to_padded_staging([u8(t) for t in pool], ids)
  np.testing.assert_array_equal(staging.cpu().numpy(), want)


def test_out_of_bounds_id_sets_error_flag(cuda):
  pool = small_pool(workloads.KVGeometry(2, 1, 4, 1, 64), 8, 3, cuda)
  table = ops.StorageTable(pool)
  staging = table.new_staging(2)
  err = torch.zeros(1, dtype=torch.int32, device=cuda)
  ops.kv_extract(table, [1, 8], staging, err_flag=err)
  torch.cuda.synchronize()
  assert int(err.item()) == 1
  np.testing.assert_array_equal(staging[0].cpu().numpy(),
                                ref.extract_to_padded_staging([u8(t) for t in pool], [1])[0])


def test_manager_free_calls_queue_without_blocking(cuda):
  """ts_kv_extract / ts_kv_insert and their fp8 variants read nothing back
  from the device: queued behind ~0.5 s of GPU work on their stream, two
  calls of each return at once, and the copies land exactly once the stream
  drains."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=8, head_dim=128)
  pool = small_pool(geom, 48, 17, cuda)
  host_pool = [u8(t) for t in pool]
  ids_a = torch.tensor([3, 40, 7, 0], dtype=torch.int64, device=cuda)
  ids_b = torch.tensor([11, 12, 47], dtype=torch.int64, device=cuda)
  table = ops.StorageTable(pool)
  ftable = ops.StorageTable(pool, fp8=True)
  sa, sb = table.new_staging(4), table.new_staging(3)
  fa, fb = ftable.new_staging(4), ftable.new_staging(3)
  err = torch.zeros(1, dtype=torch.int32, device=cuda)
  dst = [torch.empty_like(t) for t in pool]
  dtable = ops.StorageTable(dst)
  stream = torch.cuda.Stream(cuda)
  # warm-up: the first launch of each kernel (the sleep kernel too) in a
  # fresh process loads it (lazy module loading), which must not fall inside
  # the window the sleep covers
  ops.kv_extract(table, ids_a, sa, err_flag=err, stream=stream)
  ops.kv_extract(ftable, ids_a, fa, err_flag=err, stream=stream)
  ops.kv_insert(dtable, ids_a, sa, err_flag=err, stream=stream)
  with torch.cuda.stream(stream):
    torch.cuda._sleep(1000)
  torch.cuda.synchronize()
  with torch.cuda.stream(stream):
    torch.cuda._sleep(1_000_000_000)  # ~0.5 s at the B200's clocks
  import time
  t0 = time.perf_counter()
  for ids, stg, fstg in ((ids_a, sa, fa), (ids_b, sb, fb)):
    ops.kv_extract(table, ids, stg, err_flag=err, stream=stream)
    ops.kv_extract(ftable, ids, fstg, err_flag=err, stream=stream)
    ops.kv_insert(dtable, ids, stg, err_flag=err, stream=stream)
  host_s = time.perf_counter() - t0
  assert stream.query() is False  # the sleep is still running
  assert host_s < 0.1, f"calls blocked the host for {host_s:.3f} s"
  stream.synchronize()
  assert int(err.item()) == 0
  for ids, stg, fstg in ((ids_a, sa, fa), (ids_b, sb, fb)):
    idl = ids.tolist()
    np.testing.assert_array_equal(stg.cpu().numpy(), ref.extract_to_padded_staging(host_pool, idl))
    (payload, _), _ = fp8_oracle(pool, idl)
    fs = fstg.cpu().numpy()
    for k in range(len(pool)):
      off = ftable.stage_offs[k]
      np.testing.assert_array_equal(fs[:, off:off + payload.shape[2]], payload[:, k])
    for t, d in zip(pool, dst):
      for i in idl:
        assert torch.equal(t[i], d[i])


def test_fp8_misaligned_table_sets_error_flag(cuda):
  """A storage whose address is not 16-byte aligned cannot take the fp8
  kernels' 16-byte vectors: the kernel reports it as *err_flag = 2 and moves
  nothing (the table is checked on the device, not read back)."""
  geom = workloads.KVGeometry(layers=1, kv=2, block_tokens=64, heads=1, head_dim=128)
  good = small_pool(geom, 8, 5, cuda)
  raw = torch.zeros(8 * 64 * 128 + 1, dtype=torch.bfloat16, device=cuda)
  bad = raw[1:].view(8, 64, 1, 128)  # address 2 bytes past an aligned one
  bad.copy_(good[1])
  table = ops.StorageTable([good[0], bad], fp8=True)
  staging = table.new_staging(2)
  staging.fill_(0x33)
  err = torch.zeros(1, dtype=torch.int32, device=cuda)
  ops.kv_extract(table, [1, 4], staging, err_flag=err)
  torch.cuda.synchronize()
  assert int(err.item()) == 2
  assert (staging.cpu().numpy() == 0x33).all()
  err.zero_()
  before = [t.clone() for t in (good[0], bad)]
  ops.kv_insert(table, [1, 4], staging, err_flag=err)
  torch.cuda.synchronize()
  assert int(err.item()) == 2
  assert torch.equal(before[0], good[0]) and torch.equal(before[1], bad)


# ---------------------------------------------------------------------------
# fp8 fused cast
# ---------------------------------------------------------------------------

def fp8_oracle(pool, ids):
  bits = [t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(
      t.shape[0], -1) for t in pool]
  return ofp8.extract_fp8(bits, ids), bits


def test_fp8_extract_out_of_bounds_id_sets_error_flag(cuda):
  """16 KiB units (the bulk-copy kernel): an id past the storage flags the
  error and is skipped; the ids around it are still extracted exactly."""
  pool = small_pool(workloads.KVGeometry(2, 1, 64, 1, 128), 8, 4, cuda)
  table = ops.StorageTable(pool, fp8=True)
  ids = [1, 8, 2, 7, 0]
  staging = table.new_staging(len(ids))
  staging.fill_(0x5A)
  err = torch.zeros(1, dtype=torch.int32, device=cuda)
  ops.kv_extract(table, ids, staging, err_flag=err)
  torch.cuda.synchronize()
  assert int(err.item()) == 1
  good = [0, 2, 3, 4]
  (payload, scales), _ = fp8_oracle(pool, [ids[i] for i in good])
  st = staging.cpu().numpy()
  for s in range(len(pool)):
    off = table.stage_offs[s]
    np.testing.assert_array_equal(st[good, off:off + payload.shape[2]], payload[:, s])
  assert (st[1] == 0x5A).all()  # the skipped block's staging row is untouched


@pytest.mark.parametrize("block_tokens,heads,n_blocks", [(64, 1, 40), (16, 8, 9), (256, 4, 3)])
def test_fp8_extract_insert_matches_oracle(cuda, block_tokens, heads, n_blocks):
  geom = workloads.KVGeometry(layers=3, kv=2, block_tokens=block_tokens, heads=heads,
                              head_dim=128)
  pool = small_pool(geom, n_blocks + 4, 20, cuda)
  # edge units: all zero, a huge value (saturation path), tiny values
  pool[0][1].zero_()
  pool[1][2].mul_(1e4)
  pool[2][3].mul_(1e-30)
  ids = list(range(n_blocks))
  table = ops.StorageTable(pool, fp8=True)
  staging = table.new_staging(len(ids))
  ops.kv_extract(table, ids, staging)
  torch.cuda.synchronize()
  (payload, scales), bits = fp8_oracle(pool, ids)
  st = staging.cpu().numpy()
  for s in range(len(pool)):
    off = table.stage_offs[s]
    np.testing.assert_array_equal(st[:, off:off + payload.shape[2]], payload[:, s])
  got_scales = st[:, table.scale_off:table.scale_off + 4 * len(pool)].copy().view(np.float32)
  np.testing.assert_array_equal(got_scales, scales)
  assert got_scales[1, 0] == 1.0  # zero unit
  # dequant into other blocks
  dst_ids = [n_blocks + 3 - (i % 4) for i in range(len(ids))][:4]
  ops.kv_insert(table, dst_ids, staging[:4])
  torch.cuda.synchronize()
  ofp8.insert_fp8(payload[:4], scales[:4], dst_ids, bits)
  for t, b in zip(pool, bits):
    np.testing.assert_array_equal(
        t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(b.shape), b)


# ---------------------------------------------------------------------------
# KVCacheManager (pinned host tier, pipelined gather + DMA)
# ---------------------------------------------------------------------------

MODES = [dict(mode="staged", copy_streams=1), dict(mode="staged", copy_streams=2),
         dict(mode="direct", max_ctas=64), dict(mode="direct_d2h", max_ctas=148),
         dict(mode="direct_h2d"), dict(mode="direct_h2d", reload_staged_every=2),
         dict(mode="direct_h2d", sched=("offload_priority", "reload_per_piece")),
         dict(mode="direct_h2d", sched=("offload_priority", "reload_per_piece",
                                        "reload_overlap")),
         dict(mode="direct", sched=("reload_per_piece", "reload_overlap")),
         dict(mode="direct", sched=("wide_loads",)),
         dict(mode="direct_h2d", sched=("offload_priority", "reload_per_piece", "bulk_copy",
                                        "wide_loads")),
         dict(mode="staged", sched=("offload_priority",)),
         dict(mode="staged", copy_streams=1, sched=("bulk_copy",)),
         dict(mode="direct_h2d", sched=("offload_priority", "reload_per_piece", "bulk_copy"))]


def make_pair(geom, blocks, host_blocks, seed, cuda, chunk_blocks=0, **kw):
  pool = small_pool(geom, blocks, seed, cuda)
  grid = [[t] for t in pool]
  mgr = KVCacheManager(grid, host_blocks_to_allocate=host_blocks, chunk_blocks=chunk_blocks,
                       **kw)
  model = ref.RefKVManager([[u8(t).reshape(-1).copy()] for t in pool], dim0=blocks,
                           host_blocks=host_blocks)
  return pool, mgr, model


def assert_same(pool, mgr, model, host_ids):
  for l, t in enumerate(pool):
    np.testing.assert_array_equal(u8(t).reshape(-1), model.device[l][0])
    for h in host_ids:
      assert mgr.read_block_bytes(l, h) == model.host_block(l, h), (l, h)


@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("chunk_blocks", [0, 3])
def test_manager_offload_reload_matches_model(cuda, chunk_blocks, mode):
  geom = workloads.KVGeometry(layers=4, kv=2, block_tokens=16, heads=2, head_dim=128)
  pool, mgr, model = make_pair(geom, 64, 96, 5, cuda, chunk_blocks, **mode)
  rng = np.random.default_rng(3)
  for step in range(6):
    n = int(rng.integers(1, 40))
    src = list(rng.choice(64, n, replace=False))
    dst = list(rng.choice(96, n, replace=False))
    if step == 2:  # coalescible runs with sizes
      src, dst, sizes = [0, 4, 10], [50, 54, 70], [4, 3, 6]
    else:
      sizes = None
    f = mgr.d2h(src, dst, sizes)
    assert model.d2h(src, dst, sizes) == (ref.OK, "")
    f.Await()
    assert f.is_ready() and f.ok() and f.error_message() == ""
    hs = list(rng.choice(96, n, replace=False))
    ds = list(rng.choice(64, n, replace=False))
    g = mgr.h2d(hs, ds)
    assert model.h2d(hs, ds) == (ref.OK, "")
    g.Await()
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(96))


@pytest.mark.parametrize("mode", MODES)
def test_manager_repeated_destination_last_copy_wins(cuda, mode):
  """A destination block named twice in one call ends with the later copy's
  bytes, as the reference's in-order per-run copies leave it
  (kv_cache_manager_base.cc:1945-2124), also when the two copies fall into
  different pipelined chunks."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=2, head_dim=128)
  pool, mgr, model = make_pair(geom, 48, 48, 21, cuda, chunk_blocks=3, **mode)
  mgr.d2h(list(range(20)), list(range(20))).Await()
  model.d2h(list(range(20)), list(range(20)))
  hs = [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11]
  ds = [30, 31, 32, 33, 30, 34, 31, 35, 36, 30, 37, 31]
  mgr.h2d(hs, ds).Await()
  assert model.h2d(hs, ds) == (ref.OK, "")
  src = [40, 41, 42, 43, 44, 45, 46, 47]
  dst = [25, 26, 25, 27, 28, 26, 29, 25]
  mgr.d2h(src, dst).Await()
  assert model.d2h(src, dst) == (ref.OK, "")
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(48))


@pytest.mark.parametrize("mode", MODES + [dict(mode="staged", sched=("bulk_copy",)),
                                          dict(mode="direct_h2d", sched=("bulk_copy",))])
def test_manager_repeated_destination_within_one_chunk(cuda, mode):
  """Destinations named many times inside one pipelined chunk (the default
  64-block chunks run all their pieces at once): every copy of the call
  lands as if run in order, the last one to a block winning
  (kv_cache_manager_base.cc:1945-2124), in both directions."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=2, head_dim=128)
  pool, mgr, model = make_pair(geom, 96, 64, 27, cuda, **mode)
  rng = np.random.default_rng(11)
  mgr.d2h(list(range(48)), list(range(48))).Await()
  model.d2h(list(range(48)), list(range(48)))
  for _ in range(3):
    hs = [int(x) for x in rng.integers(0, 48, 40)]
    ds = [int(x) for x in rng.choice([60, 61, 62, 63, 70], 40)]
    mgr.h2d(hs, ds).Await()
    assert model.h2d(hs, ds) == (ref.OK, "")
    src = [int(x) for x in rng.integers(0, 96, 40)]
    dst = [int(x) for x in rng.choice([50, 51, 52, 5], 40)]
    mgr.d2h(src, dst).Await()
    assert model.d2h(src, dst) == (ref.OK, "")
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(64))


@pytest.mark.parametrize("numa", [None, 0, "none"])
def test_manager_numa_node_option(cuda, numa):
  """The manager's NUMA node: the device's own by default (the reference's
  DetectAndAssignNumaNode), a caller's override, or none; the host tier is
  allocated under that placement and the round trip stays exact."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=2, head_dim=128)
  pool, mgr, model = make_pair(geom, 32, 16, 41, cuda, numa_node=numa)
  if numa == 0:
    assert mgr.assigned_numa_node == 0
  elif numa == "none":
    assert mgr.assigned_numa_node is None and not mgr.host_tier_numa_placed
  else:
    assert mgr.assigned_numa_node is None or mgr.assigned_numa_node >= 0
  assert isinstance(mgr.host_tier_numa_placed, bool)
  mgr.d2h(list(range(10)), list(range(10))).Await()
  model.d2h(list(range(10)), list(range(10)))
  mgr.h2d(list(range(10)), list(range(20, 30))).Await()
  model.h2d(list(range(10)), list(range(20, 30)))
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(16))
  mgr.close()


@pytest.mark.parametrize("mode", MODES)
def test_manager_back_to_back_calls_are_ordered(cuda, mode):
  """Offload then reload of the same host blocks without waiting in between."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=8, head_dim=128)
  pool, mgr, model = make_pair(geom, 128, 128, 9, cuda, chunk_blocks=8, **mode)
  futs = []
  for i in range(4):
    src = list(range(i * 20, i * 20 + 20))
    futs.append(mgr.d2h(src, list(range(20))))
    model.d2h(src, list(range(20)))
    futs.append(mgr.h2d(list(range(20)), list(range(100, 120))))
    model.h2d(list(range(20)), list(range(100, 120)))
  for f in futs:
    f.Await()
  assert_same(pool, mgr, model, range(128))


@pytest.mark.parametrize("mode", MODES)
def test_manager_partial_hazards_reorder(cuda, mode):
  """A reload whose host blocks are partly written by an in-flight offload,
  and an offload whose device blocks are partly written by an in-flight
  reload: dependent blocks wait, independent ones do not, result as if
  the calls ran in program order."""
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=4, head_dim=128)
  pool, mgr, model = make_pair(geom, 256, 128, 13, cuda, chunk_blocks=8, **mode)
  futs = []
  for rep in range(3):
    d_src = list(range(rep * 40, rep * 40 + 40))
    h_dst = list(range(0, 40))
    futs.append(mgr.d2h(d_src, h_dst))
    model.d2h(d_src, h_dst)
    h_src = list(range(20, 60))          # 20 conflicting + 20 independent
    d_dst = list(range(200, 240))
    futs.append(mgr.h2d(h_src, d_dst))
    model.h2d(h_src, d_dst)
    d_src2 = list(range(220, 250))       # 20 written by the reload above
    h_dst2 = list(range(80, 110))
    futs.append(mgr.d2h(d_src2, h_dst2))
    model.d2h(d_src2, h_dst2)
  for f in futs:
    f.Await()
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(128))


@pytest.mark.parametrize("mode", MODES)
def test_manager_whole_storage_and_layer_restricted(cuda, mode):
  geom = workloads.KVGeometry(layers=3, kv=1, block_tokens=4, heads=2, head_dim=64)
  pool, mgr, model = make_pair(geom, 16, 16, 2, cuda, **mode)
  mgr.d2h([], []).Await()
  assert model.d2h([], []) == (ref.OK, "")
  f = mgr.h2d([3, 4], [9, 10], layer_idx=1)
  assert model.h2d([3, 4], [9, 10], layer_idx=1) == (ref.OK, "")
  f.Await()
  f = mgr.d2h([0, 1, 2], [13, 14, 15], layer_idx=2, shard_idx=0)
  assert model.d2h([0, 1, 2], [13, 14, 15], layer_idx=2, shard_idx=0) == (ref.OK, "")
  f.Await()
  assert_same(pool, mgr, model, range(16))


def test_manager_errors_match_reference(cuda):
  geom = workloads.KVGeometry(layers=2, kv=1, block_tokens=4, heads=1, head_dim=64)
  pool, mgr, model = make_pair(geom, 8, 4, 2, cuda)
  cases = [
      ("d2h", dict(src=[0], dst=[0, 1], sizes=[1])),
      ("h2d", dict(src=[-1], dst=[0], sizes=[1])),
      ("d2h", dict(src=[7], dst=[4], sizes=[1])),
      ("d2h", dict(src=[8], dst=[0], sizes=[1])),
      ("h2d", dict(src=[3], dst=[0], sizes=[2])),
      ("h2d", dict(src=[0], dst=[7], sizes=[2])),
      ("d2h", dict(src=[], dst=[], sizes=[])),          # whole storage > host tier
      ("h2d", dict(src=[], dst=[], sizes=[])),
      ("h2d", dict(src=[0], dst=[0], sizes=[1], layer_idx=2)),
  ]
  for op, kw in cases:
    code, msg = getattr(model, op)(kw["src"], kw["dst"], kw["sizes"], kw.get("layer_idx"))
    assert code != ref.OK, (op, kw)
    with pytest.raises(RuntimeError) as e:
      getattr(mgr, op)(kw["src"], kw["dst"], kw["sizes"], layer_idx=kw.get("layer_idx"))
    prefix = "KVCacheManager D2h failed: " if op == "d2h" else "KVCacheManager H2d failed: "
    assert str(e.value) == prefix + msg


def test_heterogeneous_layer_block_sizes_transfer(cuda):
  """Port of tpu_sync/frameworks/torch/kv_cache_manager_test.py:206-275."""
  shapes = [(4, 128, 8), (4, 128, 2)]
  src_t, dst_t = [], []
  for l, s in enumerate(shapes):
    n = int(np.prod(s))
    src_t.append([(torch.arange(n, dtype=torch.float32).reshape(s) + 1000.0 * (l + 1)).to(cuda)])
    dst_t.append([torch.zeros(s, dtype=torch.float32, device=cuda)])
  ws_src = KVCacheManager(src_t, 0, host_blocks_to_allocate=4, parallelism=1)
  ws_dst = KVCacheManager(dst_t, 0, host_blocks_to_allocate=4, parallelism=1)
  ws_src.D2h([2], [2], [2]).Await()
  for l in range(2):  # H2hWrite stand-in: the peer's host blocks 0..1
    for b in range(2):
      ws_dst.write_block_bytes(l, b, ws_src.read_block_bytes(l, 2 + b))
  ws_dst.H2d([0], [2], [2]).Await()
  for l in range(2):
    got, want = dst_t[l][0].cpu(), src_t[l][0].cpu()
    torch.testing.assert_close(got[2:4], want[2:4], rtol=0, atol=0)
    assert torch.count_nonzero(got[0:2]) == 0


@pytest.mark.parametrize("mode", MODES)
def test_fp8_manager_round_trip(cuda, mode):
  geom = workloads.KVGeometry(layers=4, kv=2, block_tokens=64, heads=1, head_dim=128)
  pool = small_pool(geom, 32, 21, cuda)
  mgr = KVCacheManager([[t] for t in pool], host_blocks_to_allocate=32, fp8=True, **mode)
  ids = [3, 9, 27, 30]
  mgr.d2h(ids, [0, 1, 2, 3]).Await()
  (payload, scales), bits = fp8_oracle(pool, ids)
  for s in range(len(pool)):
    for k in range(len(ids)):
      assert mgr.read_block_bytes(s, k) == payload[k, s].tobytes()
  mgr.h2d([0, 1, 2, 3], [0, 1, 2, 4]).Await()
  ofp8.insert_fp8(payload, scales, [0, 1, 2, 4], bits)
  for t, b in zip(pool, bits):
    np.testing.assert_array_equal(
        t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(b.shape), b)


def test_fp8_quantizer_exact_over_bf16_domain(cuda):
  """The in-kernel x / scale (Markstein-corrected reciprocal product, IEEE
  division for units whose scale or reciprocal is not normal) must equal the
  IEEE round-to-nearest division of the oracle: every finite bf16 value, and
  2000 units of random magnitudes below random maxima (tiny ones included)."""
  rng = np.random.default_rng(17)
  bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
  finite = bits[(bits & 0x7FFF) < 0x7F80]
  units = [np.zeros(8192, np.uint16) for _ in range(8)]
  for i, chunk in enumerate(np.array_split(finite, 8)):
    units[i][:chunk.size] = chunk
  for _ in range(2000):
    amax_bits = int(rng.integers(1, 0x7F80))
    mag = rng.integers(0, amax_bits + 1, 8192, dtype=np.uint32).astype(np.uint16)
    sign = (rng.integers(0, 2, 8192, dtype=np.uint32) << 15).astype(np.uint16)
    u = mag | sign
    u[0] = amax_bits
    units.append(u)
  host = np.stack(units)                      # [n_units, 8192] bf16 bit patterns
  store = torch.from_numpy(host.view(np.int16)).to(cuda).view(torch.bfloat16)
  store = store.view(host.shape[0], 64, 1, 128)
  table = ops.StorageTable([store], fp8=True)
  ids = list(range(host.shape[0]))
  staging = table.new_staging(len(ids))
  ops.kv_extract(table, ids, staging)
  torch.cuda.synchronize()
  payload, scales = ofp8.extract_fp8([host], ids)
  st = staging.cpu().numpy()
  np.testing.assert_array_equal(st[:, 0:8192], payload[:, 0])
  got_scales = st[:, table.scale_off:table.scale_off + 4].copy().view(np.float32)[:, 0]
  np.testing.assert_array_equal(got_scales, scales[:, 0])


@pytest.mark.parametrize("mode", [dict(mode="staged"), dict(mode="direct_h2d")])
def test_manager_concurrent_callers(cuda, mode):
  """Four host threads (ctypes releases the GIL, as the reference's bindings
  do) offload and reload disjoint block ranges through one manager at once;
  the result equals the model applying the same calls."""
  import threading
  geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=4, head_dim=128)
  pool, mgr, model = make_pair(geom, 256, 128, 21, cuda, chunk_blocks=8, **mode)
  plans = []
  for t in range(4):
    rng = np.random.default_rng(100 + t)
    dev = list(range(t * 64, t * 64 + 32))      # offload sources of thread t
    back = list(range(t * 64 + 32, t * 64 + 64))  # reload targets of thread t
    host = list(range(t * 32, t * 32 + 32))
    plans.append((list(rng.permutation(dev)), list(rng.permutation(host)), back))
  errors = []

  def worker(t):
    try:
      dev, host, back = plans[t]
      for r in range(3):
        mgr.d2h(dev, host).Await()
        mgr.h2d(host, back).Await()
    except Exception as e:  # surfaced below
      errors.append(e)

  threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
  for th in threads:
    th.start()
  for th in threads:
    th.join()
  assert not errors, errors
  for t in range(4):
    dev, host, back = plans[t]
    model.d2h(dev, host)
    model.h2d(host, back)
  torch.cuda.synchronize()
  assert_same(pool, mgr, model, range(128))

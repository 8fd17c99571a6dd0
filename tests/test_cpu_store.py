"""CPU tests of the tier-2 store: its LRU index replayed against the
reference's own LRUCache (compiled by oracle/build_ref.py), its host block
allocator against the reference's own LogicalBlockManager (operation scripts
it answered, tests/golden/block_manager.json), the LogicalBlockManager
restatement and the reference's allocator test expectations, and the local
Lookup / Insert / Save / Load / Poll state machine (host-only mode:
transfers complete at issue)."""

import ctypes
import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import block_manager as obm
from oracle import build_ref
from tpu_sync_b200 import _native
from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId


def lru_op(store, op, key=b"", val=None):
  info = _native.BlockInfo(*val, 0) if val is not None else None
  out_info = _native.BlockInfo()
  out = ctypes.c_int64()
  kbuf = ctypes.create_string_buffer(64)
  klen = ctypes.c_int64()
  _native.check(_native.lib().ts_store_lru_op(
      store._impl, op, key, len(key), ctypes.byref(info) if info is not None else None,
      ctypes.byref(out_info), ctypes.byref(out), kbuf, 64, ctypes.byref(klen)))
  return out.value, out_info, (kbuf.raw[:klen.value] if klen.value >= 0 else None)


@pytest.mark.parametrize("seed", range(6))
def test_lru_matches_reference_lrucache(seed):
  exe = build_ref.build()
  if exe is None:
    pytest.skip("reference checkout not available to build the LRU oracle")
  rng = np.random.default_rng(seed)
  cap = int(rng.integers(2, 9))
  store = KVCacheStore(capacity=cap, host_blocks=4)
  keys = [f"k{i}" for i in range(14)]
  lines, ours = [], []
  for _ in range(600):
    op = rng.choice(["put", "pin", "unpin", "erase", "contains", "peek", "peekany", "pins",
                     "avail", "size", "evictable"], p=[.3, .12, .12, .06, .06, .08, .06, .05,
                                                       .05, .05, .05])
    k = str(rng.choice(keys))
    kb = k.encode()
    if op == "put":
      v = (int(rng.integers(0, 9)), int(rng.integers(0, 9)), int(rng.integers(0, 5)))
      lines.append(f"put {k} {v[0]} {v[1]} {v[2]}")
      flag, _, demoted = lru_op(store, 0, kb, v)
      ours.append(demoted.decode() if flag else "-")
    elif op in ("pin", "unpin", "erase", "contains"):
      lines.append(f"{op} {k}")
      code = {"pin": 1, "unpin": 2, "erase": 6, "contains": 7}[op]
      ours.append(str(lru_op(store, code, kb)[0]))
    elif op in ("peek", "peekany"):
      lines.append(f"{op} {k}")
      found, info, _ = lru_op(store, 3 if op == "peek" else 4, kb)
      ours.append(f"{info.host_block_id} {info.device_block_id} {info.status}" if found else "-")
    elif op == "pins":
      lines.append(f"pins {k}")
      ours.append(str(lru_op(store, 5, kb)[0]))
    elif op in ("avail", "size"):
      lines.append(op)
      ours.append(str(lru_op(store, 8 if op == "avail" else 9)[0]))
    else:
      n = int(rng.integers(0, 10))
      lines.append(f"evictable {n}")
      ev = [x.decode() for x in store.evictable_order()][:n]
      ours.append(" ".join(ev) if ev else "-")
  ref = subprocess.run([str(exe), str(cap)], input="\n".join(lines) + "\n", text=True,
                       capture_output=True, check=True).stdout.splitlines()
  assert ref == ours


def host_op(store, op, ids):
  a = np.asarray(ids, np.int32)
  return _native.lib().ts_store_host_block_op(store._impl, op, a.ctypes.data_as(_native.c_i32_p),
                                              a.size)


def alloc(store, n, lock):
  out = np.zeros(max(n, 1), np.int32)
  rc = _native.lib().ts_store_allocate_host_blocks(store._impl, n, int(lock),
                                                   out.ctypes.data_as(_native.c_i32_p))
  return rc, (list(out[:n]) if rc == 0 else None)


def test_allocator_reference_expectations():
  # tpu_sync/kv_cache/logical_block_manager_test.cc (5 blocks)
  s = KVCacheStore(capacity=4, host_blocks=5)
  assert alloc(s, 3, False) == (0, [0, 1, 2])
  s = KVCacheStore(capacity=4, host_blocks=4)
  assert alloc(s, 2, False)[1] == [0, 1]
  assert alloc(s, 2, False)[1] == [2, 3]
  assert alloc(s, 2, False)[1] == [0, 1]          # LruEvictionOrder
  s = KVCacheStore(capacity=4, host_blocks=4)
  alloc(s, 2, False), alloc(s, 2, False)
  assert host_op(s, 3, [0]) == 0 and host_op(s, 3, [1]) == 0
  assert alloc(s, 2, False)[1] == [2, 3]          # AccessUpdatesLruOrder
  s = KVCacheStore(capacity=4, host_blocks=4)
  alloc(s, 2, True), alloc(s, 2, False)
  assert alloc(s, 3, False)[0] == _native.RESOURCE_EXHAUSTED   # LockedBlocksPreventEviction
  assert host_op(s, 2, [0, 1]) == 0
  assert alloc(s, 3, False)[0] == 0               # UnlockAllowsEviction
  s = KVCacheStore(capacity=4, host_blocks=5)
  assert alloc(s, 0, False)[0] == _native.INVALID_ARGUMENT
  assert alloc(s, 6, False)[0] == _native.INVALID_ARGUMENT
  assert host_op(s, 3, [5]) == _native.INVALID_ARGUMENT
  assert host_op(s, 3, [0]) == _native.INVALID_ARGUMENT
  assert host_op(s, 1, [1, 3]) == 0               # AllocateTarget
  assert host_op(s, 1, [1]) == _native.FAILED_PRECONDITION
  assert host_op(s, 1, [2, 2]) == _native.INVALID_ARGUMENT
  assert host_op(s, 0, [1, 3]) == 0 and s.stats()["host_free"] == 5


def test_allocator_replays_reference_scripts():
  """Every answer the reference's LogicalBlockManager gave (status code,
  allocated ids in order, state counts), from the product and the oracle."""
  g = json.loads((Path(__file__).resolve().parent / "golden" / "block_manager.json").read_text())
  ops_code = {"dealloc": 0, "target": 1, "unlock": 2, "access": 3}
  n_ops = 0
  for sc in g["scripts"]:
    n = sc["blocks"]
    s = KVCacheStore(capacity=4, host_blocks=n)
    o = obm.LogicalBlockManager(n)
    for line, want in sc["ops"]:
      op, *args = line.split()
      vals = [int(a) for a in args]
      if op == "alloc":
        rc, ids = alloc(s, vals[0], bool(vals[1]))
        got = f"{rc} " + (" ".join(str(int(i)) for i in ids) if rc == 0 else "-")
        code, oids = o.allocate(vals[0], bool(vals[1]))
        ogot = f"{code} " + (" ".join(map(str, oids)) if code == 0 else "-")
      elif op == "stats":
        st = s.stats()
        got = f"{st['host_free']} {n - st['host_free']} {st['host_locked']}"
        ogot = f"{o.num_free()} {n - o.num_free()} {o.num_locked()}"
      else:
        got = str(host_op(s, ops_code[op], vals))
        fn = {"dealloc": o.deallocate, "target": o.allocate_target, "unlock": o.unlock,
              "access": lambda v: o.access(v[0])}[op]
        ogot = str(fn(vals))
      assert got == want, (line, got, want)
      assert ogot == want, (line, ogot, want)
      n_ops += 1
  assert n_ops >= 3000


@pytest.mark.parametrize("seed", range(5))
def test_allocator_matches_oracle_random(seed):
  rng = np.random.default_rng(seed)
  n = int(rng.integers(3, 40))
  s = KVCacheStore(capacity=4, host_blocks=n)
  o = obm.LogicalBlockManager(n)
  for _ in range(400):
    op = rng.integers(0, 5)
    if op == 0:
      k, lock = int(rng.integers(-1, n + 2)), bool(rng.integers(0, 2))
      code, ids = o.allocate(k, lock)
      rc, got = alloc(s, k, lock)
      assert rc == code and (ids is None or [int(x) for x in got] == ids)
    else:
      ids = [int(x) for x in rng.integers(-1, n + 1, int(rng.integers(1, 4)))]
      if op == 4:
        ids = ids[:1]
      code = [None, o.deallocate, o.allocate_target, o.unlock, lambda v: o.access(v[0])][op](ids)
      assert host_op(s, {1: 0, 2: 1, 3: 2, 4: 3}[op], ids) == code
    assert s.stats()["host_free"] == o.num_free()
    assert s.stats()["host_locked"] == o.num_locked()


def H(i):
  return f"hash-{i:04d}".encode()


def test_store_insert_save_poll_lookup_load_flow():
  s = KVCacheStore(capacity=8, host_blocks=8)
  hs = [H(i) for i in range(3)]
  slices = [RaidenBlockId(host_block_id=-1, device_block_id=10 + i, status=BlockStatus.HBM)
            for i in range(3)]
  assert s.insert(hs, slices, on_host=False)
  assert [s.get_pin_count(h) for h in hs] == [1, 1, 1]
  assert s.save(hs)
  done, failed, pending, existing, unregistered = s.poll_save_status()
  assert done == hs and failed == [] and pending == [] and existing == [] == unregistered
  assert [s.get_pin_count(h) for h in hs] == [0, 0, 0]     # save spent the insert pin
  found = s.lookup(hs + [H(99)] + [H(0)])
  assert [f[0] for f in found] == hs                      # answer ends at the first miss
  assert all(f[1].status == BlockStatus.HOST_AND_HBM for f in found)
  assert [f[1].host_block_id for f in found] == [0, 1, 2]  # free ids in order
  assert s.get_pin_count(H(0)) == 1                        # the hit past the miss was unpinned
  assert s.load(hs, [40, 41, 42])
  done, failed, pending = s.poll_load_status()
  assert done == hs and failed == [] == pending
  got = s.lookup(hs, pin_found=False)
  assert [g[1].device_block_id for g in got] == [40, 41, 42]
  assert [s.get_pin_count(h) for h in hs] == [0, 0, 0]


def test_store_preconditions():
  s = KVCacheStore(capacity=8, host_blocks=8)
  assert not s.save([H(1)]) and "Block hash not found" in s.last_error
  s.insert([H(1)], [RaidenBlockId(device_block_id=3, status=BlockStatus.HBM)])
  s.release([H(1)])
  assert not s.save([H(1)]) and "Block is not pinned" in s.last_error
  s.insert([H(2)], [RaidenBlockId(device_block_id=-1, status=BlockStatus.HBM)])
  assert not s.save([H(2)]) and "device_block_id is -1" in s.last_error
  s.insert([H(3)], [RaidenBlockId(host_block_id=1, status=BlockStatus.HOST)])
  assert not s.save([H(3)]) and "not in HBM status" in s.last_error
  assert not s.load([H(2)], [0]) and "not on host" in s.last_error
  with pytest.raises(ValueError):
    s.load([H(3)], [0, 1])
  with pytest.raises(ValueError):
    s.insert([H(4)], [RaidenBlockId(status=BlockStatus.REMOTE)])


def test_store_insert_all_or_nothing_and_drop_evict():
  s = KVCacheStore(capacity=4, host_blocks=4)
  hs = [H(i) for i in range(4)]
  assert s.insert(hs, [RaidenBlockId(device_block_id=i, status=BlockStatus.HBM)
                       for i in range(4)])
  # everything pinned: no room for a fifth entry, nothing changes
  assert not s.insert([H(9)], [RaidenBlockId(device_block_id=9, status=BlockStatus.HBM)])
  assert s.stats()["size"] == 4
  assert s.save(hs[:2]) and s.save(hs[2:])
  s.poll_save_status()
  # host tier full (4 ids used); a new save evicts the LRU host-resident entries
  assert s.insert([H(5), H(6)], [RaidenBlockId(device_block_id=5, status=BlockStatus.HBM),
                                 RaidenBlockId(device_block_id=6, status=BlockStatus.HBM)])
  assert s.save([H(5), H(6)])
  s.poll_save_status()
  got = dict((h, b) for h, b in s.lookup([H(5), H(6)], pin_found=False))
  assert sorted(b.host_block_id for b in got.values()) == [0, 1]  # ids of the evicted saves
  assert s.lookup([H(0)], pin_found=False) == []


def test_store_concurrent_callers_keep_invariants():
  """Threads insert, look up, release and evict their own keys through one
  store at once (the native calls run without the GIL); afterwards no pin is
  left, every host block is accounted for and the index holds each thread's
  surviving keys."""
  import threading
  s = KVCacheStore(capacity=256, host_blocks=512)
  errors = []

  def worker(t):
    try:
      rng = np.random.default_rng(t)
      for r in range(200):
        keys = [f"t{t}-{int(k)}".encode() for k in rng.integers(0, 40, 4)]
        keys = list(dict.fromkeys(keys))
        hosts = [RaidenBlockId(host_block_id=t * 64 + int(rng.integers(0, 64)),
                               status=BlockStatus.HOST) for _ in keys]
        if s.insert(keys, hosts, on_host=True):
          s.release(keys)
        found = s.lookup(keys)
        s.release([h for h, _ in found])
        if r % 7 == 0:
          s.evict(keys[:1])
    except Exception as e:
      errors.append(e)

  threads = [threading.Thread(target=worker, args=(t,)) for t in range(8)]
  for th in threads:
    th.start()
  for th in threads:
    th.join()
  assert not errors, errors
  keys = [f"t{t}-{k}".encode() for t in range(8) for k in range(40)]
  assert all(s.get_pin_count(k) == 0 for k in keys)
  st = s.stats()
  assert st["size"] <= 256 + 512 and st["available"] == 256


def test_remote_surface_refuses_without_registry():
  """read_remote / poll_remote_read_status and the address properties exist
  (api/torch/kv_cache_store.py:260-272, :536-596); remote reads need a global
  registry, so they are refused."""
  s = KVCacheStore(capacity=4, host_blocks=4)
  assert s.raiden_controller_address == "" and s.store_server_address == ""
  assert not s.read_remote([b"a"], [RaidenBlockId(status=BlockStatus.REMOTE)], [0])
  assert "global registry" in s.last_error
  assert s.poll_remote_read_status() == ([], [], [])
  with pytest.raises(ValueError):
    s.read_remote([b"a", b"b"], [RaidenBlockId()], [0])


def _same_streams(ref, prod):
  assert len(ref) == len(prod)
  for i, ((rs, rl), (ps, pl)) in enumerate(zip(ref, prod)):
    assert rs == [tuple(x) for x in ps], f"saves of access batch {i} differ"
    assert rl == [tuple(x) for x in pl], f"loads of access batch {i} differ"


def test_c1_trace_decisions_match_reference_store():
  """The whole C1 access trace (bench seed 10, 32768-block tier and pool,
  512-access batches): every save's (device, host) ids and every load's
  (host, device) ids equal those of the reference's LRUCache and
  LogicalBlockManager composed as KVCacheStore's local paths
  (oracle/_ref/store_trace_ref).  bench.py's CPU reference arm takes its
  block lists from that binary, the product arm from the product store."""
  from oracle import store_trace as ost
  from tpu_sync_b200 import workloads
  if build_ref.build_store_trace() is None:
    pytest.skip("reference checkout not available to build the store trace oracle")
  trace = ost.zipf_trace(seed=10)
  assert np.array_equal(trace, workloads.zipf_trace(seed=10))
  ref, ref_stats = ost.transfer_streams(trace, 32768, 32768, 512)
  prod, prod_stats = workloads.store_transfer_streams(trace, 32768, 32768, 512)
  assert ref_stats == prod_stats
  _same_streams(ref, prod)


@pytest.mark.parametrize("seed,host_blocks,pool,batch,n", [
    (10, 4096, 32768, 512, 100_000), (11, 1024, 2048, 256, 30_000),
    (12, 300, 512, 128, 20_000), (13, 2000, 1000, 512, 30_000)])
def test_trace_decisions_under_eviction_match_reference_store(seed, host_blocks, pool, batch, n):
  """Tiers smaller than the trace's working set: saves drop-evict unpinned
  host entries (candidates first, then the LRU end) and reuse their ids in
  the allocator's order; loads pinned by lookup survive the same batch's
  saves, and completions only take effect when polled."""
  from oracle import store_trace as ost
  from tpu_sync_b200 import workloads
  if build_ref.build_store_trace() is None:
    pytest.skip("reference checkout not available to build the store trace oracle")
  trace = ost.zipf_trace(n_access=n, seed=seed)
  ref, ref_stats = ost.transfer_streams(trace, host_blocks, pool, batch)
  prod, prod_stats = workloads.store_transfer_streams(trace, host_blocks, pool, batch)
  assert ref_stats == prod_stats
  _same_streams(ref, prod)


def test_bench_c1_exactness_model_matches_an_in_order_replay():
  """bench.py's full-size C1 check names, for every reloaded pool block, the
  pool block whose bytes it must hold (c1_seed_host_blocks /
  c1_expected_sources).  Replayed here call by call on a toy pool whose
  blocks hold their own ids (offloads of a step before its reloads, the
  last copy to a block winning, as the manager orders them), the same
  steps leave exactly those ids."""
  import sys
  from pathlib import Path
  sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
  import bench
  rng = np.random.default_rng(4)
  half, host_blocks, steps = 64, 96, 9
  plans = []
  for _ in range(steps):
    n_off, n_ld = int(rng.integers(0, 20)), int(rng.integers(1, 30))
    plans.append((rng.integers(0, half, n_off), rng.choice(host_blocks, n_off, replace=False),
                   rng.integers(0, host_blocks, n_ld), half + rng.integers(0, half, n_ld)))
  executed = list(range(steps)) + list(range(3, steps))
  seed = bench.c1_seed_host_blocks(plans, executed, half)
  dev = np.arange(2 * half)              # block d holds the bytes of block d
  host = np.full(host_blocks, -1)        # unknown content
  for h, d in seed.items():              # the untimed seeding offload
    host[h] = dev[d]
  for i in executed:
    off_d, off_h, ld_h, ld_d = plans[i]
    for d, h in zip(off_d, off_h):
      host[h] = dev[d]
    for h, d in zip(ld_h, ld_d):
      dev[d] = host[h]
  expected = bench.c1_expected_sources(plans, executed, seed)
  reloaded = {int(d) for i in executed for d in plans[i][3]}
  assert set(expected) == reloaded       # seeding leaves no reload unknown
  for d, s in expected.items():
    assert dev[d] == s, (d, s, dev[d])

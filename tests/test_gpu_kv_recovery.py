"""Crash restart of the tier-2 host cache on a GPU (warm boot).

The reference's recovery e2e (tpu_sync/api/jax/kv_cache_store_recovery_e2e_test.py)
on cuda:0, through the public construction path only (RAIDEN_SHM_KEY,
RAIDEN_SHM_MODEL_UID):

* phase A (a subprocess): a KVCacheManager whose host tier is a /dev/shm
  segment and a KVCacheStore whose metadata table is another one; HBM blocks
  of distinct bytes are inserted and saved, and once the saves completed (no
  GPU work in flight) the process dies by SIGKILL, so no destructor runs;
* phase B (a fresh subprocess, same environment): the same stack over a
  zeroed device pool.  The manager re-attaches the surviving data segment,
  the store rebuilds its index from the surviving table (HOST blocks at the
  same host ids), and loading them into other device blocks must restore
  phase A's bytes exactly;
* a restart under another model uid cold-starts: no hits.
"""

import os
import signal
import subprocess
import sys
import textwrap
import uuid
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]

_PHASE = textwrap.dedent("""
    import os, signal, sys, time
    sys.path.insert(0, {root!r})
    import numpy as np, torch
    from tpu_sync_b200 import KVCacheManager, workloads
    from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId
    phase, expect_path = sys.argv[1], sys.argv[2]
    dev = torch.device("cuda", 0)
    geom = workloads.KVGeometry(layers=2, kv=2, block_tokens=16, heads=8, head_dim=128)
    hs = [b"hash_0", b"hash_1", b"hash_2", b"hash_3"]

    def poll(fn, n):
      done, t0 = [], time.time()
      while len(done) < n and time.time() - t0 < 60:
        res = fn()
        assert not res[1], res[1]
        done += res[0]
      assert len(done) >= n, (phase, done)

    if phase == "a":
      pool = workloads.kv_pool(geom, 16, 11, dev)
    else:
      pool = [torch.zeros_like(t) for t in workloads.kv_pool(geom, 16, 11, dev)]
    mgr = KVCacheManager([[t] for t in pool], host_blocks_to_allocate=8)
    store = KVCacheStore(capacity=8, manager=mgr)
    if phase == "a":
      src = [3, 5, 7, 9]
      assert store.insert(hs, [RaidenBlockId(device_block_id=d, status=BlockStatus.HBM)
                               for d in src], False)
      assert store.save(hs)
      poll(store.poll_save_status, 4)
      got = store.lookup(hs, pin_found=False)
      assert [(int(b.status), b.host_block_id) for _, b in got] == \\
          [(int(BlockStatus.HOST_AND_HBM), i) for i in range(4)], got
      torch.cuda.synchronize()
      np.save(expect_path, np.stack([np.stack([t[d].view(torch.uint8).cpu().numpy()
                                               for t in pool]) for d in src]))
      print("PHASE_A_SAVED", flush=True)
      os.kill(os.getpid(), signal.SIGKILL)
    got = store.lookup(hs)
    if phase == "b_cold":
      assert got == [] and store.recovered_blocks == 0, got
      print("PHASE_B_COLD", flush=True)
      sys.exit(0)
    assert store.recovered_blocks == 4
    assert [(h, int(b.status), b.host_block_id) for h, b in got] == \\
        [(h, int(BlockStatus.HOST), i) for i, h in enumerate(hs)], got
    print("PHASE_B_RECOVERED", flush=True)
    dst = [0, 1, 12, 15]
    assert store.load(hs, dst)
    poll(store.poll_load_status, 4)
    torch.cuda.synchronize()
    want = np.load(expect_path)
    for k, d in enumerate(dst):
      for l, t in enumerate(pool):
        np.testing.assert_array_equal(t[d].view(torch.uint8).cpu().numpy(), want[k, l])
    print("PHASE_B_BYTES_MATCH", flush=True)
""")


def _run(phase, key, uid, expect):
  env = dict(os.environ, RAIDEN_SHM_KEY=key, RAIDEN_SHM_MODEL_UID=uid)
  return subprocess.run([sys.executable, "-c", _PHASE.format(root=str(ROOT)), phase,
                         str(expect)], env=env, capture_output=True, text=True, timeout=300)


def _cleanup(key):
  for name in os.listdir("/dev/shm"):
    if name.startswith(key):
      try:
        os.unlink(os.path.join("/dev/shm", name))
      except OSError:
        pass


@pytest.fixture
def shm_key():
  key = f"tsb_recovery_{os.getpid()}_{uuid.uuid4().hex[:8]}"
  yield key
  _cleanup(key)


def test_recovers_saved_blocks_after_crash(cuda, shm_key, tmp_path):
  expect = tmp_path / "expect.npy"
  a = _run("a", shm_key, "recovery_model", expect)
  assert a.returncode == -signal.SIGKILL, a.stderr[-4000:]
  assert "PHASE_A_SAVED" in a.stdout
  names = sorted(os.listdir("/dev/shm"))
  assert f"{shm_key}_dev_0" in names and f"{shm_key}_metadata" in names
  b = _run("b", shm_key, "recovery_model", expect)
  assert b.returncode == 0, b.stderr[-4000:]
  assert "PHASE_B_RECOVERED" in b.stdout and "PHASE_B_BYTES_MATCH" in b.stdout


def test_model_uid_mismatch_cold_starts(cuda, shm_key, tmp_path):
  expect = tmp_path / "expect.npy"
  a = _run("a", shm_key, "recovery_model", expect)
  assert a.returncode == -signal.SIGKILL, a.stderr[-4000:]
  c = _run("b_cold", shm_key, "another_model", expect)
  assert c.returncode == 0, c.stderr[-4000:]
  assert "PHASE_B_COLD" in c.stdout

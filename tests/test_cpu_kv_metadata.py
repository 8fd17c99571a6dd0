"""KV metadata table and crash recovery on the CPU.

* the oracle (oracle/kv_metadata.py) and the product (tpu_sync_b200.kv_metadata
  over the C ABI) replay the command scripts of tests/golden/kv_metadata.json
  and must give the reference's answers (statuses with code and message,
  entries, table bytes; the header's padding bytes excepted);
* with the reference's own kv_cache_metadata.cc built (oracle/_ref/meta_ref):
  fresh random scripts on both sides, and /dev/shm tables written by one
  side and attached by the other (AttachOrFormat warm / cold);
* the store's metadata hooks and RecoverFromLocalManifest against the
  reference's kv_cache_store_test.cc cases (:901-965, :3170-3365);
* a crash-restart through the public construction path (RAIDEN_SHM_KEY):
  one process records host-resident blocks and dies by SIGKILL, the next
  rebuilds its index from the surviving table.
"""

import ctypes
import os
import random
import signal
import subprocess
import sys
import textwrap
import uuid
from pathlib import Path

import numpy as np
import pytest

from oracle import kv_metadata as okm
from oracle import ref_meta
from tpu_sync_b200 import _native
from tpu_sync_b200 import kv_metadata as km
from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = __import__("json").loads((ROOT / "tests" / "golden" / "kv_metadata.json").read_text())
PAD = slice(84, 128)


def _hex(b):
  return b.hex() if b else "-"


def _unhex(s):
  return b"" if s == "-" else bytes.fromhex(s)


def _masked(lines):
  out = []
  for line in lines:
    if line.startswith("bytes "):
      b = bytearray.fromhex(line[6:])
      b[PAD] = bytes(PAD.stop - PAD.start)
      line = "bytes " + b.hex()
    out.append(line)
  return out


def _status_line(code, msg):
  return "ok" if code == 0 else f"err {code} {msg}"


def replay_oracle(script):
  """The oracle restatement over a bytearray (address 0 is 64-aligned)."""
  buf, table, out = bytearray(), None, []
  for line in script:
    a = line.split(" ")
    if a[0] == "region":
      buf = bytearray(int(a[1]))
      out.append("ok")
    elif a[0] == "poke":
      d = bytes.fromhex(a[2])
      buf[int(a[1]):int(a[1]) + len(d)] = d
      out.append("ok")
    elif a[0] == "dump":
      out.append("bytes " + bytes(buf).hex())
    elif a[0] in ("format", "attach"):
      nb, uid = int(a[1]), _unhex(a[2])
      off, size, mod = 0, len(buf), 0
      if len(a) > 3:
        if a[3] == "null":
          size, mod = 0, None
        else:
          off = min(int(a[3]), len(buf))
          size, mod = min(int(a[4]), len(buf) - off), off % 64
      fn = okm.format_table if a[0] == "format" else okm.attach_table
      st, t = fn(buf, off, size, mod, nb, uid)
      if t is not None:
        table = t
      out.append(_status_line(*st))
    elif a[0] == "set":
      out.append(_status_line(*table.set(int(a[1]), _unhex(a[2]), int(a[3]))))
    elif a[0] == "clear":
      out.append(_status_line(*table.clear(int(a[1]))))
    elif a[0] == "entries":
      out += [f"entry {i} {_hex(h)} {s}" for i, h, s in table.valid_entries()] + ["end"]
  return out


def replay_product(script):
  """The product through its C ABI on a 64-byte aligned numpy region."""
  lib = _native.lib()
  buf, meta, out = None, None, []

  def status(rc):
    return "ok" if rc == 0 else f"err {rc} {_native.last_error()}"

  for line in script:
    a = line.split(" ")
    if a[0] == "region":
      n = int(a[1])
      raw = np.zeros(n + 64, np.uint8)
      o = (-raw.ctypes.data) % 64
      buf = raw[o:o + n]
      out.append("ok")
    elif a[0] == "poke":
      d = np.frombuffer(bytes.fromhex(a[2]), np.uint8)
      buf[int(a[1]):int(a[1]) + d.size] = d
      out.append("ok")
    elif a[0] == "dump":
      out.append("bytes " + buf.tobytes().hex())
    elif a[0] in ("format", "attach"):
      nb, uid = int(a[1]), _unhex(a[2])
      ptr, size = buf.ctypes.data, buf.nbytes
      if len(a) > 3:
        if a[3] == "null":
          ptr, size = None, 0
        else:
          off = min(int(a[3]), buf.nbytes)
          ptr, size = buf.ctypes.data + off, min(int(a[4]), buf.nbytes - off)
      h = ctypes.c_void_p()
      rc = lib.ts_kv_metadata_on_region(ptr, size, nb, uid, int(a[0] == "attach"),
                                        ctypes.byref(h))
      if rc == 0:
        meta = km.KVCacheMetadata(h, owner=buf)
      out.append(status(rc))
    elif a[0] == "set":
      h = _unhex(a[2])
      out.append(status(lib.ts_kv_metadata_set(meta._h, int(a[1]), h, len(h), int(a[3]))))
    elif a[0] == "clear":
      out.append(status(lib.ts_kv_metadata_clear(meta._h, int(a[1]))))
    elif a[0] == "entries":
      out += [f"entry {e.block_id} {_hex(e.hash)} {e.seq}" for e in meta.valid_entries()]
      out.append("end")
  return out


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=lambda c: c["name"])
def test_oracle_replays_reference_answers(case):
  assert _masked(replay_oracle(case["script"])) == case["out"]


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=lambda c: c["name"])
def test_product_replays_reference_answers(case):
  assert _masked(replay_product(case["script"])) == case["out"]


def test_product_zeroes_header_padding():
  r = km.aligned_region(3)
  r[:] = 0xAB
  km.KVCacheMetadata.format(r, 3, "uid")
  assert not r[PAD].any()
  assert r[:8].tobytes() == b"MKNEDIAR"  # 0x52414944454E4B4D little-endian


needs_ref = pytest.mark.skipif(ref_meta.binary() is None,
                               reason="reference checkout not present (meta_ref not built)")


@needs_ref
def test_product_matches_reference_on_fresh_random_scripts():
  rng = random.Random(77)
  for _ in range(60):
    script = ref_meta.random_script(rng)
    want = _masked(ref_meta.run(script))
    assert _masked(replay_product(script)) == want
    assert _masked(replay_oracle(script)) == want


def _shm_key():
  return f"tsb_meta_test_{os.getpid()}_{uuid.uuid4().hex[:8]}"


def _unlink(key):
  p = Path("/dev/shm") / key.lstrip("/")
  if p.exists():
    p.unlink()


@needs_ref
def test_shm_tables_interoperate_with_reference():
  key = _shm_key()
  try:
    # reference formats and records; the product attaches warm and sees it
    out = ref_meta.run([f"shm {key} 6 {_hex(b'model_x')}", "set 2 6162 5",
                        f"set 4 {_hex(b'h4')} 9", "clear 2", f"set 5 {_hex(b'h5')} 3"])
    assert out[0] == "ok warm=0"
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 6, "model_x")
    assert reg.warm
    assert reg.metadata.valid_entries() == [km.Entry(4, b"h4", 9), km.Entry(5, b"h5", 3)]
    reg.metadata.set(0, b"\x00prod", 11)
    reg.metadata.clear(5)
    reg.close()
    # the reference re-attaches the product's writes warm
    out = ref_meta.run([f"shm {key} 6 {_hex(b'model_x')}", "entries"])
    assert out[0] == "ok warm=1"
    assert ref_meta.parse_entries(out, 1)[0] == [(0, b"\x00prod", 11), (4, b"h4", 9)]
    # another model (either side) cold-starts over an empty table
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 6, "model_y")
    assert not reg.warm and reg.metadata.valid_entries() == []
    reg.metadata.set(1, b"y", 1)
    reg.close()
    out = ref_meta.run([f"shm {key} 6 {_hex(b'model_y')}", "entries"])
    assert out[0] == "ok warm=1" and ref_meta.parse_entries(out, 1)[0] == [(1, b"y", 1)]
    out = ref_meta.run([f"shm {key} 7 {_hex(b'model_y')}", "entries"])  # resized pool
    assert out[0] == "ok warm=0"
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 7, "model_y")
    assert reg.warm and reg.metadata.valid_entries() == []
    reg.reformat()
    assert not reg.warm
    reg.close(unlink=True)
    assert not (Path("/dev/shm") / key).exists()
  finally:
    _unlink(key)


def test_shm_region_key_and_errors():
  key = _shm_key()
  try:
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 4)
    assert reg.key == "/" + key and not reg.warm
    size = (Path("/dev/shm") / key).stat().st_size
    assert size == 4096  # 128 + 4 * 128 rounded up to a page
    reg.close()
    with pytest.raises(ValueError, match="num_blocks must be positive, got 0"):
      km.KVCacheMetadataShmRegion.attach_or_format(key, 0)
    with pytest.raises(ValueError, match="model_uid length 64 exceeds the maximum of 63"):
      km.KVCacheMetadataShmRegion.attach_or_format(key, 4, "u" * 64)
  finally:
    _unlink(key)


def test_metadata_shm_key_from_environment():
  assert km.metadata_shm_key({}) == ""
  assert km.metadata_shm_key({"RAIDEN_SHM_KEY": "kv"}) == "kv_metadata"
  assert km.metadata_shm_key({"RAIDEN_SHM_KEY": "kv", "RAIDEN_SHM_SERVER_NAME": "s1"}) == \
      "kv_metadata_s1"
  assert km.model_uid_from_env({}) == "default_model"
  assert km.model_uid_from_env({"RAIDEN_SHM_MODEL_UID": ""}) == ""


# -- the store's hooks and recovery (kv_cache_store_test.cc) ------------------

def _table(n):
  return km.KVCacheMetadata.format(km.aligned_region(n), n)


def _host(i):
  return RaidenBlockId(host_block_id=i, status=BlockStatus.HOST)


def _insert_resident(store, hashes, slices, on_host=True):
  ok = store.insert(hashes, slices, on_host)
  if ok:
    store.release(hashes)
  return ok


def E(*a):
  return km.Entry(*a)


def _alloc(store, n):
  """The allocator test hook: n locked host blocks, lowest free ids first."""
  out = np.zeros(n, np.int32)
  _native.check(_native.lib().ts_store_allocate_host_blocks(
      store._impl, n, 1, out.ctypes.data_as(_native.c_i32_p)))
  return [int(x) for x in out]


def test_metadata_keeps_eviction_candidates():
  """MetadataKeepsEvictionCandidates (kv_cache_store_test.cc:901-944)."""
  meta = _table(4)
  store = KVCacheStore(2, host_blocks=4, metadata=meta)
  assert _insert_resident(store, [b"host_1", b"host_2"], [_host(0), _host(1)])
  assert _insert_resident(store, [b"host_3"], [_host(2)])
  assert store.candidate_order() == [b"host_2"]
  assert meta.valid_entries() == [E(0, b"host_1", 1), E(1, b"host_2", 0), E(2, b"host_3", 2)]
  assert _insert_resident(store, [b"host_2"], [_host(3)])
  assert store.candidate_order() == []
  assert meta.valid_entries() == [E(0, b"host_1", 1), E(2, b"host_3", 2), E(3, b"host_2", 3)]


def test_evict_clears_metadata_entries():
  """EvictClearsMetadataEntries (kv_cache_store_test.cc:946-965)."""
  meta = _table(2)
  store = KVCacheStore(2, host_blocks=2, metadata=meta)
  assert _insert_resident(store, [b"host_1", b"host_2"], [_host(0), _host(1)])
  assert len(meta.valid_entries()) == 2
  assert store.evict([b"host_1"]) == 1
  assert meta.valid_entries() == [E(1, b"host_2", 0)]


def test_save_completion_records_host_blocks():
  """The HBM-insert-then-save case (kv_cache_store_test.cc:3170-3208): HBM
  slices leave the table empty; save completion binds host blocks 0 and 1."""
  meta = _table(10)
  store = KVCacheStore(10, host_blocks=10, metadata=meta)
  hashes = [b"hash_1", b"hash_2"]
  slices = [RaidenBlockId(device_block_id=i, status=BlockStatus.HBM) for i in range(2)]
  assert _insert_resident(store, hashes, slices, on_host=False)
  assert len(store.lookup(hashes)) == 2
  assert meta.valid_entries() == []
  assert store.save(hashes)
  done = store.poll_save_status()[0]
  assert sorted(done) == sorted(hashes)
  assert meta.valid_entries() == [E(0, b"hash_1", 0), E(1, b"hash_2", 1)]


def test_recover_rebuilds_lru_cache():
  """RecoverFromLocalManifestRebuildsLruCache (kv_cache_store_test.cc:3211-3255)."""
  meta = _table(10)
  meta.set(5, b"hash_b", 3)
  meta.set(7, b"hash_a", 4)
  meta.set(9, b"hash_c", 8)
  store = KVCacheStore(10, host_blocks=10, metadata=meta)
  assert store.recover_from_local_manifest() == 3
  got = store.lookup([b"hash_a", b"hash_b", b"hash_c"], pin_found=False)
  assert [(b.status, b.host_block_id) for _, b in got] == \
      [(BlockStatus.HOST, 7), (BlockStatus.HOST, 5), (BlockStatus.HOST, 9)]
  stats = store.stats()
  assert stats["host_free"] == 7 and stats["host_locked"] == 3
  assert _insert_resident(store, [b"hash_d"], [_host(0)])
  assert meta.valid_entries() == [E(0, b"hash_d", 9), E(5, b"hash_b", 3), E(7, b"hash_a", 4),
                                  E(9, b"hash_c", 8)]


def test_recover_rebuilds_lru_order():
  """RecoverFromLocalManifestRebuildsLruOrder (kv_cache_store_test.cc:3257-3280)."""
  meta = _table(10)
  meta.set(5, b"hash_b", 3)
  meta.set(7, b"hash_a", 4)
  meta.set(9, b"hash_c", 8)
  store = KVCacheStore(2, host_blocks=10, metadata=meta)
  assert store.recover_from_local_manifest() == 3
  assert store.candidate_order() == [b"hash_b"]
  assert len(meta.valid_entries()) == 3


def test_recover_keeps_newest_duplicate():
  """RecoverFromLocalManifestKeepsNewestDuplicate (kv_cache_store_test.cc:3282-3316)."""
  meta = _table(10)
  meta.set(2, b"dup_hash", 1)
  meta.set(4, b"other", 3)
  meta.set(6, b"dup_hash", 5)
  store = KVCacheStore(10, host_blocks=10, metadata=meta)
  assert store.recover_from_local_manifest() == 2
  got = store.lookup([b"dup_hash"], pin_found=False)
  assert got[0][1].host_block_id == 6
  # the stale block 2 is not allocated: it is handed out after 0 and 1
  assert _alloc(store, 3) == [0, 1, 2]
  assert meta.valid_entries() == [E(4, b"other", 3), E(6, b"dup_hash", 5)]


def test_recover_fails_cleanly_on_allocator_conflict():
  """RecoverFromLocalManifestFailsOnAllocatorConflict (kv_cache_store_test.cc:3318-3337)."""
  meta = _table(10)
  meta.set(0, b"rh1", 0)
  store = KVCacheStore(10, host_blocks=10, metadata=meta)
  assert _alloc(store, 1) == [0]
  with pytest.raises(_native.NativeError) as ei:
    store.recover_from_local_manifest()
  assert ei.value.status == "FAILED_PRECONDITION"
  assert store.lookup([b"rh1"]) == []
  assert len(meta.valid_entries()) == 1


def test_recover_preconditions():
  """RecoverFromLocalManifestPreconditions (kv_cache_store_test.cc:3339-3372)."""
  store = KVCacheStore(10, host_blocks=10)
  with pytest.raises(_native.NativeError, match="KVCacheMetadata is required"):
    store.recover_from_local_manifest()
  meta = _table(10)
  store = KVCacheStore(10, host_blocks=10, metadata=meta)
  assert _insert_resident(store, [b"hash_a"], [_host(0)])
  with pytest.raises(_native.NativeError, match="empty cache store"):
    store.recover_from_local_manifest()
  store = KVCacheStore(10, host_blocks=10, metadata=_table(10))
  assert store.recover_from_local_manifest() == 0


def test_rollback_and_replaced_hbm_binding_clear_entries():
  """Insert's rollback (host_offload_backend.cc:458-470) and the replaced HBM
  binding path (:395-409) keep the table in step with the index."""
  meta = _table(4)
  store = KVCacheStore(1, host_blocks=4, metadata=meta)
  assert store.insert([b"a"], [_host(0)], True)  # pinned: capacity 1 is full
  assert not store.insert([b"b"], [_host(1)], True)  # no space: nothing recorded
  assert meta.valid_entries() == [E(0, b"a", 0)]
  store.release([b"a"])
  assert store.evict([b"a"]) == 1
  assert meta.valid_entries() == []


# -- crash restart through the public construction path -----------------------

_PHASE = textwrap.dedent("""
    import os, signal, sys
    sys.path.insert(0, {root!r})
    from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId
    phase = sys.argv[1]
    store = KVCacheStore(4, host_blocks=4)
    if phase == "a":
      hs = [b"hash_0", b"hash_1", b"hash_2"]
      assert store.insert(hs, [RaidenBlockId(device_block_id=i, status=BlockStatus.HBM)
                               for i in range(3)], False)
      store.release(hs)
      assert store.lookup(hs)
      assert store.save(hs)
      assert sorted(store.poll_save_status()[0]) == sorted(hs)
      print("PHASE_A_SAVED", flush=True)
      os.kill(os.getpid(), signal.SIGKILL)
    got = store.lookup([b"hash_0", b"hash_1", b"hash_2"], pin_found=False)
    print("RECOVERED", store.recovered_blocks,
          [(h.decode(), int(b.status), b.host_block_id) for h, b in got], flush=True)
""")


def _run_phase(phase, key, uid):
  env = dict(os.environ, RAIDEN_SHM_KEY=key, RAIDEN_SHM_MODEL_UID=uid)
  return subprocess.run([sys.executable, "-c", _PHASE.format(root=str(ROOT)), phase],
                        env=env, capture_output=True, text=True, timeout=120)


def test_crash_restart_recovers_host_index():
  """The recovery e2e (tpu_sync/api/jax/kv_cache_store_recovery_e2e_test.py)
  for the index: phase A dies by SIGKILL after its saves complete; phase B
  (same environment) finds the blocks HOST-resident at the same host ids; a
  restart under another model uid cold-starts."""
  key = _shm_key()
  try:
    a = _run_phase("a", key, "recovery_model")
    assert a.returncode == -signal.SIGKILL, a.stderr[-2000:]
    assert "PHASE_A_SAVED" in a.stdout
    b = _run_phase("b", key, "recovery_model")
    assert b.returncode == 0, b.stderr[-2000:]
    assert ("RECOVERED 3 [('hash_0', 3, 0), ('hash_1', 3, 1), ('hash_2', 3, 2)]"
            in b.stdout), b.stdout
    # another model's restart must not resurrect the table: it is re-created
    # empty, so a later restart of the first model finds nothing either
    for uid in ("another_model", "recovery_model"):
      c = _run_phase("b", key, uid)
      assert c.returncode == 0, c.stderr[-2000:]
      assert "RECOVERED 0 []" in c.stdout, c.stdout
  finally:
    _unlink(key + "_metadata")


def test_store_keeps_a_dropped_region_mapped():
  """A store holding a shm table keeps it mapped after the caller dropped
  the region object (the table handle owns the mapping)."""
  import gc
  key = _shm_key()
  try:
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 4, "m")
    store = KVCacheStore(4, host_blocks=4, metadata=reg.metadata)
    del reg
    gc.collect()
    assert _insert_resident(store, [b"k"], [_host(2)])
    store.close()
    reg = km.KVCacheMetadataShmRegion.attach_or_format(key, 4, "m")
    assert reg.warm and reg.metadata.valid_entries() == [E(2, b"k", 0)]
    reg.close()
  finally:
    _unlink(key)

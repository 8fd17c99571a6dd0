"""CPU tests of the native library: it loads, exports every declared symbol,
and its pure host logic (copy-spec validation, run coalescing) matches the
oracle restatement of the reference on the reference's own cases and on
random ones."""

import re

import numpy as np
import pytest

from oracle import kv_blocks as ref
from tpu_sync_b200 import _native

HEADER = _native.LIB_PATH.parents[2] / "include" / "tpusync_b200.h"


def declared_in_header():
  text = HEADER.read_text()
  return sorted(set(re.findall(r"^TS_API\s+[\w\s\*]+?\b(ts_\w+)\(", text, flags=re.M)))


def test_library_exports_every_declared_symbol():
  lib = _native.lib()
  names = declared_in_header()
  assert len(names) >= 20
  for name in names:
    assert hasattr(lib, name), name
  # the ctypes table covers exactly the header
  assert names == _native.declared_symbols()
  assert b"sm_100a" in lib.ts_version()


def validate(src, dst, sizes):
  s, d, z = (_native.i64_array(x) for x in (src, dst, sizes))
  rc = _native.lib().ts_validate_copy_spec(_native.i64_ptr(s), s.size, _native.i64_ptr(d),
                                           d.size, _native.i64_ptr(z), z.size)
  return rc, (_native.last_error() if rc else "")


# Cases of tpu_sync/kv_cache/kv_cache_manager_test.cc:579-606 plus edge cases.
@pytest.mark.parametrize("src,dst,sizes", [
    ([0], [0, 1], [1]),          # D2hFailsWithMismatchedCopySpecLengths
    ([-1], [0], [1]),            # H2dFailsWithNegativeOffsets
    ([0], [0], [-1]),
    ([0, 1], [0, -5], [1, 1]),
    ([0, 1], [2, 3], [1]),
    ([], [], []),
    ([3], [], []),
    ([1, 2, 3], [4, 5, 6], [1, 1, 1]),
])
def test_validate_matches_reference(src, dst, sizes):
  code, msg = ref.validate_offsets_and_sizes(src, dst, sizes)
  rc, err = validate(src, dst, sizes)
  assert rc == code
  assert err == msg


def coalesce(src, dst, sizes):
  s, d, z = (_native.i64_array(x) for x in (src, dst, sizes))
  n = s.size
  os_, od, on = (np.zeros(max(n, 1), np.int64) for _ in range(3))
  m = np.zeros(1, np.int64)
  rc = _native.lib().ts_coalesce_runs(_native.i64_ptr(s), _native.i64_ptr(d),
                                      _native.i64_ptr(z), n, _native.i64_ptr(os_),
                                      _native.i64_ptr(od), _native.i64_ptr(on),
                                      _native.i64_ptr(m))
  assert rc == 0
  k = int(m[0])
  return list(os_[:k]), list(od[:k]), list(on[:k])


def test_coalesce_matches_reference_random():
  rng = np.random.default_rng(7)
  for _ in range(300):
    n = int(rng.integers(0, 40))
    # mix of consecutive runs and jumps
    src = np.cumsum(rng.integers(0, 3, n)) + rng.integers(0, 5)
    dst = np.cumsum(rng.integers(0, 3, n)) + rng.integers(0, 5)
    sizes = rng.integers(0, 3, n)
    assert coalesce(src, dst, sizes) == ref.coalesce_major_dim_copies(src, dst, sizes)


def test_coalesce_examples():
  # a run of N consecutive 1-block copies becomes one N-block copy
  assert coalesce([4, 5, 6], [0, 1, 2], [1, 1, 1]) == ([4], [0], [3])
  assert coalesce([0, 2], [0, 1], [1, 1]) == ([0, 2], [0, 1], [1, 1])
  assert coalesce([0, 2], [0, 2], [2, 1]) == ([0], [0], [3])


def test_host_tier_anonymous_and_shm(tmp_path):
  import ctypes
  lib = _native.lib()
  t = ctypes.c_void_p()
  warm = ctypes.c_int()
  _native.check(lib.ts_host_tier_create(1 << 20, b"", b"", 0, 0, ctypes.byref(t),
                                        ctypes.byref(warm)))
  p = lib.ts_host_tier_ptr(t)
  assert p and lib.ts_host_tier_bytes(t) == 1 << 20
  ctypes.memset(p, 7, 1 << 20)
  lib.ts_host_tier_destroy(t, 0)
  name = f"tsb_test_{np.random.randint(1 << 30)}".encode()
  _native.check(lib.ts_host_tier_create(8192, name, b"model-a", 42, 0, ctypes.byref(t),
                                        ctypes.byref(warm)))
  assert warm.value == 0
  ctypes.memset(lib.ts_host_tier_ptr(t), 9, 8192)
  lib.ts_host_tier_destroy(t, 0)
  # same name, uid and geometry: warm attach keeps the payload
  _native.check(lib.ts_host_tier_create(8192, name, b"model-a", 42, 0, ctypes.byref(t),
                                        ctypes.byref(warm)))
  assert warm.value == 1
  assert ctypes.string_at(lib.ts_host_tier_ptr(t), 4) == b"\x09" * 4
  lib.ts_host_tier_destroy(t, 0)
  # different geometry: cold start
  _native.check(lib.ts_host_tier_create(8192, name, b"model-a", 43, 0, ctypes.byref(t),
                                        ctypes.byref(warm)))
  assert warm.value == 0
  lib.ts_host_tier_destroy(t, 1)


def test_pci_numa_node_reads_sysfs(tmp_path):
  """ts_pci_numa_node: the node sysfs lists for a PCI function, from CUDA's
  8-digit-domain bus id or sysfs's own form, case-insensitive; -1 when the
  device, or its node, is unknown (DetectAndAssignNumaNode keeps no node
  then, raiden_manager_base.cc:47-78)."""
  import ctypes
  dev = tmp_path / "bus" / "pci" / "devices"
  for bus, node in (("0000:1b:00.0", "1\n"), ("0000:9a:00.0", "-1\n"), ("0000:c3:00.0", "0")):
    (dev / bus).mkdir(parents=True)
    (dev / bus / "numa_node").write_text(node)
  root = str(tmp_path).encode()
  out = ctypes.c_int(7)
  for bus, want in ((b"00000000:1B:00.0", 1), (b"0000:1b:00.0", 1), (b"0000:9A:00.0", -1),
                    (b"00000000:C3:00.0", 0), (b"0000:ff:00.0", -1)):
    assert _native.lib().ts_pci_numa_node(bus, root, ctypes.byref(out)) == _native.OK
    assert out.value == want, bus
  assert _native.lib().ts_pci_numa_node(None, root, ctypes.byref(out)) == _native.INVALID_ARGUMENT


def test_numa_option_of_the_manager():
  from tpu_sync_b200.kv_cache_manager import _numa_opt
  assert _numa_opt(None) == 0 and _numa_opt("none") == -1
  assert _numa_opt(0) == 1 and _numa_opt(3) == 4
  with pytest.raises(ValueError):
    _numa_opt(-2)
  with pytest.raises(ValueError):
    _numa_opt("local")

"""GPU test of ts_kv_offload_noalloc, the offload entry point that allocates
no device memory (for callers whose HBM is already owned by their own
allocator or KV pool, where an extra cudaMalloc would fail, fragment it, or
synchronise the device).  It is checked through the C ABI against the
manager's offload (ts_d2h) on two calls in a row, bit-exact like every other
byte-movement test here.  The file name makes pytest collect it last."""

import ctypes

import numpy as np
import pytest
import torch

from tpu_sync_b200 import KVCacheManager, _native, ops, workloads

pytestmark = pytest.mark.gpu


def noalloc_offload(table, src, dst, host_buf, host_blocks, stream):
  s = _native.i64_array(src)
  d = _native.i64_array(dst)
  return _native.lib().ts_kv_offload_noalloc(
      table.device.index, ctypes.c_void_p(table.d_table.data_ptr()), table.n,
      _native.i64_ptr(s), _native.i64_ptr(d), s.size, ctypes.c_void_p(host_buf.data_ptr()),
      table.pitch, host_blocks, ctypes.c_void_p(stream.cuda_stream))


def test_noalloc_offload_matches_manager_twice(cuda):
  geom = workloads.KVGeometry(layers=4, kv=2, block_tokens=16, heads=8, head_dim=128)
  pool = workloads.kv_pool(geom, 96, 31, cuda)
  host_blocks = 48
  mgr = KVCacheManager([[t] for t in pool], host_blocks_to_allocate=host_blocks)
  table = ops.StorageTable(pool)
  assert table.pitch == mgr.host_block_pitch
  host_buf = torch.zeros((host_blocks, table.pitch), dtype=torch.uint8, pin_memory=True)
  stream = torch.cuda.current_stream(cuda)
  rng = np.random.default_rng(12)
  written = set()
  for call in range(2):  # two calls in a row; the second reuses the static staging
    n = 40 if call == 0 else 33
    src = rng.choice(96, n, replace=False)
    dst = rng.choice(host_blocks, n, replace=False)
    if call == 1:
      dst[:10] = np.arange(5, 15)  # a coalescible run of host ids
    mgr.d2h(src.tolist(), dst.tolist()).Await()
    rc = noalloc_offload(table, src, dst, host_buf, host_blocks, stream)
    assert rc == _native.OK, _native.last_error()
    stream.synchronize()
    written.update(int(h) for h in dst)
    hb = host_buf.numpy()
    for l in range(len(pool)):
      off, bb = table.stage_offs[l], table.block_bytes[l]
      for h in sorted(written):
        assert hb[h, off:off + bb].tobytes() == mgr.read_block_bytes(l, h), (call, l, h)
  mgr.close()


def test_noalloc_offload_rejects_oversized_blocks(cuda):
  # one 65 MiB block per storage cannot fit the 64 MiB static staging
  pool = [torch.zeros((1, 65 << 20), dtype=torch.uint8, device=cuda)]
  table = ops.StorageTable(pool)
  host_buf = torch.zeros(16, dtype=torch.uint8, pin_memory=True)
  rc = noalloc_offload(table, [0], [0], host_buf, 1, torch.cuda.current_stream(cuda))
  assert rc == _native.OUT_OF_RANGE
  assert "exceeds the static staging capacity" in _native.last_error()

"""GPU tests of ts_kv_offload_noalloc, the offload entry point that allocates
no device memory.  It exists for callers whose HBM already belongs to their
own allocator or KV pool (a serving engine that reserved a memory fraction up
front), where one more cudaMalloc would fail, fragment that pool, or
synchronise the device under the engine's running work.  Its only staging is
a 64 MiB array compiled into the library.

Every case is checked bit-exact against the CPU oracle's byte model of the
reference's offload (oracle/kv_blocks.py: per storage, host bytes of block
dst = device bytes of block src, in the block-major host layout, uncovered
bytes zero); the first one also against the manager's offload (ts_d2h), on
two calls in a row.  The file name makes pytest collect it last."""

import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import kv_blocks as ref
from tpu_sync_b200 import KVCacheManager, _native, ops, workloads

pytestmark = pytest.mark.gpu


def host_table(storages, offs):
  """The storage table in host memory, as the entry point takes it."""
  arr = (_native.BlockStorage * len(storages))()
  for i, (t, off) in enumerate(zip(storages, offs)):
    nbytes = t.numel() * t.element_size()
    arr[i].dev_ptr = t.data_ptr()
    arr[i].block_bytes = nbytes // t.shape[0]
    arr[i].dev_bytes = nbytes
    arr[i].stage_off = off
  return arr


def noalloc_offload(device, table, src, dst, host_buf, pitch, host_blocks, stream):
  s = _native.i64_array(src)
  d = _native.i64_array(dst)
  return _native.lib().ts_kv_offload_noalloc(
      device.index, table, len(table), _native.i64_ptr(s), _native.i64_ptr(d), s.size,
      ctypes.c_void_p(host_buf.data_ptr()), pitch, host_blocks,
      ctypes.c_void_p(stream.cuda_stream))


def as_bytes(t):
  return t.contiguous().view(torch.uint8).cpu().numpy().reshape(t.shape[0], -1)


def expect(host_before, pool, src, dst, offs, pitch):
  """Oracle: the host tier after the offload (later copies win)."""
  out = host_before.copy()
  rows = ref.extract_to_padded_staging([as_bytes(t) for t in pool], src, offs, pitch)
  for k, h in enumerate(dst):
    out[h] = rows[k]
  return out


def run_case(cuda, pool, offs, pitch, host_buf, calls):
  """Runs each (src, dst) call in turn on one stream; checks the host tier
  against the oracle after every call."""
  table = host_table(pool, offs)
  stream = torch.cuda.current_stream(cuda)
  host_blocks = host_buf.shape[0]
  want = host_buf.numpy().copy()
  for src, dst in calls:
    rc = noalloc_offload(cuda, table, src, dst, host_buf, pitch, host_blocks, stream)
    assert rc == _native.OK, _native.last_error()
    stream.synchronize()
    want = expect(want, pool, src, dst, offs, pitch)
    np.testing.assert_array_equal(host_buf.numpy(), want)


def test_noalloc_offload_matches_oracle_and_manager_twice(cuda):
  geom = workloads.KVGeometry(layers=4, kv=2, block_tokens=16, heads=8, head_dim=128)
  pool = workloads.kv_pool(geom, 96, 31, cuda)
  host_blocks = 48
  mgr = KVCacheManager([[t] for t in pool], host_blocks_to_allocate=host_blocks)
  t = ops.StorageTable(pool)
  assert t.pitch == mgr.host_block_pitch
  host_buf = torch.zeros((host_blocks, t.pitch), dtype=torch.uint8, pin_memory=True)
  table = host_table(pool, t.stage_offs)
  stream = torch.cuda.current_stream(cuda)
  rng = np.random.default_rng(12)
  want = host_buf.numpy().copy()
  for call in range(2):  # two calls in a row; the second reuses the static staging
    n = 40 if call == 0 else 33
    src = rng.choice(96, n, replace=False)
    dst = rng.choice(host_blocks, n, replace=False)
    if call == 1:
      dst[:10] = np.arange(5, 15)  # a coalescible run of host ids
    mgr.d2h(src.tolist(), dst.tolist()).Await()
    rc = noalloc_offload(cuda, table, src, dst, host_buf, t.pitch, host_blocks, stream)
    assert rc == _native.OK, _native.last_error()
    stream.synchronize()
    want = expect(want, pool, src, dst, t.stage_offs, t.pitch)
    np.testing.assert_array_equal(host_buf.numpy(), want)
    hb = host_buf.numpy()
    for l in range(len(pool)):
      off, bb = t.stage_offs[l], t.block_bytes[l]
      for h in sorted(set(int(x) for x in dst)):
        assert hb[h, off:off + bb].tobytes() == mgr.read_block_bytes(l, h), (call, l, h)
  mgr.close()


def test_noalloc_offload_c1_pitch_several_chunks(cuda):
  """C1 geometry (64 storages of 32 KiB: 2 MiB per block), 70 and then 45
  blocks: the 64 MiB array holds 32 blocks, so a call runs in chunks whose
  gathers wait for the previous chunk's DMAs out of the same rows.  Host ids
  repeat (last copy wins) and run backwards as well as forwards."""
  g = workloads.C1
  pool = workloads.kv_pool(g, 72, 5, cuda)
  t = ops.StorageTable(pool)
  assert t.pitch == 2 << 20
  host_blocks = 100
  host_buf = torch.full((host_blocks, t.pitch), 0x5A, dtype=torch.uint8, pin_memory=True)
  rng = np.random.default_rng(3)
  src1 = rng.choice(72, 70, replace=False)
  dst1 = np.concatenate([np.arange(10, 40), np.arange(90, 60, -1), rng.choice(60, 10)])
  src2 = rng.integers(0, 72, 45)
  dst2 = np.concatenate([np.arange(20, 50), [5, 5, 6, 5, 99, 0, 98, 97, 96, 1, 2, 3, 4, 7, 8]])
  run_case(cuda, pool, t.stage_offs, t.pitch, host_buf, [(src1, dst1), (src2, dst2)])


def test_noalloc_offload_clears_padding_left_by_an_earlier_call(cuda):
  """A layout with gaps between and after the slots: the gaps reach the host
  as zeros, although an earlier call (one 512-byte storage filling the whole
  pitch) left data in those bytes of the shared staging."""
  full = [torch.randint(1, 255, (20, 512), dtype=torch.uint8, device=cuda)]
  host_buf = torch.full((16, 512), 0xAB, dtype=torch.uint8, pin_memory=True)
  run_case(cuda, full, [0], 512, host_buf, [(np.arange(12), np.arange(12))])
  gappy = [torch.randint(0, 255, (20, 32), dtype=torch.uint8, device=cuda) for _ in range(3)]
  run_case(cuda, gappy, [16, 80, 160], 512, host_buf,
           [(np.array([3, 19, 0, 7]), np.array([2, 3, 4, 11])),
            (np.array([8, 9]), np.array([15, 0]))])


def test_noalloc_offload_unaligned_blocks_byte_path(cuda):
  """6-byte blocks (3 x int16) at 16-byte rounded slots: no 16-byte vectors
  are possible, the byte path gathers them, and the slot padding is zero."""
  pool = [torch.arange(30 * 3, dtype=torch.int16, device=cuda).view(30, 3) + 100 * s
          for s in range(3)]
  t = ops.StorageTable(pool)
  host_buf = torch.full((12, t.pitch), 0x77, dtype=torch.uint8, pin_memory=True)
  run_case(cuda, pool, t.stage_offs, t.pitch, host_buf,
           [(np.array([29, 3, 0, 14]), np.array([0, 11, 5, 6])),
            (np.array([1, 1, 2]), np.array([6, 7, 6]))])


def test_noalloc_offload_more_blocks_than_one_launch_takes(cuda):
  """300 small blocks: one gather takes at most 256 ids, so the call runs two
  chunks even though the staging would hold far more rows."""
  pool = [torch.randint(0, 255, (320, 256), dtype=torch.uint8, device=cuda) for _ in range(2)]
  host_buf = torch.zeros((400, 512), dtype=torch.uint8, pin_memory=True)
  rng = np.random.default_rng(9)
  run_case(cuda, pool, [0, 256], 512, host_buf,
           [(rng.choice(320, 300, replace=False), rng.choice(400, 300, replace=False))])


def test_noalloc_offload_rejects_bad_ids_and_queues_nothing(cuda):
  pool = [torch.randint(0, 255, (8, 64), dtype=torch.uint8, device=cuda) for _ in range(2)]
  table = host_table(pool, [0, 64])
  host_buf = torch.full((4, 128), 0x11, dtype=torch.uint8, pin_memory=True)
  stream = torch.cuda.current_stream(cuda)
  rc = noalloc_offload(cuda, table, [0, 8], [0, 1], host_buf, 128, 4, stream)
  assert rc == _native.INVALID_ARGUMENT
  assert "source device buffer" in _native.last_error()
  rc = noalloc_offload(cuda, table, [0, 1], [0, 4], host_buf, 128, 4, stream)
  assert rc == _native.INVALID_ARGUMENT
  assert "destination host buffer" in _native.last_error()
  rc = noalloc_offload(cuda, host_table(pool, [0, 100]), [0], [0], host_buf, 128, 4, stream)
  assert rc == _native.INVALID_ARGUMENT  # slot past the pitch
  stream.synchronize()
  assert (host_buf.numpy() == 0x11).all()


def test_noalloc_offload_rejects_oversized_pitch_and_tables(cuda):
  # one 65 MiB block per storage cannot fit the 64 MiB static staging
  pool = [torch.zeros((1, 65 << 20), dtype=torch.uint8, device=cuda)]
  host_buf = torch.zeros(16, dtype=torch.uint8, pin_memory=True)
  stream = torch.cuda.current_stream(cuda)
  rc = noalloc_offload(cuda, host_table(pool, [0]), [0], [0], host_buf, 65 << 20, 1, stream)
  assert rc == _native.OUT_OF_RANGE
  assert "exceeds the static staging capacity" in _native.last_error()
  small = torch.zeros((2, 16), dtype=torch.uint8, device=cuda)
  many = host_table([small] * 513, [16 * i for i in range(513)])
  rc = noalloc_offload(cuda, many, [0], [0], host_buf, 16 * 513, 1, stream)
  assert rc == _native.OUT_OF_RANGE


def test_noalloc_offload_returns_without_waiting_for_the_device(cuda):
  """Queued behind ~0.5 s of GPU work on its stream, the call returns at
  once (it reads nothing back from the device) and the bytes land when the
  stream drains."""
  pool = [torch.randint(0, 255, (64, 4096), dtype=torch.uint8, device=cuda) for _ in range(4)]
  offs = [4096 * i for i in range(4)]
  host_buf = torch.zeros((64, 4 * 4096), dtype=torch.uint8, pin_memory=True)
  table = host_table(pool, offs)
  stream = torch.cuda.Stream(cuda)
  src, dst = np.arange(40)[::-1].copy(), np.arange(40)
  # warm-up (kernel loading in a fresh process), outside the slept window
  rc = noalloc_offload(cuda, table, src, dst, host_buf, 4 * 4096, 64, stream)
  assert rc == _native.OK, _native.last_error()
  with torch.cuda.stream(stream):
    torch.cuda._sleep(1000)
  torch.cuda.synchronize()
  host_buf.zero_()
  with torch.cuda.stream(stream):
    torch.cuda._sleep(1_000_000_000)
  t0 = time.perf_counter()
  rc = noalloc_offload(cuda, table, src, dst, host_buf, 4 * 4096, 64, stream)
  host_s = time.perf_counter() - t0
  assert rc == _native.OK, _native.last_error()
  assert stream.query() is False
  assert host_s < 0.1, f"the call blocked the host for {host_s:.3f} s"
  stream.synchronize()
  np.testing.assert_array_equal(host_buf.numpy(),
                                expect(np.zeros((64, 4 * 4096), np.uint8), pool, src, dst,
                                       offs, 4 * 4096))

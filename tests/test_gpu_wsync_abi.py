"""GPU tests of the native weight synchronizer (ts_wsync_*) through the C ABI,
as a non-Python host would call it: the reference's PushWeightsResharded
cases (tpu_sync/weight_sync/weight_synchronizer_test.cc:184-460) case by case,
the check order across shards, overflow-safe ranges, random strided entries
against the oracle's entry expansion, and a push that queues without
blocking the host."""

import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import reshard as ors
from tpu_sync_b200 import _native

pytestmark = pytest.mark.gpu

PEER = b"localhost:0"


class Wsync:
  """Minimal C-ABI client: buffers [layer][shard], plan, push, wait."""

  def __init__(self, grid, names=None):
    L, S = len(grid), len(grid[0])
    bufs = (_native.WsyncBuffer * (L * S))()
    for l, layer in enumerate(grid):
      for s, t in enumerate(layer):
        b = bufs[l * S + s]
        b.dev_ptr, b.nbytes, b.device = t.data_ptr(), t.numel() * t.element_size(), t.device.index
    arr = (ctypes.c_char_p * L)(*[n.encode() for n in names]) if names else None
    self.h = ctypes.c_void_p()
    assert _native.lib().ts_wsync_create(bufs, L, S, arr, ctypes.byref(self.h)) == _native.OK

  def register(self, entries, dests, src_data_name=None):
    e = (_native.ShardPushEntry * max(len(entries), 1))(*entries)
    d = (_native.WsyncDest * max(len(dests), 1))(*dests)
    return _native.lib().ts_wsync_register_plan(self.h, e, len(entries), src_data_name, d,
                                                len(dests))

  def push(self, stream=None):
    s = stream or torch.cuda.current_stream()
    return _native.lib().ts_wsync_push(self.h, ctypes.c_void_p(s.cuda_stream))

  def wait(self):
    return _native.lib().ts_wsync_wait(self.h, 30_000)

  def close(self):
    _native.lib().ts_wsync_destroy(self.h)


def entry(shard=0, layer=0, size=0, so=0, do=0, ss=0, ds=0, count=1, dst_shard=0, peer=PEER):
  e = _native.ShardPushEntry(src_shard_idx=shard, has_layer_idx=int(layer is not None),
                             layer_idx=layer if layer is not None else 0, dst_peer=peer,
                             dst_shard_idx=dst_shard, src_offset_bytes=so, dst_offset_bytes=do,
                             size_bytes=size, src_stride_bytes=ss, dst_stride_bytes=ds,
                             count=count)
  return e


def dest(t, layer=0, shard=0, peer=PEER):
  return _native.WsyncDest(peer=peer, layer_idx=layer, dst_shard_idx=shard, dst_ptr=t.data_ptr(),
                           nbytes=t.numel() * t.element_size(), device=t.device.index)


def filled(cuda, sizes, value):
  return [[torch.full((n,), value, dtype=torch.uint8, device=cuda)] for n in sizes]


def test_exact_boundary(cuda):
  """PushWeightsReshardedExactBoundary (:184-227): one entry of the whole
  16 KiB slice copies every byte."""
  src, dst = filled(cuda, [16384], 0xAB), filled(cuda, [16384], 0)
  w = Wsync(src)
  assert w.register([entry(size=16384)], [dest(dst[0][0])]) == _native.OK
  assert w.push() == _native.OK and w.wait() == _native.OK
  assert bool((dst[0][0] == 0xAB).all())
  w.close()


def test_zero_bytes(cuda):
  """PushWeightsReshardedZeroBytes (:229-272): a zero-byte entry succeeds
  and writes nothing."""
  src, dst = filled(cuda, [16384], 0xAB), filled(cuda, [16384], 0)
  w = Wsync(src)
  assert w.register([entry(size=0)], [dest(dst[0][0])]) == _native.OK
  assert w.push() == _native.OK and w.wait() == _native.OK
  assert int(dst[0][0].count_nonzero()) == 0
  w.close()


def test_out_of_bounds(cuda):
  """PushWeightsReshardedOutOfBoundsError (:274-307): 500 + 600 > 1024 is
  INVALID_ARGUMENT, and nothing is registered."""
  src, dst = filled(cuda, [1024], 0xAB), filled(cuda, [1024], 0)
  w = Wsync(src)
  assert w.register([entry(so=500, size=600)], [dest(dst[0][0])]) == _native.INVALID_ARGUMENT
  assert _native.last_error() == "Push range out of bounds"
  n, b = ctypes.c_int64(), ctypes.c_uint64()
  assert _native.lib().ts_wsync_info(w.h, ctypes.byref(n), ctypes.byref(b)) == _native.OK
  assert n.value == 0 and b.value == 0
  w.close()


def test_invalid_layer_index(cuda):
  """PushWeightsReshardedInvalidLayerIndexError (:309-342)."""
  src, dst = filled(cuda, [1024, 1024], 0xAB), filled(cuda, [1024, 1024], 0)
  w = Wsync(src)
  rc = w.register([entry(layer=2, size=128)], [dest(dst[0][0])])
  assert rc == _native.INVALID_ARGUMENT
  assert _native.last_error() == "Layer index out of bounds: 2"
  w.close()


def test_empty_schedule(cuda):
  """PushWeightsReshardedEmptySchedule (:344-360)."""
  w = Wsync(filled(cuda, [1024], 0xAB))
  assert w.register([], []) == _native.OK
  assert w.push() == _native.OK and w.wait() == _native.OK
  w.close()


def test_fallback_by_name(cuda):
  """PushWeightsReshardedFallbackByNameSuccess (:362-416) and
  ...NotFoundError (:418-460): an entry without layer_idx uses the layer
  named by the first source unit."""
  src = filled(cuda, [16384, 8192], 0xAB)
  dst = filled(cuda, [16384, 8192], 0)
  w = Wsync(src, names=["layer_A", "layer_B"])
  d = [dest(dst[0][0], layer=0), dest(dst[1][0], layer=1)]
  assert w.register([entry(layer=None, size=8192)], d, b"layer_B") == _native.OK
  assert w.push() == _native.OK and w.wait() == _native.OK
  assert bool((dst[1][0] == 0xAB).all()) and int(dst[0][0].count_nonzero()) == 0
  rc = w.register([entry(layer=None, size=1024)], d, b"unknown_layer")
  assert rc == _native.NOT_FOUND
  assert _native.last_error() == "Layer name not found in WeightSynchronizer: unknown_layer"
  rc = w.register([entry(layer=None, size=1024)], d, None)
  assert rc == _native.INVALID_ARGUMENT
  assert _native.last_error() == "src_units list cannot be empty"
  w.close()


def test_checks_run_shard_by_shard_before_any_byte_moves(cuda):
  """Shards are visited in order (shard 0's schedule first, whatever the
  array order), and a later failing entry leaves nothing registered or
  moved; destinations must exist and hold the entry's range; ranges near
  2^64 do not wrap around."""
  src = [[torch.full((1024,), 0xAB, dtype=torch.uint8, device=cuda) for _ in range(2)]]
  dst = [torch.zeros(1024, dtype=torch.uint8, device=cuda) for _ in range(2)]
  w = Wsync(src)
  d = [dest(dst[0], shard=0), dest(dst[1], shard=1)]
  bad_s1 = entry(shard=1, so=1000, size=100, dst_shard=1)
  bad_s0 = entry(shard=0, layer=5, size=8)
  assert w.register([bad_s1, bad_s0], d) == _native.INVALID_ARGUMENT
  assert _native.last_error() == "Layer index out of bounds: 5"
  good = entry(shard=0, size=64)
  assert w.register([good, bad_s1], d) == _native.INVALID_ARGUMENT
  assert _native.last_error() == "Push range out of bounds"
  rc = w.register([entry(size=64, peer=b"nobody")], d)
  assert rc == _native.INVALID_ARGUMENT and "No destination for peer nobody" in _native.last_error()
  assert w.register([entry(size=64, do=1000)], d) == _native.INVALID_ARGUMENT
  assert _native.last_error() == "Push destination range out of bounds"
  huge = (1 << 64) - 16
  assert w.register([entry(so=huge, size=32)], d) == _native.INVALID_ARGUMENT
  assert w.register([entry(size=16, ss=huge, ds=16, count=3)], d) == _native.INVALID_ARGUMENT
  assert w.register([entry(size=16, do=huge)], d) == _native.INVALID_ARGUMENT
  assert w.push() == _native.OK and w.wait() == _native.OK  # nothing registered
  assert int(dst[0].count_nonzero()) == 0 and int(dst[1].count_nonzero()) == 0
  w.close()


def test_random_strided_entries_match_oracle(cuda):
  """40 random strided entries over two shards against the oracle's entry
  expansion (weight_synchronizer_base.cc:606-667), then a second plan on
  the same object."""
  rng = np.random.default_rng(23)
  nbytes = 1 << 16
  g = torch.Generator().manual_seed(8)
  src_host = [torch.randint(0, 256, (nbytes,), generator=g, dtype=torch.uint8) for _ in range(2)]
  src = [[t.to(cuda) for t in src_host]]
  dst = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(2)]
  w = Wsync(src)
  d = [dest(dst[0], shard=0), dest(dst[1], shard=1)]
  for rep in range(2):
    want = [t.cpu().numpy().copy() for t in dst]
    entries, used = [], [np.zeros(nbytes, bool) for _ in range(2)]
    while len(entries) < 40:
      sh = int(rng.integers(0, 2))
      size = int(rng.integers(1, 300))
      count = int(rng.integers(1, 6))
      ss = size + int(rng.integers(0, 50)) if count > 1 else 0
      ds = size + int(rng.integers(0, 50)) if count > 1 else 0
      so = int(rng.integers(0, nbytes - (count * max(ss, size) + size)))
      do = int(rng.integers(0, nbytes - (count * max(ds, size) + size)))
      span = [(do + c * (ds if count > 1 else size), size) for c in range(count)]
      if any(used[sh][a:a + n].any() for a, n in span):
        continue  # destinations of one push are disjoint
      for a, n in span:
        used[sh][a:a + n] = True
      entries.append(entry(shard=sh, so=so, do=do, size=size, ss=ss, ds=ds, count=count,
                           dst_shard=sh))
      ors.apply_byte_entries(src_host[sh].numpy(), want[sh], [(so, do, size, ss, ds, count)])
    assert w.register(entries, d) == _native.OK, _native.last_error()
    assert w.push() == _native.OK and w.wait() == _native.OK
    for k in range(2):
      np.testing.assert_array_equal(dst[k].cpu().numpy(), want[k])
  w.close()


def test_push_queues_without_blocking(cuda):
  """ts_wsync_push only queues: behind ~0.5 s of GPU work on the caller's
  stream it returns at once, query says pending, and the bytes land after."""
  src, dst = filled(cuda, [1 << 20], 0x5C), filled(cuda, [1 << 20], 0)
  w = Wsync(src)
  assert w.register([entry(size=1 << 20)], [dest(dst[0][0])]) == _native.OK
  s = torch.cuda.Stream(cuda)
  # warm-up (kernel loading in a fresh process), outside the slept window
  assert w.push(s) == _native.OK and w.wait() == _native.OK
  with torch.cuda.stream(s):
    torch.cuda._sleep(1000)
  dst[0][0].zero_()
  torch.cuda.synchronize()
  with torch.cuda.stream(s):
    torch.cuda._sleep(1_000_000_000)
  t0 = time.perf_counter()
  assert w.push(s) == _native.OK
  assert time.perf_counter() - t0 < 0.1
  assert _native.lib().ts_wsync_query(w.h) == _native.PENDING
  assert w.wait() == _native.OK
  assert bool((dst[0][0] == 0x5C).all())
  w.close()

"""Block hand-off between managers on one node (the reference's pull protocol:
register_read / start_read / poll_stats, api/torch/kv_cache_manager.py:172-175,
:334-396) over a /dev/shm mailbox, CUDA IPC and the peer copy kernel.

Bytes are checked against the producer's pool (every storage, every block
pair); the protocol's outcomes against the reference's: a consumer's read is
done or failed (never registered in time, unregistered block), a producer's
send is done once consumed or when nobody claimed it before its deadline.
"""

import os
import subprocess
import sys
import textwrap
import time
from pathlib import Path

import numpy as np
import pytest
import torch

from tpu_sync_b200 import KVCacheManager

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
LAYERS, BLOCKS, BB = 3, 64, 8192


def pool(seed, device, blocks=BLOCKS, bb=BB, layers=LAYERS):
  g = torch.Generator().manual_seed(seed)
  return [torch.randint(0, 256, (blocks, bb), generator=g, dtype=torch.uint8).to(device)
          for _ in range(layers)]


def poll_until(mgr, which, want, timeout=20.0):
  got = []
  t0 = time.time()
  while time.time() - t0 < timeout:
    res = mgr.poll_stats()
    got += res[which]
    if want in got:
      return got
    time.sleep(0.01)
  return got


def test_same_process_read_moves_blocks(cuda):
  src, dst = pool(1, cuda), pool(2, cuda)
  before = [t.clone() for t in dst]
  prod = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4)
  cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4)
  remote_ids, local_ids = [5, 9, 40, 41, 63], [0, 1, 2, 30, 17]
  assert prod.register_read("req-a", 11, remote_ids)
  assert not prod.register_read("req-empty", 12, [])
  cons.start_read("req-a", 11, prod.get_local_endpoints(), remote_ids, local_ids)
  assert "req-a" in poll_until(cons, 1, "req-a")
  torch.cuda.synchronize()
  for l in range(LAYERS):
    for r, d in zip(remote_ids, local_ids):
      assert torch.equal(dst[l][d], src[l][r])
    untouched = [b for b in range(BLOCKS) if b not in local_ids]
    assert torch.equal(dst[l][untouched], before[l][untouched])
  assert "req-a" in poll_until(prod, 0, "req-a")
  prod.close()
  cons.close()


def test_read_before_registration_and_stream_order(cuda):
  """The consumer may start first: its read launches once the producer
  registers; later work on the consumer's stream sees the blocks."""
  src, dst = pool(3, cuda), pool(4, cuda)
  prod = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4)
  cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4)
  ep = prod.get_local_endpoints()[0]["endpoint"]
  cons.start_read("req-b", 21, ep, [1, 2, 3], [10, 11, 12])
  assert cons.poll_stats() == ([], [], [])
  s = torch.cuda.Stream(cuda)
  with torch.cuda.stream(s):
    src[0][1].fill_(7)  # the producer writes, then registers on the same stream
    prod.register_read("req-b", 21, [1, 2, 3], stream=s)
  assert "req-b" in poll_until(cons, 1, "req-b")
  torch.cuda.synchronize()
  assert bool((dst[0][10] == 7).all())
  assert torch.equal(dst[2][12], src[2][3])
  prod.close()
  cons.close()


def test_failures_and_timeouts(cuda):
  src, dst = pool(5, cuda), pool(6, cuda)
  prod = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4, timeout_s=0.5)
  cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4, timeout_s=0.5)
  ep = prod.get_local_endpoints()
  # a block the producer did not register for this uuid
  prod.register_read("req-c", 31, [1, 2])
  with pytest.raises(RuntimeError, match="block 3 was not registered for read by uuid 31"):
    cons.start_read("req-c", 31, ep, [1, 3], [0, 1])
  assert "req-c" in poll_until(prod, 0, "req-c")  # the producer is released
  # never registered: the consumer's read fails at its deadline
  cons.start_read("req-d", 41, ep, [1], [0])
  assert "req-d" in poll_until(cons, 2, "req-d", timeout=5.0)
  # registered, never claimed: the producer's send times out (done sending)
  prod.register_read("req-e", 51, [4])
  assert "req-e" in poll_until(prod, 0, "req-e", timeout=5.0)
  # argument checks
  with pytest.raises(RuntimeError, match="out of range"):
    prod.register_read("req-f", 61, [BLOCKS])
  with pytest.raises(RuntimeError, match="local block id 64 out of range"):
    cons.start_read("req-g", 71, ep, [0], [BLOCKS])
  with pytest.raises(RuntimeError, match="already registered"):
    prod.register_read("req-h", 81, [1])
    prod.register_read("req-h2", 81, [2])
  with pytest.raises(RuntimeError, match="no transfer endpoint"):
    cons.start_read("req-i", 91, "ipc:/tsb_no_such_endpoint", [0], [0])
  prod.close()
  cons.close()


def test_geometry_mismatch_is_rejected(cuda):
  prod = KVCacheManager([[t] for t in pool(7, cuda)], host_blocks_to_allocate=4)
  other = KVCacheManager([[t] for t in pool(8, cuda, bb=4096)], host_blocks_to_allocate=4)
  prod.register_read("req-j", 1, [0])
  with pytest.raises(RuntimeError, match="remote block bytes 8192 differ from the local 4096"):
    other.start_read("req-j", 1, prod.get_local_endpoints(), [0], [0])
  prod.close()
  other.close()


_PRODUCER = textwrap.dedent("""
    import sys, time
    sys.path.insert(0, {root!r})
    import torch
    from tpu_sync_b200 import KVCacheManager
    dev = torch.device("cuda", {device})
    g = torch.Generator().manual_seed(99)
    src = [torch.randint(0, 256, ({blocks}, {bb}), generator=g, dtype=torch.uint8).to(dev)
           for _ in range({layers})]
    mgr = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4)
    assert mgr.register_read("xproc", 7, list(range(0, {blocks}, 3)))
    print(mgr.get_local_endpoints()[0]["endpoint"], flush=True)
    t0 = time.time()
    while time.time() - t0 < 60:
      if "xproc" in mgr.poll_stats()[0]:
        print("SENT", flush=True)
        break
      time.sleep(0.01)
    mgr.close()
""")


def run_cross_process(producer_device, consumer_device):
  script = _PRODUCER.format(root=str(ROOT), device=producer_device, blocks=BLOCKS, bb=BB,
                            layers=LAYERS)
  p = subprocess.Popen([sys.executable, "-c", script], stdout=subprocess.PIPE,
                       stderr=subprocess.PIPE, text=True)
  try:
    endpoint = p.stdout.readline().strip()
    assert endpoint.startswith("ipc:"), p.stderr.read()[-3000:]
    dev = torch.device("cuda", consumer_device)
    dst = pool(123, dev)
    cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4)
    remote = list(range(0, BLOCKS, 3))
    local = list(reversed(range(len(remote))))
    cons.start_read("xproc", 7, endpoint, remote, local)
    assert "xproc" in poll_until(cons, 1, "xproc")
    torch.cuda.synchronize(dev)
    want = pool(99, "cpu")
    for l in range(LAYERS):
      for r, d in zip(remote, local):
        assert torch.equal(dst[l][d].cpu(), want[l][r])
    out, err = p.communicate(timeout=60)
    assert "SENT" in out, err[-3000:]
    cons.close()
  finally:
    if p.poll() is None:
      p.kill()
      p.wait()


def test_cross_process_read_same_gpu(cuda):
  run_cross_process(0, 0)


def test_read_state_progression(cuda):
  src, dst = pool(9, cuda), pool(10, cuda)
  prod = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4)
  cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4)
  assert prod.read_state(5) == "none"
  prod.register_read("req-s", 5, [0, 1])
  t0 = time.time()
  while prod.read_state(5) != "ready" and time.time() - t0 < 5:
    time.sleep(0.001)
  assert prod.read_state(5) == "ready"
  cons.start_read("req-s", 5, prod.get_local_endpoints(), [0, 1], [2, 3])
  assert "req-s" in poll_until(cons, 1, "req-s")
  assert prod.read_state(5) == "consumed"
  assert "req-s" in poll_until(prod, 0, "req-s")
  assert prod.read_state(5) == "none"
  prod.close()
  cons.close()

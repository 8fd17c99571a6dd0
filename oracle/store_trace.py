"""C1 access trace and the reference's tier-2 decisions for it.

TEST AND BASELINE INFRASTRUCTURE ONLY (not product code): the CPU reference
arm of bench.py takes its offload / reload block lists from here, so it runs
without the product library, and tests check that the product store makes
the same decisions.

* zipf_trace: the configuration's synthetic access stream (100k accesses,
  Zipf(1.1) over 200k prefix ids; rank r has probability proportional to
  r^-s and ranks map to ids through a seeded permutation).
* transfer_streams: runs the trace through oracle/_ref/store_trace_ref, the
  reference's own LRUCache (tpu_sync/kv_cache/lru_cache.h) and
  LogicalBlockManager (tpu_sync/kv_cache/logical_block_manager.cc) compiled
  from source and composed as KVCacheStore's local Lookup / Insert / Save /
  Load / Poll compose them (tpu_sync/kv_cache/kv_cache_store.cc:977-1137,
  :1743-1781, :2113-2254; host_offload_backend.cc:154-536, :656-688).
  Per access: a device block from a ring over the HBM pool; a hit is looked
  up (pinned) and loaded into it, a miss is inserted from it and saved.
"""

from __future__ import annotations

import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
STORE_TRACE_REF = HERE / "_ref" / "store_trace_ref"


def zipf_trace(n_access: int = 100_000, n_ids: int = 200_000, s: float = 1.1,
               seed: int = 10) -> np.ndarray:
  """n_access prefix ids drawn Zipf(s) over n_ids (seeded)."""
  rng = np.random.default_rng(seed)
  p = np.arange(1, n_ids + 1, dtype=np.float64) ** (-s)
  p /= p.sum()
  ranks = rng.choice(n_ids, size=n_access, p=p)
  return rng.permutation(n_ids)[ranks].astype(np.int64)


def available() -> bool:
  return STORE_TRACE_REF.exists()


def transfer_streams(trace: np.ndarray, host_blocks: int, device_blocks: int,
                     batch: int = 512, capacity: int | None = None):
  """The reference's (saves, loads) per access batch for the trace.

  saves = [(device id, host id)], loads = [(host id, device id)]; stats as a
  dict with accesses, hits, misses and hit_rate.  The LRU capacity defaults
  to host_blocks.
  """
  if not available():
    raise RuntimeError(f"{STORE_TRACE_REF} is not built (oracle/build_ref.py needs the "
                       "reference checkout)")
  cap = host_blocks if capacity is None else capacity
  out = subprocess.run([str(STORE_TRACE_REF), str(cap), str(host_blocks), str(device_blocks),
                        str(batch)], input=" ".join(map(str, trace.tolist())).encode(),
                       stdout=subprocess.PIPE, check=True).stdout.decode().split("\n")
  batches, i = [], 0
  hits = misses = 0
  while i < len(out):
    f = out[i].split()
    i += 1
    if not f:
      continue
    if f[0] == "H":
      hits, misses = int(f[1]), int(f[2])
      continue
    ns, nl = int(f[1]), int(f[2])
    saves = [tuple(int(v) for v in out[i + k].split()[1:]) for k in range(ns)]
    loads = [tuple(int(v) for v in out[i + ns + k].split()[1:]) for k in range(nl)]
    i += ns + nl
    batches.append((saves, loads))
  stats = {"accesses": int(len(trace)), "hits": hits, "misses": misses,
           "hit_rate": round(hits / max(hits + misses, 1), 4)}
  return batches, stats

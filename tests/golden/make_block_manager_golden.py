"""Generates tests/golden/block_manager.json: host block allocator fixtures.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_block_manager_golden.py

Seeded random operation scripts (Allocate with and without lock, including
sizes out of range and requests that need LRU eviction; AllocateTarget,
Unlock, Deallocate with valid, duplicate, unallocated and out-of-range ids;
AccessBlock; state counts) answered by the REFERENCE
tpu_sync/kv_cache/logical_block_manager.cc itself, compiled by
oracle/build_ref.py into oracle/_ref/bm_ref (driver oracle/ref_bm_driver.cc).

The output is committed; tests never read the reference.
"""

from __future__ import annotations

import json
import random
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "block_manager.json"
sys.path.insert(0, str(ROOT))


def script(rng: random.Random):
  n = rng.randint(1, 40)
  ops = []
  for _ in range(300):
    x = rng.random()
    if x < 0.35:
      k = rng.choice([rng.randint(1, max(1, n // 3)), rng.randint(-1, n + 2)])
      ops.append(f"alloc {k} {int(rng.random() < 0.4)}")
    elif x < 0.85:
      op = rng.choice(["target", "unlock", "dealloc"])
      m = rng.randint(1, 4)
      ids = [rng.randrange(-1, n + 1) for _ in range(m)]
      if rng.random() < 0.15 and ids:
        ids.append(ids[0])  # a duplicate id
      ops.append(f"{op} " + " ".join(map(str, ids)))
    elif x < 0.95:
      ops.append(f"access {rng.randrange(-1, n + 1)}")
    else:
      ops.append("stats")
  return n, ops


def main():
  from oracle import build_ref
  exe = build_ref.build_bm()
  if exe is None:
    raise SystemExit("bm_ref is not built (the reference checkout is absent)")
  rng = random.Random(424242)
  scripts = []
  for _ in range(12):
    n, ops = script(rng)
    out = subprocess.run([str(exe)], input="\n".join([f"new {n}"] + ops) + "\n", text=True,
                         capture_output=True, check=True, timeout=60).stdout.splitlines()
    assert out[0] == "ok" and len(out) == len(ops) + 1
    scripts.append({"blocks": n, "ops": [[o, a] for o, a in zip(ops, out[1:])]})
  OUT.write_text(json.dumps({
      "source": "tpu_sync/kv_cache/logical_block_manager.cc, compiled by oracle/build_ref.py "
                "(oracle/_ref/bm_ref)",
      "generator": "tests/golden/make_block_manager_golden.py, random.Random(424242)",
      "answers": "alloc: '<status code> <ids>' ('-' on error); target / unlock / dealloc / "
                 "access: '<status code>'; stats: '<free> <allocated> <locked>'",
      "scripts": scripts}, separators=(",", ":")) + "\n")
  print(f"{len(scripts)} scripts -> {OUT}")


if __name__ == "__main__":
  main()

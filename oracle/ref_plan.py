"""Runs the reference's pool reshard planning flow through oracle/_ref/plan_ref.

Test infrastructure only (the golden-fixture script uses it): the reference's
pool_layout.cc and reshard/{declaration_types, work_unit_directory,
request_block_registry, pool_reshard_planner}.cc, compiled by
oracle/build_ref.py, register the units and their byte-span declarations and
build the plan exactly as the reference's service does
(oracle/ref_pool_reshard_driver.cc); each outcome comes back as one JSON line.

A request is a plain dict:
  src_pools: [[pool dict, ...] per source unit]   dst_pools: [pool dict, ...]
  tags, dst_ids, dst_block_counts (or None), dst_skip_bytes (or None),
  parallelism (or None), transfer_parallelism: [per unit], transfer_ranks: [per unit],
  decls: [[unit, {"tag", "block_ids", "spans": [[8 ints]], "declared_bytes",
                  "dst_space_version"}], ...]
with pool dicts in the form of PoolSpec.to_dict().  A span's 8 ints are the
PoolByteSpan fields in declaration order (src_block_ordinal, src_offset_bytes,
dst_block_index, dst_offset_bytes, size_bytes, src_stride_bytes,
dst_stride_bytes, count).
"""

from __future__ import annotations

import json
import subprocess
from typing import Dict, List, Optional

from oracle import build_ref


def binary() -> Optional[str]:
  p = build_ref.build_plan()
  return str(p) if p is not None and p.exists() else None


def _pool_tokens(p: Dict) -> List[str]:
  t = [p["tag"], p["storage_index"], p.get("base_offset_bytes", 0), p["block_stride_bytes"],
       p["num_blocks"], p.get("dtype_tag") or "-", len(p["regions"])]
  for r in p["regions"]:
    t += [r["name"], r["offset_bytes"], r["stride_bytes"], r["unit_bytes"], r["num_units"],
          r["units_per_stride"]]
  return [str(x) for x in t]


def _ints(v: Optional[List[int]]) -> List[str]:
  if v is None:
    return ["-1"]
  return [str(len(v))] + [str(int(x)) for x in v]


def encode(req: Dict) -> str:
  """One request in the driver's token format."""
  nu = len(req["src_pools"])
  t = ["REQ", str(nu)]
  for u in range(nu):
    t += [str(req["transfer_parallelism"][u]), str(req["transfer_ranks"][u]),
          str(len(req["src_pools"][u]))]
    for p in req["src_pools"][u]:
      t += _pool_tokens(p)
  t.append(str(len(req["dst_pools"])))
  for p in req["dst_pools"]:
    t += _pool_tokens(p)
  t += [str(len(req["tags"]))] + list(req["tags"])
  t += _ints(req["dst_ids"])
  t += _ints(req.get("dst_block_counts"))
  t += _ints(req.get("dst_skip_bytes"))
  t.append(str(req.get("parallelism") or 0))
  t.append(str(len(req["decls"])))
  for unit, d in req["decls"]:
    t += [str(unit), d["tag"], str(d["dst_space_version"]), str(d["declared_bytes"])]
    t += _ints(d["block_ids"])
    t.append(str(len(d["spans"])))
    for s in d["spans"]:
      t += [str(int(x)) for x in s]
  return " ".join(t)


def run(requests: List[Dict]) -> List[Dict]:
  """The reference's outcome for every request (fresh directory and registry
  each): {"ok": true, plan fields...} or {"ok": false, "stage", "code", "message"}."""
  exe = binary()
  if exe is None:
    raise FileNotFoundError("plan_ref is not built (the reference checkout is absent)")
  text = "\n".join(encode(r) for r in requests) + "\n"
  r = subprocess.run([exe], input=text.encode(), capture_output=True, timeout=300, check=True)
  out = [json.loads(line) for line in r.stdout.decode().splitlines()]
  if len(out) != len(requests):
    raise RuntimeError(f"plan_ref answered {len(out)} of {len(requests)} requests: "
                       f"{r.stderr.decode()[-2000:]}")
  return out

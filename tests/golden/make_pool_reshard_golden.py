"""Generates tests/golden/pool_reshard_plans.json: pool reshard plan fixtures.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_pool_reshard_golden.py

Seeded random hand-off requests answered by the REFERENCE's own planning
flow: tpu_sync/kv_cache/pool_layout.cc and
tpu_sync/kv_cache/reshard/{declaration_types, work_unit_directory,
request_block_registry, pool_reshard_planner}.cc, compiled by
oracle/build_ref.py into oracle/_ref/plan_ref, register every unit, register
each source unit's byte-span declarations and build the plan
(oracle/ref_pool_reshard_driver.cc).

Requests: one to three source units over "fa" / "ssm" pools with sparse live
regions (so live copies split at region edges), one or two requested tags,
page-indexed (dst_space_version 0) and request-global (1) declarations,
strided page-indexed spans (two interleaved row sets per piece), destination
clips, admission parallelism; about a third carry one fault (a coverage gap
or overlap, declared bytes that disagree, an out-of-range source id or span
ordinal, a bad count or field, a duplicate tag, rank / parallelism errors,
a clip that is not a page multiple).  Each case stores the request and the
reference's outcome: the plan, or the stage (unit registration, span
registration, planning) and message of its error.

The output is committed; tests never read the reference.
"""

from __future__ import annotations

import json
import random
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "pool_reshard_plans.json"
sys.path.insert(0, str(ROOT))

N_CASES = 300


def region(name, off, stride, unit, n, ups=1):
  return {"name": name, "offset_bytes": off, "stride_bytes": stride, "unit_bytes": unit,
          "num_units": n, "units_per_stride": ups}


def pool(tag, storage, stride, nb, regions, dtype="bf16"):
  return {"tag": tag, "storage_index": storage, "base_offset_bytes": 0,
          "block_stride_bytes": stride, "num_blocks": nb, "dtype_tag": dtype,
          "regions": regions}


def span(ordinal, soff, page, doff, size, sstride=0, dstride=0, count=1):
  return [ordinal, soff, page, doff, size, sstride, dstride, count]


def random_request(rng: random.Random):
  nu = rng.randint(1, 3)
  tags = ["fa"] if rng.random() < 0.65 else (["fa", "ssm"] if rng.random() < 0.7 else ["ssm"])
  geo = {}
  src_pools, dst_pools = [], []
  for t in ("fa", "ssm"):
    su = rng.choice([16, 32, 48])
    du = rng.choice([16, 32, 64])
    sn, dn = rng.randint(2, 6), rng.randint(1, 4)
    geo[t] = (su * sn, du * dn)
    # source: sn live units of su bytes every 2*su (gaps between them)
    src_pools.append(pool(t, 0, su * 2 * sn + 64, 12, [region("r", 8, su * 2, su, sn)]))
    dst_pools.append(pool(t, 1, du * dn + 32, 10, [region("r", 0, du, du, dn)]))
  decls, dst_ids, counts = [], [], []
  for t in tags:
    s_live, d_live = geo[t]
    k = rng.randint(1, 3)
    ids = rng.sample(range(10), k)
    dst_ids += ids
    counts.append(k)
    total = k * d_live - rng.choice([0, 0, 0, rng.randrange(1, d_live)])
    cuts = sorted(rng.sample(range(1, total), min(total - 1, rng.randint(0, 5))))
    edges = [0] + cuts + [total]
    per_unit = {}
    for a, b in zip(edges, edges[1:]):
      u = rng.randrange(nu)
      o = a
      while o < b:  # pieces no longer than a source block's live bytes
        n = min(s_live, b - o)
        per_unit.setdefault(u, []).append((o, n))
        o += n
    for u, pieces in sorted(per_unit.items()):
      version = rng.choice([0, 1])
      spans = []
      # distinct source ids per registration; pieces beyond 12 reuse a block
      blocks = rng.sample(range(12), min(len(pieces), 12))
      for i, (goff, size) in enumerate(pieces):
        ordinal = i % len(blocks)
        if version == 1:
          spans.append(span(ordinal, rng.randrange(0, s_live - size + 1), 0, goff, size))
          continue
        o, left = goff, size
        while left:
          page, inp = divmod(o, d_live)
          take = min(left, d_live - inp)
          if take % 8 == 0 and take >= 16 and rng.random() < 0.4:
            # two interleaved row sets: rows of `row` bytes, even rows from
            # one span, odd rows from the other (strided on both sides)
            # the source rows interleave the same way, inside [base, base + take)
            row = rng.choice([r for r in (4, 8) if take % (2 * r) == 0])
            rows = take // row
            base = rng.randrange(0, s_live - take + 1)
            ev, od = (rows + 1) // 2, rows // 2
            spans.append(span(ordinal, base, page, inp, row, 2 * row, 2 * row, ev))
            if od:
              spans.append(span(ordinal, base + row, page, inp + row, row, 2 * row, 2 * row,
                                od))
          else:
            spans.append(span(ordinal, rng.randrange(0, s_live - take + 1), page, inp,
                              take))
          o += take
          left -= take
      d = {"tag": t, "block_ids": blocks, "spans": spans,
           "declared_bytes": sum(s[4] * s[7] for s in spans), "dst_space_version": version}
      decls.append([u, d])
  par = [max(nu, rng.choice([1, 2, 3]))] * nu
  ranks = rng.sample(range(nu), nu)
  req = {"src_pools": [src_pools for _ in range(nu)], "dst_pools": dst_pools, "tags": tags,
         "dst_ids": dst_ids, "dst_block_counts": None, "dst_skip_bytes": None,
         "parallelism": None, "transfer_parallelism": par, "transfer_ranks": ranks,
         "decls": decls}
  if len(tags) > 1 or rng.random() < 0.3:
    req["dst_block_counts"] = counts
  if rng.random() < 0.15:
    req["parallelism"] = rng.choice([1, nu, nu + 2])
  if rng.random() < 0.12 and all(d["dst_space_version"] == 1 for _, d in decls):
    req["dst_skip_bytes"] = [geo[t][1] * rng.choice([0, 1]) for t in tags]
  fault(rng, req, geo)
  return req


def fault(rng: random.Random, req, geo):
  """Plants at most one fault (about a third of the requests)."""
  x = rng.random()
  decls = req["decls"]
  if x > 0.36 or not decls:
    return
  _, d = rng.choice(decls)
  nu = len(req["src_pools"])
  kinds = ["gap", "overlap", "declared", "src_id", "ordinal", "count0", "negative",
           "dup_tag", "rank_par", "rank_dup", "par_mixed", "skip_odd", "dst_dup", "tag_unknown",
           "span_past_live", "dup_id"]
  k = rng.choice(kinds)
  if k == "gap" and len(d["spans"]) > 1:
    d["spans"] = d["spans"][1:]
    d["declared_bytes"] = sum(s[4] * s[7] for s in d["spans"])
  elif k == "overlap":
    d["spans"] = d["spans"] + [list(d["spans"][0])]
    d["declared_bytes"] = sum(s[4] * s[7] for s in d["spans"])
  elif k == "declared":
    d["declared_bytes"] += rng.choice([1, -1])
  elif k == "src_id":
    d["block_ids"][-1] = 12 + rng.randrange(4)
  elif k == "dup_id" and len(d["block_ids"]) > 1:
    d["block_ids"][1] = d["block_ids"][0]
  elif k == "ordinal":
    d["spans"][0][0] = len(d["block_ids"]) + rng.randrange(2)
  elif k == "count0":
    d["spans"][0][7] = 0
  elif k == "negative":
    d["spans"][0][rng.choice([1, 3, 5, 6])] = -8
  elif k == "dup_tag":
    u = next(u for u, dd in decls if dd is d)
    decls.append([u, json.loads(json.dumps(d))])
  elif k == "rank_par" and nu > 1:
    req["transfer_parallelism"] = [nu - 1] * nu
  elif k == "rank_dup" and nu > 1:
    req["transfer_ranks"] = [0] * nu
  elif k == "par_mixed" and nu > 1:
    req["transfer_parallelism"] = [nu] * (nu - 1) + [nu + 1]
  elif k == "skip_odd":
    req["dst_skip_bytes"] = [rng.choice([8, 24, -16]) for _ in req["tags"]]
  elif k == "dst_dup" and len(req["dst_ids"]) > 1:
    req["dst_ids"][1] = req["dst_ids"][0]
  elif k == "tag_unknown":
    req["tags"] = req["tags"] + ["mamba"]
    if req["dst_block_counts"] is not None:
      req["dst_block_counts"] = req["dst_block_counts"] + [1]
  elif k == "span_past_live":
    s_live = geo[d["tag"]][0]
    d["spans"][0][1] = s_live - d["spans"][0][4] + 8
    d["spans"][0][7] = 1


# -- compact fixture form (expand() restores the request dicts) ---------------

POOL_KEYS = ("tag", "storage_index", "base_offset_bytes", "block_stride_bytes", "num_blocks",
             "dtype_tag")
REGION_KEYS = ("name", "offset_bytes", "stride_bytes", "unit_bytes", "num_units",
               "units_per_stride")
ENTRY_CONSTANTS = [0, 0, 1, 0, 0, "dst-0"]  # strides, count, dst shard, layer, dst peer


def compact_pool(p):
  return [p[k] for k in POOL_KEYS] + [[[r[k] for k in REGION_KEYS] for r in p["regions"]]]


def expand_pool(c):
  d = dict(zip(POOL_KEYS, c[:-1]))
  d["regions"] = [dict(zip(REGION_KEYS, r)) for r in c[-1]]
  return d


def compact(req):
  """Every source unit carries the same manifest: stored once."""
  assert all(u == req["src_pools"][0] for u in req["src_pools"])
  out = dict(req)
  out["n_units"] = len(req["src_pools"])
  out["src_pools"] = [compact_pool(p) for p in req["src_pools"][0]]
  out["dst_pools"] = [compact_pool(p) for p in req["dst_pools"]]
  return out


def expand(c):
  req = dict(c)
  n = req.pop("n_units")
  src = [expand_pool(p) for p in c["src_pools"]]
  req["src_pools"] = [src for _ in range(n)]
  req["dst_pools"] = [expand_pool(p) for p in c["dst_pools"]]
  return req


def compact_answer(a):
  """Schedule entries as (src_block, dst_block, src_off, dst_off, size,
  pool_group); the remaining fields are checked to be ENTRY_CONSTANTS."""
  if not a["ok"]:
    return a
  out = dict(a)
  out["schedules"] = {}
  for u, es in a["schedules"].items():
    for e in es:
      assert e[6:] == ENTRY_CONSTANTS, e
    out["schedules"][u] = [e[:6] for e in es]
  return out


def main():
  from oracle import ref_plan
  rng = random.Random(20260)
  cases = [random_request(rng) for _ in range(N_CASES)]
  answers = ref_plan.run(cases)
  n_ok = sum(a["ok"] for a in answers)
  stages = {}
  for a in answers:
    if not a["ok"]:
      stages[a["stage"]] = stages.get(a["stage"], 0) + 1
  packed = [compact(c) for c in cases]
  assert all(expand(p) == c for p, c in zip(packed, cases))
  OUT.write_text(json.dumps({
      "source": "reference pool reshard planning flow, compiled by oracle/build_ref.py "
                "(oracle/_ref/plan_ref)",
      "generator": "tests/golden/make_pool_reshard_golden.py, random.Random(20260)",
      "pool_keys": POOL_KEYS, "region_keys": REGION_KEYS,
      "entry": "src_block_id, dst_block_id, src_offset_bytes, dst_offset_bytes, size_bytes, "
               "pool_group (strides 0, count 1, dst_shard_idx 0, layer_idx 0 in every entry)",
      "cases": [{"request": c, "reference": compact_answer(a)}
                for c, a in zip(packed, answers)]},
      separators=(",", ":")) + "\n")
  print(f"{len(cases)} cases: {n_ok} plans, errors by stage {stages} -> {OUT}")


if __name__ == "__main__":
  main()

"""Pool reshard planner on the CPU: reference known answers, oracle parity.

* the known answers of the reference's planner tests
  (tpu_sync/kv_cache/reshard/reshard_service_test.cc:288-487), for both the
  product planner (tpu_sync_b200.pool_reshard, C ABI) and the oracle
  (oracle/pool_reshard.py);
* 300 seeded requests answered by the reference's own planning flow
  (tests/golden/pool_reshard_plans.json, made by
  tests/golden/make_pool_reshard_golden.py from the compiled reference):
  product and oracle give the same plan, or the same error message at the
  same step (unit registration, span registration, planning);
* product vs oracle on seeded random requests -- valid ones (entries,
  groups, active units equal) and broken ones (same error message);
* the C3 hand-off written as pool span declarations, applied by the oracle,
  equals the oracle's head-major -> token-major relayout.
"""

import json
import random
from pathlib import Path

import numpy as np
import pytest

from oracle import pool_reshard as opr
from oracle import reshard as ors
from tpu_sync_b200 import workloads
from tpu_sync_b200.pool_layout import PoolSpec, RegionSpec, coerce_pool_spec
from tpu_sync_b200.pool_reshard import (PoolByteSpan, PoolSpanRegistration,
                                        build_pool_reshard_plan)


def make_pool(live, stride, nb, tag="fa"):
  """MakePool of reshard_service_test.cc:63-80: one region over [0, live)."""
  return PoolSpec(tag, 0, 0, stride, nb, (RegionSpec("live", 0, live, live, 1, 1),), "uint8")


def reg(block_ids, spans, version=0, tag="fa", declared=None):
  return PoolSpanRegistration(tag, block_ids, [PoolByteSpan(*s) for s in spans], declared,
                              version)


def to_oracle(r: PoolSpanRegistration):
  return {"tag": r.tag, "block_ids": list(r.block_ids), "declared_bytes": r.declared(),
          "dst_space_version": r.dst_space_version,
          "spans": [dict(src_block_ordinal=s.src_block_ordinal, src_offset_bytes=s.src_offset_bytes,
                         dst_block_index=s.dst_block_index, dst_offset_bytes=s.dst_offset_bytes,
                         size_bytes=s.size_bytes, src_stride_bytes=s.src_stride_bytes,
                         dst_stride_bytes=s.dst_stride_bytes, count=s.count) for s in r.spans]}


def both(src_pools, dst_pools, tags, dst_ids, decls, **kw):
  """(product result or error, oracle result or error) in one comparable form."""
  try:
    p = build_pool_reshard_plan(src_pools, dst_pools, tags, dst_ids, decls, **kw)
    prod = {"schedules": {u: [(e.src_block_id, e.dst_block_id, e.src_offset_bytes,
                               e.dst_offset_bytes, e.size_bytes, e.pool_group) for e in es]
                          for u, es in p.schedules.items()},
            "groups": [dict(pool_indices=g.pool_indices, dst_device_block_ids=g.dst_device_block_ids,
                            expected_pushes=g.expected_pushes,
                            dst_expected_extent_bytes=g.dst_expected_extent_bytes,
                            order_rank=g.order_rank) for g in p.pool_groups],
            "src_units": p.src_units, "transfer_pool_indices": p.transfer_pool_indices}
  except ValueError as e:
    prod = {"error": str(e)}
  try:
    o = opr.build_plan([[x.to_dict() for x in u] for u in src_pools],
                       [x.to_dict() for x in dst_pools], list(tags), list(dst_ids),
                       [(u, to_oracle(r)) for u, r in decls],
                       dst_block_counts=kw.get("dst_block_counts"),
                       dst_skip_bytes=kw.get("dst_skip_bytes"),
                       parallelism=kw.get("parallelism"), ranks=kw.get("transfer_ranks"),
                       unit_parallelism=kw.get("transfer_parallelism"),
                       unit_names=kw.get("unit_names"))
  except opr.PlanError as e:
    o = {"error": str(e)}
  return prod, o


P1024 = [make_pool(1024, 1024, 16)]


def test_full_pool_reshard_flow():  # reshard_service_test.cc:288-318
  prod, orc = both([P1024, P1024], P1024, ["fa"], [7, 9],
                   [(0, reg([3], [(0, 0, 0, 0, 1024)])), (1, reg([5], [(0, 0, 1, 0, 512)]))],
                   transfer_parallelism=[2, 2])
  assert prod == orc
  g = prod["groups"][0]
  assert g["expected_pushes"] == 2 and g["dst_expected_extent_bytes"] == (1024, 512)
  assert len(prod["schedules"][0]) == 1 and len(prod["schedules"][1]) == 1


def test_global_space_spans_split_at_page_boundaries():  # :339-380
  prod, orc = both([P1024, P1024], P1024, ["fa"], [7, 9],
                   [(0, reg([3], [(0, 0, 0, 512, 1024)], version=1)),
                    (1, reg([5], [(0, 0, 0, 0, 512)]))], transfer_parallelism=[2, 2])
  assert prod == orc
  assert prod["groups"][0]["dst_expected_extent_bytes"] == (1024, 512)
  e0, e1 = prod["schedules"][0]
  assert (e0[1], e0[3], e0[4]) == (7, 512, 512)
  assert (e1[1], e1[3], e1[4]) == (9, 0, 512)


def test_clip_drops_trims_and_rebases_global_spans():  # :382-438
  prod, orc = both([P1024, P1024], P1024, ["fa"], [9],
                   [(0, reg([3], [(0, 0, 0, 512, 1024)], version=1)),
                    (1, reg([5, 6], [(0, 0, 0, 0, 512), (1, 0, 0, 1536, 512)], version=1))],
                   transfer_parallelism=[2, 2], dst_skip_bytes=[1024])
  assert prod == orc
  g = prod["groups"][0]
  assert g["expected_pushes"] == 2 and g["dst_expected_extent_bytes"] == (1024,)
  assert prod["schedules"][0] == [(3, 9, 512, 0, 512, 0)]
  assert prod["schedules"][1] == [(6, 9, 0, 512, 512, 0)]


@pytest.mark.parametrize("skip,needle", [([512], "whole multiple"), ([1024, 0], "align 1:1"),
                                         ([1024], "removes the entire tag"), ([0], None)])
def test_clip_validation_fails_closed(skip, needle):  # :440-473
  prod, orc = both([P1024], P1024, ["fa"], [9],
                   [(0, reg([3], [(0, 0, 0, 0, 1024)], version=1))], dst_skip_bytes=skip)
  assert prod == orc
  if needle is None:
    assert "error" not in prod
  else:
    assert needle in prod["error"]


def test_clip_rejects_page_indexed_declarations():  # :475-487
  prod, orc = both([P1024], P1024, ["fa"], [9], [(0, reg([3], [(0, 0, 0, 0, 1024)]))],
                   dst_skip_bytes=[1024])
  assert prod == orc and "destination-page-agnostic" in prod["error"]


def _random_request(rng):
  nu = rng.randint(1, 3)
  tags = ["fa"] if rng.random() < 0.7 else ["fa", "ssm"]
  src_pools, dst_pools = [], []
  geo = {}
  for t in ["fa", "ssm"]:
    # live geometry per side: sparse regions make TranslateLiveCopy split
    su = rng.choice([16, 32, 48])
    du = rng.choice([16, 24, 64])
    sn, dn = rng.randint(2, 6), rng.randint(1, 4)
    s_live, d_live = su * sn, du * dn
    geo[t] = (su, sn, du, dn, s_live, d_live)
  for t in ["fa", "ssm"]:
    su, sn, du, dn, _, _ = geo[t]
    sstride = su * sn + rng.choice([0, 16])
    src_pools.append(PoolSpec(t, 0, 0, su * 2 * sn + 64, 12,
                              (RegionSpec("r", 8, su * 2, su, sn, 1),), "bf16"))
    dst_pools.append(PoolSpec(t, 1, 0, du * dn + 32, 10, (RegionSpec("r", 0, du, du, dn, 1),),
                              "bf16"))
    del sstride
  decls, dst_ids, counts = [], [], []
  for t in tags:
    _, _, _, _, s_live, d_live = geo[t]
    k = rng.randint(1, 3)
    ids = rng.sample(range(10), k)
    dst_ids += ids
    counts.append(k)
    total = k * d_live - rng.choice([0, 0, rng.randrange(1, d_live)])
    cuts = sorted(rng.sample(range(1, total), min(total - 1, rng.randint(0, 5))))
    edges = [0] + cuts + [total]
    per_unit = {}
    for a, b in zip(edges, edges[1:]):
      u = rng.randrange(nu)
      size = b - a
      if size > s_live:
        # split big pieces into source-sized spans
        o = a
        while o < b:
          n = min(s_live, b - o)
          per_unit.setdefault(u, []).append((o, n))
          o += n
      else:
        per_unit.setdefault(u, []).append((a, size))
    for u, pieces in per_unit.items():
      version = rng.choice([0, 1])
      spans, blocks = [], []
      for (goff, size) in pieces:
        blocks.append(rng.randrange(12))
        soff = rng.randrange(0, s_live - size + 1)
        if version == 1:
          spans.append((len(blocks) - 1, soff, 0, goff, size))
        else:
          # page-indexed: split at destination pages ourselves
          o = goff
          left = size
          while left:
            page, inp = divmod(o, d_live)
            take = min(left, d_live - inp)
            spans.append((len(blocks) - 1, soff + (o - goff), page, inp, take))
            o += take
            left -= take
      r = reg(blocks, spans, version=version, tag=t)
      # occasional faults
      x = rng.random()
      if x < 0.05 and len(r.spans) > 1:
        r.spans = r.spans[1:]                      # gap
      elif x < 0.10:
        r.spans = list(r.spans) + [r.spans[0]]     # overlap
      elif x < 0.13:
        r.declared_bytes = r.declared() + 1        # totals disagree
      elif x < 0.15:
        r.block_ids = list(r.block_ids[:-1]) + [99]  # source id out of range
      decls.append((u, r))
  kw = dict(transfer_parallelism=[rng.choice([1, 2])] * nu,
            transfer_ranks=rng.sample(range(nu), nu))
  if len(tags) > 1 or rng.random() < 0.3:
    kw["dst_block_counts"] = counts
  if rng.random() < 0.1:
    kw["parallelism"] = 3
  return [list(src_pools) for _ in range(nu)], dst_pools, tags, dst_ids, decls, kw


def test_product_matches_oracle_on_random_requests():
  rng = random.Random(11)
  n_ok = n_err = 0
  for _ in range(300):
    src, dst, tags, ids, decls, kw = _random_request(rng)
    prod, orc = both(src, dst, tags, ids, decls, **kw)
    assert prod == orc, (tags, ids, kw, prod, orc)
    if "error" in prod:
      n_err += 1
    else:
      n_ok += 1
  assert n_ok > 50 and n_err > 20


def test_c3_handoff_as_pool_spans_equals_relayout():
  rng = np.random.default_rng(3)
  n_st, n_seqs, T, H, HB = 3, 2, 256, 2, 32
  sbps, dbps = T // 16, T // 64
  st = rng.permutation(n_seqs * sbps + 3)[:n_seqs * sbps].reshape(n_seqs, sbps).astype(np.int32)
  dt = rng.permutation(n_seqs * dbps + 2)[:n_seqs * dbps].reshape(n_seqs, dbps).astype(np.int32)
  src_pools, dst_pools, dst_ids, r = workloads.handoff_pool_plan_inputs(n_st, st, dt, H, HB)
  plan = build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids, [(0, r)])
  assert plan.pool_groups[0].dst_expected_extent_bytes == (64 * H * HB,) * (n_seqs * dbps)
  sbb, dbb = 16 * H * HB, 64 * H * HB
  src = [rng.integers(0, 256, (int(st.max()) + 1) * sbb, dtype=np.uint8) for _ in range(n_st)]
  got = [np.zeros((int(dt.max()) + 1) * dbb, np.uint8) for _ in range(n_st)]
  o_plan = {"schedules": {u: [(e.src_block_id, e.dst_block_id, e.src_offset_bytes,
                               e.dst_offset_bytes, e.size_bytes, e.pool_group) for e in es]
                          for u, es in plan.schedules.items()},
            "groups": [{"pool_indices": g.pool_indices} for g in plan.pool_groups]}
  opr.apply_plan(o_plan, 0, [p.to_dict() for p in src_pools], [p.to_dict() for p in dst_pools],
                 src, got)
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  for s in range(n_st):
    want = np.zeros_like(got[s]).reshape(-1, dbb)
    ors.relayout(src[s].reshape(-1, sbb), want, sg, dg, st, dt, T)
    np.testing.assert_array_equal(got[s], want.reshape(-1))


GOLDEN = Path(__file__).resolve().parent / "golden" / "pool_reshard_plans.json"


def _golden_case(case, keys):
  pk, rk = keys
  pool = lambda c: coerce_pool_spec(dict(zip(pk, c[:-1]),
                                         regions=[dict(zip(rk, r)) for r in c[-1]]))
  r = case["request"]
  nu = r["n_units"]
  src = [[pool(p) for p in r["src_pools"]] for _ in range(nu)]
  dst = [pool(p) for p in r["dst_pools"]]
  decls = [(u, PoolSpanRegistration(d["tag"], d["block_ids"], [PoolByteSpan(*sp) for sp in d["spans"]],
                                    d["declared_bytes"], d["dst_space_version"]))
           for u, d in r["decls"]]
  # the reference's units are RaidenId("src", "<u>", "kv", 0): messages name them so
  names = [f"RaidenId(job_name='src', job_replica_id='{u}', data_name='kv', data_replica_idx=0)"
           for u in range(nu)]
  kw = dict(dst_block_counts=r["dst_block_counts"], dst_skip_bytes=r["dst_skip_bytes"],
            parallelism=r["parallelism"], transfer_ranks=r["transfer_ranks"],
            transfer_parallelism=r["transfer_parallelism"], unit_names=names)
  return src, dst, r["tags"], r["dst_ids"], decls, kw


def test_reference_planning_flow_golden():
  g = json.loads(GOLDEN.read_text())
  keys = (g["pool_keys"], g["region_keys"])
  stages = {}
  for i, case in enumerate(g["cases"]):
    ref = case["reference"]
    src, dst, tags, ids, decls, kw = _golden_case(case, keys)
    prod, orc = both(src, dst, tags, ids, decls, **kw)
    assert prod == orc, (i, prod, orc)
    if not ref["ok"]:
      assert prod == {"error": ref["message"]}, (i, ref, prod)
      stages[ref["stage"]] = stages.get(ref["stage"], 0) + 1
      continue
    assert "error" not in prod, (i, prod)
    assert prod["src_units"] == ref["src_units"], i
    assert list(prod["transfer_pool_indices"]) == ref["transfer_pool_indices"], i
    assert {str(u): [list(e) for e in es] for u, es in prod["schedules"].items()} == \
        ref["schedules"], i
    assert [dict(g_, pool_indices=list(g_["pool_indices"]),
                 dst_device_block_ids=list(g_["dst_device_block_ids"]),
                 dst_expected_extent_bytes=list(g_["dst_expected_extent_bytes"]))
            for g_ in prod["groups"]] == ref["groups"], i
    p = build_pool_reshard_plan(src, dst, tags, ids, decls, **kw)
    assert (p.expected_block_count, p.parallelism, p.expected_pushes_per_pool) == \
        (ref["expected_block_count"], ref["parallelism"], ref["expected_pushes_per_pool"]), i
  # every step of the reference's flow rejects some requests
  assert set(stages) == {"register_unit", "register_spans", "plan"}, stages
  assert sum(c["reference"]["ok"] for c in g["cases"]) > 150


def test_default_parallelism_is_the_unit_count():
  """Units without explicit transfer_parallelism / ranks register as ranks
  0..n-1 of n (a registration the reference accepts)."""
  p = build_pool_reshard_plan([P1024, P1024], P1024, ["fa"], [7, 9],
                              [(0, reg([3], [(0, 0, 0, 0, 1024)])),
                               (1, reg([5], [(0, 0, 1, 0, 512)]))])
  assert p.parallelism == 2 and p.pool_groups[0].expected_pushes == 2
  with pytest.raises(ValueError, match="transfer_rank must be less than transfer_parallelism"):
    build_pool_reshard_plan([P1024, P1024], P1024, ["fa"], [7, 9],
                            [(0, reg([3], [(0, 0, 0, 0, 1024)]))], transfer_parallelism=[1, 1])


@pytest.mark.parametrize("unit", [-1, 2])
def test_declaration_of_an_unknown_unit_is_rejected(unit):
  """Register for a unit the request does not have fails in the reference
  ("Work unit is not registered", request_block_registry.cc:266-268)."""
  prod, orc = both([P1024, P1024], P1024, ["fa"], [7, 9],
                   [(0, reg([3], [(0, 0, 0, 0, 1024)])), (unit, reg([5], [(0, 0, 1, 0, 1024)]))])
  assert prod == orc == {"error": f"Work unit is not registered: src unit {unit}"}

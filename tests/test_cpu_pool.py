"""Pool geometry on the CPU: oracle pin, product parity, Python surface.

* the oracle (oracle/pool_layout.py) against the fixtures of
  tests/golden/pool_layout.json: the reference unit test's known answers
  (tpu_sync/kv_cache/pool_layout_test.cc) and random requests answered by the
  reference's own pool_layout.cc (tests/golden/make_pool_golden.py);
* the product (tpu_sync_b200.pool_layout over the C ABI) against the same
  fixtures, codes and messages included;
* product vs oracle on fresh seeded random pools;
* the reference Python surface (RegionSpec / PoolSpec properties, coerce_*).

No GPU needed: the geometry is host code in the native library.
"""

import json
import random
from pathlib import Path

import pytest

from oracle import pool_layout as opl
from tpu_sync_b200 import pool_layout as pl

GOLDEN = json.loads((Path(__file__).parent / "golden" / "pool_layout.json").read_text())


def _spec(p):
  return pl.coerce_pool_spec(p)


def run_oracle(case):
  op = case["op"]
  try:
    if op == "ext":
      return {"ok": [list(e) for e in opl.copy_extents(case["pool"], case["ids"])]}
    if op == "segs":
      return {"ok": [list(s) for s in opl.live_segments(case["pool"])]}
    if op == "val":
      opl.validate_pool(case["pool"], case["storage_bytes"])
      return {"ok": True}
    if op == "rval":
      opl.validate_region(case["region"], case["slot"])
      return {"ok": True}
    if op == "end":
      return {"ok": opl.storage_extent_end(case["pool"])}
    if op == "p2l":
      return {"ok": list(opl.physical_to_logical(case["segs"], case["off"], case["size"]))}
    if op == "xl":
      return {"ok": [list(c) for c in opl.translate_live_copy(
          case["src_segs"], case["dst_segs"], case["src_off"], case["dst_off"], case["size"])]}
    if op == "cover":
      return {"ok": int(opl.regions_cover_range(case["regions"], case["start"], case["end"]))}
  except opl.PoolError as e:
    return {"code": e.code, "message": e.message}
  raise ValueError(op)


def run_product(case):
  op = case["op"]
  try:
    if op == "ext":
      return {"ok": [list(e) for e in pl.compute_pool_block_copy_extents(_spec(case["pool"]),
                                                                         case["ids"])]}
    if op == "segs":
      return {"ok": [list(s) for s in pl.expand_pool_live_segments(_spec(case["pool"]))]}
    if op == "val":
      sb = case["storage_bytes"]
      _spec(case["pool"]).validate(None if sb < 0 else sb)
      return {"ok": True}
    if op == "rval":
      pl.coerce_region_spec(case["region"]).validate(case["slot"])
      return {"ok": True}
    if op == "end":
      import ctypes
      from tpu_sync_b200 import _native
      keep = pl._pool_c(_spec(case["pool"]))
      end = ctypes.c_int64()
      _native.check(_native.lib().ts_pool_geometry(ctypes.byref(keep[0]), ctypes.byref(end),
                                                   None, None))
      return {"ok": end.value}
    if op == "p2l":
      return {"ok": list(pl.physical_live_range_to_logical(case["segs"], case["off"],
                                                           case["size"]))}
    if op == "xl":
      return {"ok": [list(c) for c in pl.translate_live_copy(
          case["src_segs"], case["dst_segs"], case["src_off"], case["dst_off"], case["size"])]}
    if op == "cover":
      return {"ok": int(pl.regions_cover_range([pl.coerce_region_spec(r) for r in case["regions"]],
                                               case["start"], case["end"]))}
  except pl.PoolLayoutError as e:
    return {"code": e.code, "message": str(e)}
  raise ValueError(op)


def check_expect(got, want, exact_message):
  if "ok" in want:
    assert got.get("ok") == want["ok"], (got, want)
  else:
    assert got.get("code") == want["code"], (got, want)
    if exact_message:
      assert got["message"] == want["message"], (got, want)
    else:
      assert want.get("substr", "") in got["message"], (got, want)


@pytest.mark.parametrize("runner", [run_oracle, run_product], ids=["oracle", "product"])
def test_known_answers_of_reference_unit_test(runner):
  for case in GOLDEN["kat"]:
    check_expect(runner(case), case["expect"], exact_message=False)


@pytest.mark.parametrize("runner", [run_oracle, run_product], ids=["oracle", "product"])
def test_reference_answered_random_cases(runner):
  for case in GOLDEN["random"]:
    check_expect(runner(case), case["expect"], exact_message=True)


def _rand_pool(rng):
  stride = rng.choice([64, 96, 256, 1000, 2048])
  regs = []
  for i in range(rng.randint(1, 4)):
    unit = rng.choice([1, 2, 16, 24, 64])
    ups = rng.choice([1, 2])
    n = rng.choice([0, 1, 2, 4, 9])
    regs.append(opl_region(f"r{i}", rng.randrange(0, stride), unit * ups + rng.choice([0, 8, -1, 40]),
                           unit, n, ups))
  return {"tag": "t", "storage_index": 0, "base_offset_bytes": rng.choice([0, 16, 3]),
          "block_stride_bytes": stride, "num_blocks": rng.randint(1, 16), "regions": regs,
          "dtype_tag": ""}


def opl_region(name, off, stride, unit, n, ups):
  return {"name": name, "offset_bytes": off, "stride_bytes": stride, "unit_bytes": unit,
          "num_units": n, "units_per_stride": ups}


def test_product_matches_oracle_on_fresh_random_pools():
  rng = random.Random(7)
  for _ in range(600):
    p = _rand_pool(rng)
    ids = [rng.randrange(-1, p["num_blocks"] + 1) for _ in range(rng.randint(0, 10))]
    for case in ({"op": "ext", "pool": p, "ids": ids}, {"op": "segs", "pool": p},
                 {"op": "val", "pool": p, "storage_bytes": rng.randrange(-1, 40000)},
                 {"op": "end", "pool": p}):
      a, b = run_oracle(case), run_product(case)
      assert a == b, (case, a, b)


def test_python_surface_properties_and_coercion():
  r = pl.RegionSpec("key", 0, 100, 10, 5, 2)
  assert r.live_bytes == 100 and r.extent_end_bytes == 420
  p = pl.PoolSpec("pool0", 0, 0, 1000, 10, (r,))
  assert p.storage_extent_end_bytes == 9420 and p.live_bytes_per_block == 100
  d = p.to_dict()
  assert pl.coerce_pool_spec(d) == p
  assert p.to_native_tuple() == ("pool0", 0, 0, 1000, 10, [("key", 0, 100, 10, 5, 2)], "")
  with pytest.raises(ValueError, match="exceeds slot bytes"):
    r.validate(400)
  with pytest.raises(ValueError, match="must contain at least one region"):
    pl.PoolSpec("p", 0, 0, 64, 1, ()).validate()
  with pytest.raises(ValueError, match="storage_index must be >= 0"):
    pl.PoolSpec("p", -1, 0, 64, 1, (r,)).validate()
  with pytest.raises(ValueError, match="out of range"):
    pl.compute_pool_block_copy_extents(p, [10])
  with pytest.raises(TypeError):
    pl.coerce_pool_spec({"tag": "x", "storage_index": 0, "block_stride_bytes": 8,
                         "num_blocks": 1, "regions": 5})


def test_extent_capacity_protocol_and_large_expansion():
  # 4096 sparse units per block x 8 blocks: far beyond the first output guess
  r = pl.RegionSpec("u", 0, 32, 16, 4096)
  p = pl.PoolSpec("big", 0, 0, 131072, 8, (r,))
  ext = pl.compute_pool_block_copy_extents(p, list(range(8)))
  assert len(ext) == 8 * 4096
  assert ext[:2] == [(0, 16), (32, 16)] and ext[-1] == (7 * 131072 + 4095 * 32, 16)
  assert ext == [tuple(e) for e in opl.copy_extents(
      {"tag": "big", "num_blocks": 8, "block_stride_bytes": 131072, "base_offset_bytes": 0,
       "regions": [opl_region("u", 0, 32, 16, 4096, 1)]}, list(range(8)))]

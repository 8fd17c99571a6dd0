"""Generates tests/golden/pool_layout.json: pool-geometry fixtures.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_pool_golden.py

Two parts:

* "kat": the known answers of the reference's own unit test
  tpu_sync/kv_cache/pool_layout_test.cc (line ranges cited per case),
  written here as data;
* "random": seeded random requests answered by the REFERENCE
  tpu_sync/kv_cache/pool_layout.cc itself, compiled by oracle/build_ref.py
  into oracle/_ref/pool_ref (valid and invalid geometries, out-of-range ids,
  overlapping regions, copies that cross padding).

The output is committed; tests never read the reference.
"""

from __future__ import annotations

import json
import random
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "pool_layout.json"
sys.path.insert(0, str(ROOT))


def region(name, off, stride, unit, n, ups=1):
  return {"name": name, "offset_bytes": off, "stride_bytes": stride, "unit_bytes": unit,
          "num_units": n, "units_per_stride": ups}


def pool(tag, storage, base, stride, nb, regions, dtype=""):
  return {"tag": tag, "storage_index": storage, "base_offset_bytes": base,
          "block_stride_bytes": stride, "num_blocks": nb, "regions": regions, "dtype_tag": dtype}


VALID_REGION = region("key", 0, 100, 10, 5, 2)                 # pool_layout_test.cc:35-44
VALID_POOL = pool("pool0", 0, 0, 1000, 10, [VALID_REGION])     # :46-55


def kat_cases():
  c = []
  c.append({"src": "pool_layout_test.cc:62-66", "op": "end", "pool": VALID_POOL,
            "expect": {"ok": 9420}})
  c.append({"src": "pool_layout_test.cc:73-77", "op": "rval", "region": VALID_REGION,
            "slot": 400, "expect": {"code": 3, "substr": "exceeds slot bytes"}})
  c.append({"src": "pool_layout_test.cc:79-84", "op": "rval",
            "region": dict(VALID_REGION, offset_bytes=-1), "slot": 1000, "expect": {"code": 3}})
  c.append({"src": "pool_layout_test.cc:86-89", "op": "val", "pool": VALID_POOL,
            "storage_bytes": 10000, "expect": {"ok": True}})
  c.append({"src": "pool_layout_test.cc:91-100", "op": "val", "pool": VALID_POOL,
            "storage_bytes": 9420, "expect": {"ok": True}})
  c.append({"src": "pool_layout_test.cc:91-100", "op": "val", "pool": VALID_POOL,
            "storage_bytes": 9419, "expect": {"code": 3, "substr": "exceeds storage bytes"}})
  gdn = pool("gdn.ssm.g0", 0, 65536, 4194304, 16, [region("ssm", 0, 2097152, 2097152, 1)])
  c.append({"src": "pool_layout_test.cc:102-123", "op": "end", "pool": gdn,
            "expect": {"ok": 65077248}})
  c.append({"src": "pool_layout_test.cc:102-123", "op": "val", "pool": gdn,
            "storage_bytes": 67108864, "expect": {"ok": True}})
  r1, r2 = region("r1", 0, 20, 10, 2), region("r2", 10, 20, 10, 2)
  c.append({"src": "pool_layout_test.cc:139-162", "op": "cover", "regions": [r1, r2],
            "start": 0, "end": 40, "expect": {"ok": 1}})
  c.append({"src": "pool_layout_test.cc:139-162", "op": "cover", "regions": [r1, r2],
            "start": 0, "end": 41, "expect": {"ok": 0}})
  c.append({"src": "pool_layout_test.cc:164-182", "op": "ext",
            "pool": dict(VALID_POOL, regions=[region("payload", 0, 1000, 1000, 1)]),
            "ids": [0, 1, 3, 4, 5], "expect": {"ok": [[0, 2000], [3000, 3000]]}})
  pad = pool("pool0", 0, 8, 128, 2, [region("payload", 0, 32, 16, 2)])
  c.append({"src": "pool_layout_test.cc:184-210", "op": "val", "pool": pad,
            "storage_bytes": 184, "expect": {"ok": True}})
  c.append({"src": "pool_layout_test.cc:184-210", "op": "ext", "pool": pad, "ids": [0, 1],
            "expect": {"ok": [[8, 16], [40, 16], [136, 16], [168, 16]]}})
  fa = pool("fa", 0, 0, 2162688, 1,
            [region("fa", h * 540672, 1024, 512, 256, 2) for h in range(4)])
  c.append({"src": "pool_layout_test.cc:212-241", "op": "val", "pool": fa,
            "storage_bytes": 1884160, "expect": {"ok": True}})
  c.append({"src": "pool_layout_test.cc:212-241", "op": "ext", "pool": fa, "ids": [0],
            "expect": {"ok": [[h * 540672, 262144] for h in range(4)]}})
  c.append({"src": "pool_layout_test.cc:243-253", "op": "segs", "pool": VALID_POOL,
            "expect": {"ok": [[u * 20, u * 100, 20] for u in range(5)]}})
  ab = dict(VALID_POOL, regions=[region("a", 0, 20, 20, 1), region("b", 20, 30, 30, 1)])
  c.append({"src": "pool_layout_test.cc:255-282", "op": "segs", "pool": ab,
            "expect": {"ok": [[0, 0, 50]]}})
  ov = dict(VALID_POOL, regions=[region("a", 0, 20, 20, 1), region("b", 10, 30, 30, 1)])
  c.append({"src": "pool_layout_test.cc:284-287", "op": "segs", "pool": ov,
            "expect": {"code": 3, "substr": "overlapping live regions"}})
  segs = [[u * 20, u * 100, 20] for u in range(5)]
  c.append({"src": "pool_layout_test.cc:289-299", "op": "p2l", "segs": segs, "off": 105,
            "size": 10, "expect": {"ok": [25, 35]}})
  c.append({"src": "pool_layout_test.cc:301-306", "op": "p2l", "segs": segs, "off": 15,
            "size": 10, "expect": {"code": 3, "substr": "crosses padding"}})
  return c


# -- reference driver protocol (oracle/ref_pool_driver.cc) -------------------

def _s(x):
  return x if x else "-"


def enc_region(r):
  return f"{_s(r['name'])} {r['offset_bytes']} {r['stride_bytes']} {r['unit_bytes']} " \
         f"{r['num_units']} {r['units_per_stride']}"


def enc_pool(p):
  regs = " ".join(enc_region(r) for r in p["regions"])
  return (f"{_s(p['tag'])} {p['storage_index']} {p['base_offset_bytes']} "
          f"{p['block_stride_bytes']} {p['num_blocks']} {_s(p['dtype_tag'])} "
          f"{len(p['regions'])} {regs}").strip()


def enc_segs(segs):
  return f"{len(segs)} " + " ".join(f"{a} {b} {c}" for a, b, c in segs)


def request(case) -> str:
  op = case["op"]
  if op == "ext":
    return f"ext {enc_pool(case['pool'])} {len(case['ids'])} " + " ".join(map(str, case["ids"]))
  if op == "segs":
    return f"segs {enc_pool(case['pool'])}"
  if op == "val":
    return f"val {enc_pool(case['pool'])} {case['storage_bytes']}"
  if op == "end":
    return f"end {enc_pool(case['pool'])}"
  if op == "p2l":
    return f"p2l {enc_segs(case['segs'])} {case['off']} {case['size']}"
  if op == "xl":
    return (f"xl {enc_segs(case['src_segs'])} {enc_segs(case['dst_segs'])} {case['src_off']} "
            f"{case['dst_off']} {case['size']}")
  if op == "cover":
    return (f"cover {len(case['regions'])} " + " ".join(enc_region(r) for r in case["regions"]) +
            f" {case['start']} {case['end']}")
  raise ValueError(op)


def parse(op, line: str):
  parts = line.strip().split(" ")
  if parts[0] == "ERR":
    return {"code": int(parts[1]), "message": " ".join(parts[2:])}
  nums = [int(x) for x in parts[1:]]
  if op == "val":
    return {"ok": True}
  if op in ("end",):
    return {"ok": nums[0]}
  if op == "cover":
    return {"ok": nums[0]}
  if op == "p2l":
    return {"ok": nums}
  if op == "ext":
    return {"ok": [nums[i:i + 2] for i in range(0, len(nums), 2)]}
  return {"ok": [nums[i:i + 3] for i in range(0, len(nums), 3)]}


def random_region(rng, i, stride):
  unit = rng.choice([1, 4, 16, 32, 48, 64, 100])
  ups = rng.choice([1, 1, 1, 2, 3])
  n = rng.choice([0, 1, 1, 2, 3, 5, 8])
  packed = unit * ups
  rstride = packed + rng.choice([0, 0, 4, 16, packed, -1])
  off = rng.randrange(0, max(stride // 2, 1))
  return region(f"r{i}", off, rstride, unit, n, ups)


def random_pool(rng):
  stride = rng.choice([64, 128, 256, 500, 1000, 4096])
  regs = [random_region(rng, i, stride) for i in range(rng.randint(1, 3))]
  return pool(rng.choice(["p", "fa", "kv"]), 0, rng.choice([0, 0, 8, 100]), stride,
              rng.randint(1, 8), regs, rng.choice(["", "bf16"]))


def random_cases(rng, n):
  out = []
  for _ in range(n):
    p = random_pool(rng)
    kind = rng.choice(["ext", "ext", "segs", "val", "end", "xl", "p2l", "cover"])
    if kind == "ext":
      ids = [rng.randrange(-1, p["num_blocks"] + 1) if rng.random() < 0.1
             else rng.randrange(0, p["num_blocks"]) for _ in range(rng.randint(0, 6))]
      out.append({"op": "ext", "pool": p, "ids": ids})
    elif kind == "segs":
      out.append({"op": "segs", "pool": p})
    elif kind == "val":
      out.append({"op": "val", "pool": p,
                  "storage_bytes": rng.choice([-1, p["block_stride_bytes"] * p["num_blocks"],
                                               rng.randrange(0, 20000)])})
    elif kind == "end":
      out.append({"op": "end", "pool": p})
    elif kind == "cover":
      out.append({"op": "cover", "regions": p["regions"], "start": rng.randrange(0, 64),
                  "end": rng.randrange(0, 600)})
    else:
      # segments of two well-formed pools (tightly generated so most are valid)
      segs = []
      for _k in range(2):
        cur, logical, s = rng.randrange(0, 16), 0, []
        for _j in range(rng.randint(1, 5)):
          size = rng.randint(1, 40)
          s.append([logical, cur, size])
          logical += size
          cur += size + rng.choice([0, 0, 8, 24])
        segs.append(s)
      total = min(sum(x[2] for x in segs[0]), sum(x[2] for x in segs[1]))
      if kind == "xl":
        so = rng.randrange(0, total)
        size = rng.randint(1, total - so + rng.choice([0, 0, 3]))
        out.append({"op": "xl", "src_segs": segs[0], "dst_segs": segs[1], "src_off": so,
                    "dst_off": rng.randrange(0, max(total - size + 1, 1)), "size": size})
      else:
        last = segs[0][-1]
        end = last[1] + last[2]
        off = rng.randrange(0, end + 2)
        out.append({"op": "p2l", "segs": segs[0], "off": off, "size": rng.randint(0, 30)})
  return out


def main():
  from oracle import build_ref
  exe = build_ref.build_pool(force=True)
  if exe is None:
    raise SystemExit("reference checkout not found; cannot build oracle/_ref/pool_ref")
  rng = random.Random(20260)
  cases = random_cases(rng, 400)
  req = "".join(request(c) + "\n" for c in cases)
  res = subprocess.run([str(exe)], input=req, capture_output=True, text=True, check=True)
  lines = res.stdout.splitlines()
  assert len(lines) == len(cases)
  for c, line in zip(cases, lines):
    c["expect"] = parse(c["op"], line)
  kats = kat_cases()
  # The known answers must hold for the compiled reference too.
  req = "".join(request(c) + "\n" for c in kats if c["op"] != "rval")
  lines = subprocess.run([str(exe)], input=req, capture_output=True, text=True,
                         check=True).stdout.splitlines()
  for c, line in zip([c for c in kats if c["op"] != "rval"], lines):
    got = parse(c["op"], line)
    want = c["expect"]
    if "ok" in want:
      assert got.get("ok") == want["ok"], (c, got)
    else:
      assert got.get("code") == want["code"] and want.get("substr", "") in got["message"], (c, got)
  OUT.write_text(json.dumps({"kat": kats, "random": cases}, separators=(",", ":")) + "\n")
  n_err = sum("code" in c["expect"] for c in cases)
  print(f"wrote {OUT}: {len(kats)} known answers, {len(cases)} random ({n_err} errors)")


if __name__ == "__main__":
  main()

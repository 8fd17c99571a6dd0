"""Pins the CPU oracle before it is trusted as the checker.

* fp8 e4m3 encoder (written from the format definition) against ml_dtypes and
  torch on every finite fp32 value representable as bf16 in range;
* the byte-level manager model on the reference's own heterogeneous
  block-size scenario (tpu_sync/frameworks/torch/kv_cache_manager_test.py:206-275)
  and round trip (tpu_sync/benchmarks/perf_core.py:112-142);
* the planner restatement against plans produced by the reference planner
  (tests/golden/reshard_plans.json, made by tests/golden/make_golden.py).
"""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import kv_blocks as ref
from oracle import reshard as ors

GOLDEN = Path(__file__).resolve().parent / "golden" / "reshard_plans.json"


def all_bf16_finite():
  bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
  v = ofp8.bf16_bits_to_f32(bits)
  return v[np.isfinite(v)]


def test_e4m3_encoder_matches_ml_dtypes_in_range():
  ml_dtypes = pytest.importorskip("ml_dtypes")
  v = all_bf16_finite()
  v = v[np.abs(v) <= 448]
  ours = ofp8.e4m3_encode(v)
  theirs = v.astype(ml_dtypes.float8_e4m3fn).view(np.uint8)
  # ml_dtypes keeps the sign of zero results; so do we
  np.testing.assert_array_equal(ours, theirs)


def test_e4m3_encoder_matches_torch_in_range():
  v = all_bf16_finite()
  v = v[np.abs(v) <= 448]
  theirs = torch.from_numpy(v).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
  np.testing.assert_array_equal(ofp8.e4m3_encode(v), theirs)


def test_e4m3_saturates_and_decodes():
  big = np.array([448.0, 449.0, 463.9, 464.0, 1e6, np.inf, -np.inf, -500.0], np.float32)
  enc = ofp8.e4m3_encode(big)
  assert list(enc) == [0x7E, 0x7E, 0x7E, 0x7E, 0x7E, 0x7E, 0xFE, 0xFE]
  assert ofp8.e4m3_encode(np.array([np.nan], np.float32))[0] & 0x7F == 0x7F
  codes = np.arange(256, dtype=np.uint8)
  dec = ofp8.e4m3_decode(codes)
  finite = ~np.isnan(dec)
  np.testing.assert_array_equal(ofp8.e4m3_encode(dec[finite]), codes[finite])


def test_fp8_unit_roundtrip_error_bound():
  rng = np.random.default_rng(0)
  x = torch.from_numpy(rng.standard_normal(8192).astype(np.float32)).to(torch.bfloat16)
  bits = x.view(torch.int16).numpy().view(np.uint16)
  q, scale = ofp8.quantize_unit(bits)
  assert scale == np.float32(np.abs(x.float().numpy()).max()) / np.float32(448)
  back = ofp8.bf16_bits_to_f32(ofp8.dequantize_unit(q, scale))
  # e4m3 has 3 mantissa bits: relative error <= 2^-4 for normals
  err = np.abs(back - x.float().numpy())
  assert np.all(err <= np.abs(x.float().numpy()) * 2.0 ** -4 * 1.01 + scale * 2.0 ** -9)


def test_zero_unit_scale_is_one():
  q, scale = ofp8.quantize_unit(np.zeros(64, np.uint16))
  assert scale == 1.0 and not q.any()


def test_bf16_rne_matches_torch():
  rng = np.random.default_rng(1)
  v = np.concatenate([rng.standard_normal(100000).astype(np.float32) * 1e3,
                      np.array([0.0, -0.0, 1e38, -1e-38, np.inf, -np.inf], np.float32)])
  ours = ofp8.f32_to_bf16_bits_rne(v)
  theirs = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
  np.testing.assert_array_equal(ours, theirs)


def pattern(shape, layer):
  n = int(np.prod(shape))
  return (np.arange(n, dtype=np.float32).reshape(shape) + 1000.0 * (layer + 1))


def test_heterogeneous_block_sizes_model():
  """kv_cache_manager_test.py:206-275 on the byte model."""
  shapes = [(4, 128, 8), (4, 128, 2)]
  src = ref.RefKVManager([[pattern(s, l).view(np.uint8).reshape(-1)] for l, s in
                          enumerate(shapes)], dim0=4, host_blocks=4)
  dst_dev = [[np.zeros(int(np.prod(s)) * 4, np.uint8)] for s in shapes]
  dst = ref.RefKVManager(dst_dev, dim0=4, host_blocks=4)
  assert src.d2h([2], [2], [2]) == (ref.OK, "")
  for l in range(2):  # H2hWrite: copy host blocks 2..3 to the peer's host 0..1
    bb = src.layer_block_bytes(l)
    dst.host[l][0][:2 * bb] = src.host[l][0][2 * bb:4 * bb]
  assert dst.h2d([0], [2], [2]) == (ref.OK, "")
  for l, s in enumerate(shapes):
    got = dst.device[l][0].view(np.float32).reshape(s)
    np.testing.assert_array_equal(got[2:4], pattern(s, l)[2:4])
    np.testing.assert_array_equal(got[0:2], 0)


def test_round_trip_and_errors_model():
  dev = [[np.arange(8 * 64, dtype=np.uint8).copy()] for _ in range(2)]
  m = ref.RefKVManager(dev, dim0=8, host_blocks=8)
  assert m.d2h([0, 1, 2, 3], [0, 1, 2, 3]) == (ref.OK, "")
  assert m.h2d([0, 1, 2, 3], [4, 5, 6, 7]) == (ref.OK, "")
  np.testing.assert_array_equal(dev[0][0][:256], dev[0][0][256:])
  assert m.d2h([7], [8])[0] == ref.INVALID_ARGUMENT
  assert m.d2h([8], [0])[1] == "Copy range exceeds source device buffer size"
  assert m.h2d([0], [0], layer_idx=2) == (ref.OUT_OF_RANGE, ref.LAYER_RANGE)
  assert m.d2h([], []) == (ref.OK, "")


def test_planner_oracle_matches_reference_goldens():
  data = json.loads(GOLDEN.read_text())
  for case in data["slices"]:
    got = ors.compute_nd_shard_slices(case["global_shape"], case["mesh_shape"])
    assert [[list(d) for d in s] for s in got] == case["slices"]
  for case in data["plans"]:
    s_sl = ors.compute_nd_shard_slices(case["shape"], case["src_mesh"])
    d_sl = ors.compute_nd_shard_slices(case["shape"], case["dst_mesh"])
    pairs = []
    for i, s in enumerate(s_sl):
      for j, d in enumerate(d_sl):
        inter = ors.intersect_nd_slices(s, d)
        if inter is None:
          continue
        pairs.append({"src": i, "dst": j, "chunks": [list(c) for c in
                      ors.generate_strided_copy_chunks(s, d, inter, case["itemsize"])]})
    assert pairs == case["pairs"], case["param"]


def test_product_planner_matches_reference_goldens():
  from tpu_sync_b200 import reshard_plan as rp
  data = json.loads(GOLDEN.read_text())
  for case in data["slices"]:
    got = rp.shard_boxes(case["global_shape"], case["mesh_shape"])
    assert [[list(d) for d in b] for b in got] == case["slices"]
  for case in data["plans"]:
    sb = rp.shard_boxes(case["shape"], case["src_mesh"])
    db = rp.shard_boxes(case["shape"], case["dst_mesh"])
    pairs = []
    for i, s in enumerate(sb):
      for j, d in enumerate(db):
        inter = rp.box_intersection(s, d)
        if inter is not None:
          pairs.append({"src": i, "dst": j, "chunks": [list(c) for c in
                        rp.plan_bytes(s, d, inter, case["itemsize"])]})
    assert pairs == case["pairs"], case["param"]


def test_unit_shard_indices_match_reference_goldens():
  """_get_global_indices (raiden_controller.py:129-263), both restatements,
  against 1077 answers of the reference function itself."""
  from tpu_sync_b200 import reshard_plan as rp
  data = json.loads(GOLDEN.read_text())
  assert len(data["global_indices"]) > 1000
  for c in data["global_indices"]:
    args = (c["replica"], c["local"], c["var_mesh"], c["layout"], c["hosts"], c["spec"],
            c["axes"], c["unit_mesh"])
    want = [tuple(x) for x in c["out"]]
    assert ors.global_indices(*args) == want, c
    assert rp.shard_index_of_units(*args) == want, c


def test_replicated_source_dedup_matches_reference_test():
  """raiden_controller_test.py:1868-1960: 4 trainer units on a (fsdp=1, tp=4)
  mesh all hold layer_19.input_layernorm (2304,); 4 sampler units on a
  (fsdp=2, tp=2) mesh hold halves.  Every destination expects exactly one
  chunk for the layer and every destination peer gets exactly one push."""
  from tpu_sync_b200 import reshard_plan as rp
  sh = rp.slot_holders(4, [1], ["fsdp"], ["fsdp", "tp"], [1, 4])
  dh = rp.slot_holders(4, [2], ["fsdp"], ["fsdp", "tp"], [2, 2])
  assert sh == [0, 0, 0, 0] and dh == [0, 0, 1, 1]
  v = rp.VariableSpec("layer_19.input_layernorm", (2304,), (1,), (2,), 198, sh, dh)
  plan = rp.build_plan([v])
  per_dst = {}
  for (vi, s, d), cs in plan.chunks.items():
    per_dst[d] = per_dst.get(d, 0) + len(cs)
  assert per_dst == {0: 1, 1: 1, 2: 1, 3: 1}
  # holder d mod 4: each source pushes to one destination
  assert sorted((s, d) for (_, s, d) in plan.chunks) == [(0, 0), (1, 1), (2, 2), (3, 3)]
  raw = rp.build_plan([v], normalize_runs=False)
  want = ors.plan_with_replicas((2304,), (1,), (2,), sh, dh)
  assert {(s, d): cs for (_, s, d), cs in raw.chunks.items()} == want


def test_replicated_plans_product_matches_oracle():
  from tpu_sync_b200 import reshard_plan as rp
  rng = np.random.default_rng(21)
  for _ in range(200):
    rank = int(rng.integers(1, 4))
    shape = tuple(int(x) for x in rng.integers(3, 40, rank))
    sm = tuple(int(x) for x in rng.integers(1, 4, rank))
    dm = tuple(int(x) for x in rng.integers(1, 4, rank))
    ns, nd = int(np.prod(sm)), int(np.prod(dm))
    # every box held at least once, some several times, slots shuffled
    sh = list(range(ns)) + [int(x) for x in rng.integers(0, ns, int(rng.integers(0, 4)))]
    dh = list(range(nd)) + [int(x) for x in rng.integers(0, nd, int(rng.integers(0, 4)))]
    rng.shuffle(sh)
    rng.shuffle(dh)
    v = rp.VariableSpec("x", shape, sm, dm, 0, sh, dh)
    got = {(s, d): cs for (_, s, d), cs in rp.build_plan([v], normalize_runs=False).chunks.items()}
    assert got == ors.plan_with_replicas(shape, sm, dm, sh, dh)
    # every destination slot's box is covered exactly once
    dboxes = rp.shard_boxes(shape, dm)
    for d, b in enumerate(dh):
      hits = np.zeros(int(np.prod(rp.local_shape(dboxes[b]))), np.int64)
      for (s, dd), cs in got.items():
        if dd == d:
          for (so, do, size, ss, ds, cnt) in cs:
            for c in range(cnt):
              hits[do + c * ds: do + c * ds + size] += 1
      assert (hits == 1).all()


def test_plan_rejects_unheld_source_box():
  from tpu_sync_b200 import reshard_plan as rp
  with pytest.raises(ValueError, match="no source slot holds box 1"):
    rp.build_plan([rp.VariableSpec("x", (8,), (2,), (1,), 0, [0, 0], None)])
  with pytest.raises(ValueError, match="dst slot holds box 3 of 2"):
    rp.build_plan([rp.VariableSpec("x", (8,), (2,), (2,), 0, None, [0, 3])])


def test_planner_covers_every_destination_element_once():
  from tpu_sync_b200 import reshard_plan as rp, workloads
  for name, shape, split in workloads.llama3_8b_params()[:12]:
    small = tuple(max(8, d // 64) for d in shape)
    v = rp.VariableSpec(name, small, workloads.mesh_for(small, "fsdp", 4),
                        workloads.mesh_for(small, split, 4))
    plan = rp.build_plan([v])
    dboxes = rp.shard_boxes(small, v.dst_mesh)
    for d, box in enumerate(dboxes):
      n = int(np.prod(rp.local_shape(box)))
      hits = np.zeros(n, np.int64)
      for (vi, s, dd), chunks in plan.chunks.items():
        if dd != d:
          continue
        for (so, do, size, ss, ds, cnt) in chunks:
          for c in range(cnt):
            hits[do + c * ds: do + c * ds + size] += 1
      assert (hits == 1).all(), (name, d)


def test_normalized_plan_moves_same_elements():
  from tpu_sync_b200 import reshard_plan as rp
  v = rp.VariableSpec("x", (64, 48), (4, 1), (1, 1))
  raw = rp.build_plan([v], normalize_runs=False)
  norm = rp.build_plan([v])
  src = np.arange(64 * 48, dtype=np.float32)
  for key in raw.chunks:
    a = np.zeros(64 * 48, np.float32)
    b = np.zeros(64 * 48, np.float32)
    ors.apply_element_chunks(src, a, raw.chunks[key], False)
    ors.apply_element_chunks(src, b, norm.chunks[key], False)
    np.testing.assert_array_equal(a, b)


# ---------------------------------------------------------------------------
# C restatements used as the timed CPU baselines of C2 / C3
# ---------------------------------------------------------------------------

def test_c_e4m3_encoder_matches_oracle():
  from oracle import cpu_ref
  rng = np.random.default_rng(8)
  vals = np.concatenate([
      rng.standard_normal(20000).astype(np.float32) * np.float32(100),
      (rng.standard_normal(20000) * 2.0 ** rng.integers(-20, 10, 20000)).astype(np.float32),
      np.array([0.0, -0.0, 448.0, -448.0, 464.0, 465.0, 1e30, 2 ** -9, 2 ** -10, 3 * 2 ** -11,
                2 ** -6, 2 ** -6 - 2 ** -12, np.inf, -np.inf], np.float32)])
  want = ofp8.e4m3_encode(vals)
  got = np.array([cpu_ref.lib().oref_e4m3(float(v)) for v in vals], np.uint8)
  np.testing.assert_array_equal(got, want)


def test_c_extract_fp8_matches_oracle():
  from oracle import cpu_ref
  bits = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16)
  finite = bits[(bits & 0x7FFF) < 0x7F80]  # every finite bf16 bit pattern
  units = [np.zeros(8192, np.uint16) for _ in range(8)]
  for i, chunk in enumerate(np.array_split(finite, 8)):
    units[i][:chunk.size] = chunk
  rng = np.random.default_rng(3)
  for _ in range(40):
    amax_bits = int(rng.integers(1, 0x7F80))
    u = rng.integers(0, amax_bits + 1, 8192, dtype=np.uint32).astype(np.uint16)
    u |= (rng.integers(0, 2, 8192, dtype=np.uint32) << 15).astype(np.uint16)
    u[0] = amax_bits
    units.append(u)
  store = np.stack(units)                 # one storage, [blocks, 8192]
  ids = list(range(store.shape[0]))[::-1]
  payload, scales = ofp8.extract_fp8([store], ids)
  pitch, scale_off = 8192 + 16, 8192
  staging = np.zeros((len(ids), pitch), np.uint8)
  cpu_ref.extract_fp8([store], ids, staging, pitch, [0], scale_off, 4)
  np.testing.assert_array_equal(staging[:, :8192], payload[:, 0])
  np.testing.assert_array_equal(staging[:, scale_off:scale_off + 4].copy().view(np.float32)[:, 0],
                                scales[:, 0])


def test_c_relayout_matches_oracle():
  from oracle import cpu_ref
  rng = np.random.default_rng(5)
  n_st, n_seqs, T, H, HB = 3, 2, 256, 2, 16
  st = rng.permutation(n_seqs * T // 16).reshape(n_seqs, -1).astype(np.int32)
  dt = rng.permutation(n_seqs * T // 64).reshape(n_seqs, -1).astype(np.int32)
  src = [rng.integers(0, 256, (n_seqs * T // 16, 16 * H * HB), dtype=np.uint8) for _ in range(n_st)]
  got = [np.zeros((n_seqs * T // 64, 64 * H * HB), np.uint8) for _ in range(n_st)]
  cpu_ref.relayout(src, got, H, HB, 16, 64, st, dt, T, 2)
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  for s in range(n_st):
    want = np.zeros_like(got[s])
    ors.relayout(src[s], want, sg, dg, st, dt, T)
    np.testing.assert_array_equal(got[s], want)

"""Generates the golden reshard-plan fixtures by running the REFERENCE planner.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_golden.py

It imports tpu_sync.kv_cache.nd_slice_math and the planner functions of
tpu_sync.rpc.raiden_controller from the reference sources.  Their generated
protobuf modules (raiden_service_pb2, controller_service_pb2) are not part of
the checkout, so minimal stand-ins are put in sys.modules: the functions used
here only need NDSliceProto.dimensions.add(start=, end=).  The output
(reshard_plans.json) is committed; tests never read the reference.
"""

from __future__ import annotations

import json
import os
import sys
import types
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from oracle.build_ref import reference_root  # noqa: E402

REF = str(reference_root())
OUT = Path(__file__).resolve().parent / "reshard_plans.json"
sys.path.insert(0, str(Path(__file__).resolve().parents[2]))


class _Dim:
  def __init__(self, start=0, end=0):
    self.start, self.end = start, end


class _Dims(list):
  def add(self, start=0, end=0):
    d = _Dim(start, end)
    self.append(d)
    return d


class NDSliceProto:
  def __init__(self):
    self.dimensions = _Dims()


def _install_stubs():
  pkg = types.ModuleType("tpu_sync.rpc.raiden_service_pb2")
  pkg.NDSliceProto = NDSliceProto
  sys.modules["tpu_sync.rpc.raiden_service_pb2"] = pkg
  sys.modules["tpu_sync.rpc.controller_service_pb2"] = types.ModuleType(
      "tpu_sync.rpc.controller_service_pb2")


def main():
  _install_stubs()
  sys.path.insert(0, REF)
  from tpu_sync.kv_cache import nd_slice_math  # noqa: E402  (reference)
  from tpu_sync.rpc import raiden_controller as rc  # noqa: E402  (reference)
  from tpu_sync_b200 import workloads

  def bounds(protos):
    return [[(d.start, d.end) for d in p.dimensions] for p in protos]

  cases = []
  # nd_slice goldens (the reference's own test cases + the model layouts)
  slice_cases = [((5, 10), (2, 3)), ((16, 32, 64), (2, 1, 4)), ((8, 12), (2, 3)),
                 ((4096, 14336), (4, 1)), ((14336, 4096), (1, 4)), ((4097, 3), (4, 1))]
  slices = [{"global_shape": list(g), "mesh_shape": list(m),
             "slices": bounds(nd_slice_math.compute_nd_shard_slices(g, m))}
            for g, m in slice_cases]

  # chunk plans: every (src shard, dst shard) pair of each case
  def plan(shape, src_mesh, dst_mesh, itemsize):
    s_sl = bounds(nd_slice_math.compute_nd_shard_slices(shape, src_mesh))
    d_sl = bounds(nd_slice_math.compute_nd_shard_slices(shape, dst_mesh))
    pairs = []
    for i, s in enumerate(s_sl):
      for j, d in enumerate(d_sl):
        inter = rc.intersect_nd_slices(s, d)
        if inter is None:
          continue
        chunks = rc.generate_strided_copy_chunks(s, d, inter, itemsize)
        pairs.append({"src": i, "dst": j, "chunks": [list(c) for c in chunks]})
    return pairs

  shapes = {}
  for name, shape, split in workloads.llama3_8b_params():
    key = (shape, split)
    if key in shapes or name.startswith("layers.") and not name.startswith("layers.0."):
      continue
    shapes[key] = name
  for (shape, split), name in shapes.items():
    for n_src, n_dst in ((4, 4), (1, 1), (1, 2)):
      src_mesh = workloads.mesh_for(shape, "fsdp", n_src)
      dst_mesh = workloads.mesh_for(shape, split, n_dst)
      cases.append({"param": name, "shape": list(shape), "src_mesh": list(src_mesh),
                    "dst_mesh": list(dst_mesh), "itemsize": 1,
                    "pairs": plan(shape, src_mesh, dst_mesh, 1)})
  # odd shapes: remainders, 3-D / 4-D, column+row meshes
  extra = [((10, 7), (3, 1), (1, 2)), ((6, 5, 4), (2, 1, 1), (1, 1, 2)),
           ((4, 6, 8, 2), (2, 3, 1, 1), (1, 1, 2, 2)), ((9,), (2,), (3,)),
           ((12, 10), (2, 2), (3, 5))]
  for shape, sm, dm in extra:
    for itemsize in (1, 4):
      cases.append({"param": "extra", "shape": list(shape), "src_mesh": list(sm),
                    "dst_mesh": list(dm), "itemsize": itemsize,
                    "pairs": plan(shape, sm, dm, itemsize)})
  # unit -> slice index mapping (_get_global_indices), both branches:
  # named-axis sharding specs over a unit mesh, and the legacy host-axis rule
  import random
  rng = random.Random(44)
  index_cases = []
  unit_meshes = [([2, 2], ["fsdp", "tp"]), ([1, 4], ["fsdp", "tp"]), ([4, 1], ["fsdp", "tp"]),
                 ([2, 4], ["data", "model"]), ([8], ["x"]), ([2, 2, 2], ["a", "b", "c"])]
  for _ in range(300):
    umesh, axes = rng.choice(unit_meshes)
    n_units = rng.choice([1, 2, 4, 8])
    local = rng.choice([1, 1, 2])
    rank = rng.randint(1, 3)
    spec, vmesh = [], []
    for _d in range(rank):
      k = rng.random()
      if k < 0.3:
        spec.append("")
        vmesh.append(1)
      elif k < 0.8:
        i = rng.randrange(len(axes))
        spec.append(axes[i])
        vmesh.append(umesh[i])
      elif len(axes) > 1:
        i, j = sorted(rng.sample(range(len(axes)), 2))
        spec.append(f"{axes[i]},{axes[j]}")
        vmesh.append(umesh[i] * umesh[j])
      else:
        spec.append("missing_axis")
        vmesh.append(rng.choice([1, 2]))
    if rng.random() < 0.2:
      vmesh[rng.randrange(rank)] = n_units  # a dimension as large as the unit count
    layout = list(range(rank - 1, -1, -1))
    if rng.random() < 0.3:
      rng.shuffle(layout)
    with_spec = rng.random() < 0.85
    for replica in range(n_units):
      unit = rc.RaidenId("job", str(replica), "data")
      got = rc._get_global_indices(unit, ["s"] * local, list(vmesh), list(layout), n_units,
                                   sharding_spec=spec if with_spec else None,
                                   mesh_axes=axes if with_spec else None,
                                   physical_mesh_shape=umesh if with_spec else None)
      index_cases.append({"replica": replica, "local": local, "var_mesh": vmesh,
                          "layout": layout, "hosts": n_units,
                          "spec": spec if with_spec else None,
                          "axes": axes if with_spec else None,
                          "unit_mesh": umesh if with_spec else None,
                          "out": [list(x) for x in got]})
  OUT.write_text(json.dumps({"generator": "reference tpu_sync planner",
                             "slices": slices, "plans": cases,
                             "global_indices": index_cases}, indent=None))
  print(f"wrote {OUT} ({len(cases)} plans)")


if __name__ == "__main__":
  main()

"""Weight-sync reshard planner: trainer shards -> sampler shards.

Restates the reference controller's plan math (tpu_sync/rpc/raiden_controller.py):

* compute_nd_shard_slices  (tpu_sync/kv_cache/nd_slice_math.py:23-67): row-major
  device coordinates, tile = global // mesh per dim, remainder to the last shard;
* intersect_nd_slices      (raiden_controller.py:869-892);
* generate_strided_copy_chunks (raiden_controller.py:895-1013): the innermost
  dims that are full on both sides merge into one contiguous run; the dim
  above the split becomes the strided `count` dim; dims above that are
  enumerated as separate chunks.

Chunks are produced in ELEMENTS (itemsize 1): element offsets and strides
mean the same thing on both sides even when the destination dtype differs
(fp32 trainer master -> bf16 sampler), which the byte plans of the reference
cannot express.  `plan_bytes` gives the reference's byte form for a single
dtype.  The TPU (8, 128) tile-aware variant (raiden_controller.py:1016-1184)
is not needed: CUDA tensors are linear row-major.

Units and replicas: a plan is keyed by SLOTS, a slot being one shard of one
unit (a process or rank), flattened unit-major.  A slot holds one box of the
variable; by default slot i holds box i, and `shard_index_of_units` restates
the reference's mapping (_get_global_indices, raiden_controller.py:129-263)
for units on a named device mesh with a per-dimension sharding spec, where
several slots can hold the same box (replication).  Every destination slot
receives its box; when several source slots hold a box, destination slot d
takes it from holder d mod (number of holders), holders in slot order — the
reference's de-duplication and load balancing (raiden_controller.py:2283-2321,
:2460-2476).

Execution: chunks of one source rank, for every destination rank, become one
ts_reshard_copy launch (tpu_sync_b200.ops.ReshardProgram) that reads the
local shard and stores into the destination tensors, local or on a peer GPU.
"""

from __future__ import annotations

import itertools
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

Box = List[Tuple[int, int]]
Chunk = Tuple[int, int, int, int, int, int]  # src_off, dst_off, size, src_stride, dst_stride, count


def shard_boxes(global_shape: Sequence[int], mesh: Sequence[int]) -> List[Box]:
  """Per-device N-D bounding boxes in row-major device order."""
  if len(global_shape) != len(mesh):
    raise ValueError(
        f"Tensor rank ({len(global_shape)}) and sharding mesh rank ({len(mesh)}) "
        "must match exactly.")
  for d, m in enumerate(mesh):
    if m <= 0:
      raise ValueError(f"Mesh shape at dimension {d} must be positive.")
  per_dim = []
  for g, m in zip(global_shape, mesh):
    t = g // m
    per_dim.append([(c * t, g if c == m - 1 else (c + 1) * t) for c in range(m)])
  return [list(b) for b in itertools.product(*per_dim)]


def box_intersection(a: Box, b: Box) -> Optional[Box]:
  out = []
  for (s1, e1), (s2, e2) in zip(a, b):
    lo, hi = max(s1, s2), min(e1, e2)
    if lo >= hi:
      return None
    out.append((lo, hi))
  return out


def _row_major_strides(shape: Sequence[int]) -> List[int]:
  st = [1] * len(shape)
  for i in range(len(shape) - 2, -1, -1):
    st[i] = st[i + 1] * shape[i + 1]
  return st


def strided_chunks(src: Box, dst: Box, inter: Box, itemsize: int = 1) -> List[Chunk]:
  """Strided copy chunks of `inter` between the src and dst shard boxes."""
  rank = len(src)
  sshape = [e - s for s, e in src]
  dshape = [e - s for s, e in dst]
  ishape = [e - s for s, e in inter]
  # deepest dim that is not full on both sides
  split = next((d for d in range(rank - 1, -1, -1)
                if not (ishape[d] == sshape[d] == dshape[d])), -1)
  if split < 0:
    run, sdim = math.prod(ishape), -1
  else:
    run, sdim = math.prod(ishape[max(1, split):]), max(0, split - 1)
  sst, dst_ = _row_major_strides(sshape), _row_major_strides(dshape)
  s_lo = [i - s for (s, _), (i, _) in zip(src, inter)]
  d_lo = [i - s for (s, _), (i, _) in zip(dst, inter)]
  if sdim >= 0:
    count, s_stride, d_stride = ishape[sdim], sst[sdim] * itemsize, dst_[sdim] * itemsize
    outer = ishape[:sdim]
  else:
    count, s_stride, d_stride, outer = 1, 0, 0, []
  base_s = sum(s_lo[d] * sst[d] for d in range(len(outer), rank))
  base_d = sum(d_lo[d] * dst_[d] for d in range(len(outer), rank))
  chunks = []
  for idx in itertools.product(*[range(n) for n in outer]):
    so = base_s + sum((s_lo[d] + idx[d]) * sst[d] for d in range(len(outer)))
    do = base_d + sum((d_lo[d] + idx[d]) * dst_[d] for d in range(len(outer)))
    chunks.append((so * itemsize, do * itemsize, run * itemsize, s_stride, d_stride, count))
  return chunks


def normalize(chunks: Sequence[Chunk]) -> List[Chunk]:
  """Folds chunks whose rows are back to back on both sides into one run.

  Same bytes moved; matches the receiver-side expansion rule of the
  reference (count == 1 or both strides == size -> one contiguous copy,
  tpu_sync/weight_sync/weight_synchronizer_base.cc:634-645).
  """
  out = []
  for so, do, size, ss, ds, cnt in chunks:
    if cnt > 1 and ss == size and ds == size:
      out.append((so, do, size * cnt, 0, 0, 1))
    else:
      out.append((so, do, size, ss, ds, max(cnt, 1)))
  return out


def shard_index_of_units(replica_id: int, num_local_shards: int, var_mesh: Sequence[int],
                         layout: Sequence[int], num_physical_hosts: int,
                         sharding_spec: Optional[Sequence[str]] = None,
                         mesh_axes: Optional[Sequence[str]] = None,
                         physical_mesh: Optional[Sequence[int]] = None) -> List[Tuple[int, int]]:
  """(local shard, index of the variable's shard box it holds) for the
  `num_local_shards` shards of unit `replica_id`.

  Restates _get_global_indices (raiden_controller.py:129-263).  `layout` is
  the variable's minor-to-major dimension order.  With a sharding spec (one
  mesh-axis name per tensor dimension: "" = not split, "a,b" = split over the
  product of axes a and b), the unit mesh's axis names and shape, and no
  variable mesh dimension equal to the number of units, a shard's mesh
  coordinates come from its global device id (replica_id * local shards +
  local) in row-major order over the unit mesh; otherwise the legacy rule
  puts the unit on the variable mesh dimension whose size equals the number
  of units and its local shards, row-major, on the others.
  """
  n = int(num_local_shards)
  if n == 0:
    return []
  var_mesh = list(var_mesh)
  if not var_mesh:
    return [(j, j) for j in range(n)]
  if all(m == 1 for m in var_mesh):
    return [(j, 0) for j in range(n)]
  order = list(reversed(list(layout)))            # major to minor
  phys = [var_mesh[d] for d in order]
  host_dim = next((d for d, m in enumerate(var_mesh) if m == num_physical_hosts), None)

  def flat(coords, dims):
    idx, stride = 0, 1
    for c, m in zip(reversed(coords), reversed(dims)):
      idx += c * stride
      stride *= m
    return idx

  if host_dim is None and sharding_spec and mesh_axes and physical_mesh:
    axes, pmesh = list(mesh_axes), list(physical_mesh)
    out = []
    for j in range(n):
      dev = replica_id * n + j
      coords = [0] * len(pmesh)
      for a in range(len(pmesh) - 1, -1, -1):
        coords[a] = dev % pmesh[a]
        dev //= pmesh[a]
      tcoords = []
      for spec in sharding_spec:
        if not spec:
          tcoords.append(0)
        elif "," in spec:
          c = 0
          for sub in (x.strip() for x in spec.split(",")):
            if sub and sub in axes:
              k = axes.index(sub)
              c = c * pmesh[k] + coords[k]
          tcoords.append(c)
        else:
          tcoords.append(coords[axes.index(spec)] if spec in axes else 0)
      out.append((j, flat(tcoords, var_mesh)))
    return out
  others = [d for d in range(len(var_mesh)) if d != host_dim]
  out = []
  for j in range(n):
    full = [0] * len(var_mesh)
    rest = j
    for d in reversed(others):
      full[d] = rest % var_mesh[d]
      rest //= var_mesh[d]
    if host_dim is not None:
      full[host_dim] = replica_id
    out.append((j, flat([full[d] for d in order], phys)))
  return out


def slot_holders(n_units: int, var_mesh: Sequence[int], sharding_spec: Sequence[str],
                 mesh_axes: Sequence[str], unit_mesh: Sequence[int],
                 shards_per_unit: int = 1) -> List[int]:
  """Box index held by every slot (unit-major) of `n_units` units on a
  row-major variable layout."""
  layout = list(range(len(var_mesh) - 1, -1, -1))
  out = []
  for u in range(n_units):
    out += [g for _, g in shard_index_of_units(u, shards_per_unit, var_mesh, layout, n_units,
                                                sharding_spec, mesh_axes, unit_mesh)]
  return out


@dataclass
class VariableSpec:
  """One tensor to move: global shape, source mesh and destination mesh.

  src_holders / dst_holders: the box index each slot holds (None: slot i
  holds box i, one slot per box).
  """
  name: str
  shape: Tuple[int, ...]
  src_mesh: Tuple[int, ...]
  dst_mesh: Tuple[int, ...]
  layer_idx: int = 0
  src_holders: Optional[List[int]] = None
  dst_holders: Optional[List[int]] = None

  def src_box_of(self, slot: int) -> int:
    return slot if self.src_holders is None else self.src_holders[slot]

  def dst_box_of(self, slot: int) -> int:
    return slot if self.dst_holders is None else self.dst_holders[slot]


@dataclass
class ReshardPlan:
  """Element-unit chunks per (variable, src slot, dst slot)."""
  variables: List[VariableSpec]
  # (var index, src slot, dst slot) -> chunks
  chunks: Dict[Tuple[int, int, int], List[Chunk]] = field(default_factory=dict)

  def for_source(self, src_shard: int) -> Dict[Tuple[int, int], List[Chunk]]:
    """(var index, dst slot) -> chunks of one source slot."""
    return {(v, d): c for (v, s, d), c in self.chunks.items() if s == src_shard}

  def elements_to(self, dst_shard: int) -> int:
    """Elements every source together writes into one destination slot."""
    return sum(size * max(cnt, 1) for (v, s, d), cs in self.chunks.items() if d == dst_shard
               for (_, _, size, _, _, cnt) in cs)


def build_plan(variables: Sequence[VariableSpec], normalize_runs: bool = True) -> ReshardPlan:
  """Chunks for every (destination slot, intersecting source box), taken
  from one holder of that box (see the module docstring)."""
  plan = ReshardPlan(list(variables))
  for vi, v in enumerate(plan.variables):
    sboxes = shard_boxes(v.shape, v.src_mesh)
    dboxes = shard_boxes(v.shape, v.dst_mesh)
    src_holders = v.src_holders if v.src_holders is not None else list(range(len(sboxes)))
    dst_holders = v.dst_holders if v.dst_holders is not None else list(range(len(dboxes)))
    for name, hs, boxes in (("src", src_holders, sboxes), ("dst", dst_holders, dboxes)):
      bad = [b for b in hs if not 0 <= b < len(boxes)]
      if bad:
        raise ValueError(f"{v.name}: {name} slot holds box {bad[0]} of {len(boxes)}")
    holders: Dict[int, List[int]] = {}
    for slot, b in enumerate(src_holders):
      holders.setdefault(b, []).append(slot)
    for di, b_d in enumerate(dst_holders):
      db = dboxes[b_d]
      for b_s, sb in enumerate(sboxes):
        inter = box_intersection(sb, db)
        if inter is None:
          continue
        cands = holders.get(b_s)
        if not cands:
          raise ValueError(f"{v.name}: no source slot holds box {b_s}")
        si = cands[di % len(cands)]
        cs = strided_chunks(sb, db, inter, 1)
        plan.chunks[(vi, si, di)] = normalize(cs) if normalize_runs else cs
  return plan


def plan_bytes(src: Box, dst: Box, inter: Box, itemsize: int) -> List[Chunk]:
  """The reference's byte-unit chunks for one dtype."""
  return strided_chunks(src, dst, inter, itemsize)


def local_shape(box: Box) -> Tuple[int, ...]:
  return tuple(e - s for s, e in box)

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


@dataclass
class VariableSpec:
  """One tensor to move: global shape, source mesh and destination mesh."""
  name: str
  shape: Tuple[int, ...]
  src_mesh: Tuple[int, ...]
  dst_mesh: Tuple[int, ...]
  layer_idx: int = 0


@dataclass
class ReshardPlan:
  """Element-unit chunks per (variable, src shard, dst shard)."""
  variables: List[VariableSpec]
  # (var index, src shard, dst shard) -> chunks
  chunks: Dict[Tuple[int, int, int], List[Chunk]] = field(default_factory=dict)

  def for_source(self, src_shard: int) -> Dict[Tuple[int, int], List[Chunk]]:
    """(var index, dst shard) -> chunks of one source shard."""
    return {(v, d): c for (v, s, d), c in self.chunks.items() if s == src_shard}

  def elements_to(self, dst_shard: int) -> int:
    """Elements every source together writes into one destination shard."""
    return sum(size * max(cnt, 1) for (v, s, d), cs in self.chunks.items() if d == dst_shard
               for (_, _, size, _, _, cnt) in cs)


def build_plan(variables: Sequence[VariableSpec], normalize_runs: bool = True) -> ReshardPlan:
  plan = ReshardPlan(list(variables))
  for vi, v in enumerate(plan.variables):
    sboxes = shard_boxes(v.shape, v.src_mesh)
    dboxes = shard_boxes(v.shape, v.dst_mesh)
    for si, sb in enumerate(sboxes):
      for di, db in enumerate(dboxes):
        inter = box_intersection(sb, db)
        if inter is None:
          continue
        cs = strided_chunks(sb, db, inter, 1)
        plan.chunks[(vi, si, di)] = normalize(cs) if normalize_runs else cs
  return plan


def plan_bytes(src: Box, dst: Box, inter: Box, itemsize: int) -> List[Chunk]:
  """The reference's byte-unit chunks for one dtype."""
  return strided_chunks(src, dst, inter, itemsize)


def local_shape(box: Box) -> Tuple[int, ...]:
  return tuple(e - s for s, e in box)

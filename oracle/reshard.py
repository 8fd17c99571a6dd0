"""CPU oracle for the weight-sync reshard and the KV hand-off relayout --
TEST INFRASTRUCTURE ONLY (tests/, smoke(), bench.py's CPU arms).

Weight sync (reference path: planner tpu_sync/rpc/raiden_controller.py, executor
tpu_sync/weight_sync/weight_synchronizer_base.cc):

* compute_nd_shard_slices       tpu_sync/kv_cache/nd_slice_math.py:23-67
* intersect_nd_slices           tpu_sync/rpc/raiden_controller.py:869-892
* generate_strided_copy_chunks  tpu_sync/rpc/raiden_controller.py:895-1013
* entry expansion: count == 1 or both strides == size -> one contiguous copy
  of count*size bytes, else one copy per repeat
                                tpu_sync/weight_sync/weight_synchronizer_base.cc:606-667
* receiver writes each copy at dst_offset of its host buffer, then H2D
                                tpu_sync/weight_sync/weight_synchronizer_base.cc:824-845

The planner functions here are a second, independent restatement used only
to check the product planner (tpu_sync_b200/reshard_plan.py); both are pinned
against golden plans produced by running the reference planner itself
(tests/golden/make_golden.py -> tests/golden/reshard_plans.json).

The fp32 -> bf16 cast of the B200 path has no reference counterpart (the
reference moves bytes unchanged); it is round-to-nearest-even, restated in
oracle/fp8.py:f32_to_bf16_bits_rne.

KV hand-off relayout: the reference moves pages with a D2H into a host slot,
a TCP push and an H2D at the consumer, relaying out between page sizes with
byte spans planned by BuildPoolReshardPlan
(tpu_sync/kv_cache/reshard/pool_reshard_planner.cc:547-781).  relayout()
below states the resulting byte mapping directly: every (token, head) vector
moves from its source page position to its destination page position.
"""

from __future__ import annotations

import itertools
import math
from typing import List, Sequence, Tuple

import numpy as np

from oracle.fp8 import f32_to_bf16_bits_rne

NDSlice = List[Tuple[int, int]]


def compute_nd_shard_slices(global_shape, mesh_shape) -> List[NDSlice]:
  if len(global_shape) != len(mesh_shape):
    raise ValueError("rank mismatch")
  tiles = [g // m for g, m in zip(global_shape, mesh_shape)]
  out = []
  for coord in itertools.product(*[range(m) for m in mesh_shape]):
    out.append([(c * t, (c + 1) * t if c < m - 1 else g)
                for c, t, m, g in zip(coord, tiles, mesh_shape, global_shape)])
  return out


def intersect_nd_slices(a: NDSlice, b: NDSlice):
  res = []
  for (s1, e1), (s2, e2) in zip(a, b):
    s, e = max(s1, s2), min(e1, e2)
    if s >= e:
      return None
    res.append((s, e))
  return res


def generate_strided_copy_chunks(src: NDSlice, dst: NDSlice, inter: NDSlice,
                                 itemsize: int):
  """(src_off, dst_off, size, src_stride, dst_stride, count), bytes."""
  rank = len(src)
  src_shape = [e - s for s, e in src]
  dst_shape = [e - s for s, e in dst]
  int_shape = [e - s for s, e in inter]
  split = -1
  for d in range(rank - 1, -1, -1):
    if not (int_shape[d] == src_shape[d] and int_shape[d] == dst_shape[d]):
      split = d
      break
  if split != -1:
    contiguous = math.prod(int_shape[max(1, split):])
    stride_dim = max(0, split - 1)
  else:
    contiguous = math.prod(int_shape)
    stride_dim = -1
  sst = [1] * rank
  dstt = [1] * rank
  for i in range(rank - 2, -1, -1):
    sst[i] = sst[i + 1] * src_shape[i + 1]
    dstt[i] = dstt[i + 1] * dst_shape[i + 1]
  if stride_dim >= 0:
    count = int_shape[stride_dim]
    s_stride, d_stride = sst[stride_dim] * itemsize, dstt[stride_dim] * itemsize
    outer = int_shape[:stride_dim]
  else:
    count, s_stride, d_stride, outer = 1, 0, 0, []
  n_outer = math.prod(outer) if outer else 1
  s_loc = [i0 - s0 for (s0, _), (i0, _) in zip(src, inter)]
  d_loc = [i0 - d0 for (d0, _), (i0, _) in zip(dst, inter)]
  chunks = []
  for i in range(n_outer):
    idx, t = [], i
    for sz in reversed(outer):
      idx.append(t % sz)
      t //= sz
    idx.reverse()
    so = sum((s_loc[d] + idx[d]) * sst[d] for d in range(len(outer)))
    do = sum((d_loc[d] + idx[d]) * dstt[d] for d in range(len(outer)))
    so += sum(s_loc[d] * sst[d] for d in range(len(outer), rank))
    do += sum(d_loc[d] * dstt[d] for d in range(len(outer), rank))
    chunks.append((so * itemsize, do * itemsize, contiguous * itemsize, s_stride,
                   d_stride, count))
  return chunks


def expand_entry(src_off, dst_off, size, src_stride, dst_stride, count):
  """weight_synchronizer_base.cc:634-666: list of (src_off, dst_off, nbytes)."""
  count = count if count > 0 else 1
  if count == 1 or (src_stride == size and dst_stride == size):
    return [(src_off, dst_off, count * size)]
  return [(src_off + c * src_stride, dst_off + c * dst_stride, size)
          for c in range(count)]


def apply_byte_entries(src: np.ndarray, dst: np.ndarray, entries) -> None:
  """Executes byte-unit entries on uint8 buffers (the reference's memcpys)."""
  for e in entries:
    for so, do, n in expand_entry(*e):
      if so + n > src.size:
        raise ValueError("Push range out of bounds")
      dst[do:do + n] = src[so:so + n]


def apply_element_chunks(src: np.ndarray, dst: np.ndarray, chunks, cast_bf16: bool):
  """Element-unit chunks; with cast_bf16, src is fp32 and dst holds bf16 bits."""
  for so, do, size, ss, ds, count in chunks:
    for c in range(max(count, 1)):
      seg = src[so + c * ss: so + c * ss + size]
      if cast_bf16:
        dst[do + c * ds: do + c * ds + size] = f32_to_bf16_bits_rne(seg)
      else:
        dst[do + c * ds: do + c * ds + size] = seg


def relayout(src_pages: np.ndarray, dst_pages: np.ndarray, src_geom: dict,
             dst_geom: dict, src_table: np.ndarray, dst_table: np.ndarray,
             seq_tokens: int) -> None:
  """Token/head vector permutation between two paged layouts (in place).

  src_pages: uint8 [num_src_blocks, src_block_bytes] of ONE storage; same for
  dst.  Geometry dicts: block_tokens, heads, head_bytes, head_major.
  """
  H, hb = src_geom["heads"], src_geom["head_bytes"]
  st_, dt_ = src_geom["block_tokens"], dst_geom["block_tokens"]
  sv = src_pages.reshape(src_pages.shape[0], -1)
  dv = dst_pages.reshape(dst_pages.shape[0], -1)
  for q in range(src_table.shape[0]):
    t = np.arange(seq_tokens)
    sb = src_table[q, t // st_].astype(np.int64)
    dbk = dst_table[q, t // dt_].astype(np.int64)
    for h in range(H):
      so = (h * st_ + t % st_) if src_geom["head_major"] else ((t % st_) * H + h)
      do = (h * dt_ + t % dt_) if dst_geom["head_major"] else ((t % dt_) * H + h)
      cols = np.arange(hb)
      dv[dbk[:, None], do[:, None] * hb + cols] = sv[sb[:, None], so[:, None] * hb + cols]


# ---------------------------------------------------------------------------
# Units, replicas and de-duplication (weight sync)
# ---------------------------------------------------------------------------

def global_indices(replica_id, num_shards, logical_mesh, layout, num_hosts,
                   sharding_spec=None, mesh_axes=None, physical_mesh=None):
  """_get_global_indices (tpu_sync/rpc/raiden_controller.py:129-263):
  [(local shard, global slice index)] of one unit."""
  if num_shards == 0:
    return []
  if not logical_mesh:
    return [(i, i) for i in range(num_shards)]
  if all(d == 1 for d in logical_mesh):
    return [(i, 0) for i in range(num_shards)]
  m2m = list(layout)[::-1]
  phys = [logical_mesh[d] for d in m2m]
  host = None
  for d, size in enumerate(logical_mesh):
    if size == num_hosts:
      host = d
      break

  def ravel(coords, shape):
    g, stride = 0, 1
    for c, s in list(zip(coords[::-1], shape[::-1])):
      g += c * stride
      stride *= s
    return g

  res = []
  if host is None and sharding_spec and mesh_axes and physical_mesh:
    for j in range(num_shards):
      rem = replica_id * num_shards + j
      pc = []
      for size in physical_mesh[::-1]:
        pc.append(rem % size)
        rem //= size
      pc = pc[::-1]
      tc = []
      for name in sharding_spec:
        if not name:
          tc.append(0)
          continue
        if "," in name:
          v = 0
          for sub in [x.strip() for x in name.split(",") if x.strip()]:
            if sub in mesh_axes:
              i = list(mesh_axes).index(sub)
              v = v * physical_mesh[i] + pc[i]
          tc.append(v)
          continue
        tc.append(pc[list(mesh_axes).index(name)] if name in mesh_axes else 0)
      res.append((j, ravel(tc, list(logical_mesh))))
    return res
  non_host = [d for d in range(len(logical_mesh)) if d != host]
  for j in range(num_shards):
    loc, t = {}, j
    for d in non_host[::-1]:
      loc[d] = t % logical_mesh[d]
      t //= logical_mesh[d]
    full = [replica_id if d == host else loc[d] for d in range(len(logical_mesh))]
    res.append((j, ravel([full[m] for m in m2m], phys)))
  return res


def plan_with_replicas(shape, src_mesh, dst_mesh, src_holders, dst_holders, itemsize=1):
  """Schedule emission with replicated holders (raiden_controller.py:2283-2321,
  :2392-2476): for each destination slot and each source box intersecting
  its box, the chunks come from holder (slot index mod holders) of that
  source box, holders in slot order.  Returns {(src slot, dst slot): chunks}."""
  s_sl = compute_nd_shard_slices(shape, src_mesh)
  d_sl = compute_nd_shard_slices(shape, dst_mesh)
  by_box = {}
  for slot, b in enumerate(src_holders):
    by_box.setdefault(b, []).append(slot)
  out = {}
  for src_slot, b_s in enumerate(src_holders):
    for dst_slot, b_d in enumerate(dst_holders):
      inter = intersect_nd_slices(s_sl[b_s], d_sl[b_d])
      if inter is None:
        continue
      cands = by_box[b_s]
      if len(cands) > 1 and cands[dst_slot % len(cands)] != src_slot:
        continue
      out[(src_slot, dst_slot)] = generate_strided_copy_chunks(s_sl[b_s], d_sl[b_d], inter,
                                                               itemsize)
  return out

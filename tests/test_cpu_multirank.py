"""Multi-rank host logic of the weight-sync leg on CPU (gloo, world sizes 2,
4 and 8), the path `bench.py --gpus N` runs over NCCL and NVLink.

Ranks [0, N/2) are FSDP trainers (fp32), ranks [N/2, N) TP samplers (bf16).
Every rank builds the same plan and flat-buffer layout
(workloads.weight_sync_specs / weight_sync_layout); samplers publish their
buffer sizes with all_gather_object (the bench publishes IPC descriptors the
same way); each trainer takes its own chunks (workloads.weight_sync_chunks,
the list the bench hands to ops.ReshardProgram), applies them with the
oracle's chunk executor (fp32 -> bf16 RNE) and sends each sampler the bytes
and the mask of elements it wrote.  Each sampler checks that every element
of its buffer was written exactly once and equals its TP shards of the
global tensors.  The timing reduction the bench uses (max over ranks) is
checked on the same group.
"""

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from oracle import reshard as ors
from tpu_sync_b200 import reshard_plan as rp
from tpu_sync_b200 import workloads

PARAMS = [("embed", (320, 64), "vocab"), ("q", (64, 64), "col"), ("o", (64, 64), "row"),
          ("down", (64, 160), "row"), ("norm", (64,), "rep"), ("up", (160, 64), "col")]
DST_BASE = 1 << 40  # dst_bases[d] = d * DST_BASE tells the chunks' sampler apart


def _global_tensors():
  g = torch.Generator().manual_seed(7)
  return [torch.randn(shape, generator=g) * 0.02 for _, shape, _ in PARAMS]


def _box(t, box):
  return t[tuple(slice(a, b) for a, b in box)]


def _rank_main(rank, world, port, errors):
  os.environ["MASTER_ADDR"] = "127.0.0.1"
  os.environ["MASTER_PORT"] = str(port)
  import torch.distributed as dist
  dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
  try:
    half = world // 2
    specs = workloads.weight_sync_specs(half, half, PARAMS)
    plan = rp.build_plan(specs)
    layout = workloads.weight_sync_layout(specs, half, half)
    full = _global_tensors()
    is_src = rank < half
    idx = rank if is_src else rank - half
    descs = [None] * world
    dist.all_gather_object(descs, None if is_src else layout[1][idx][1])
    if is_src:
      flat = torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.src_mesh)[v.src_box_of(idx)])
                        .reshape(-1) for vi, v in enumerate(specs)]).numpy()
      assert flat.size == layout[0][idx][1]
      chunks = workloads.weight_sync_chunks(plan, layout, idx, 0,
                                            {d: d * DST_BASE for d in range(half)})
      for d in range(half):
        n = descs[half + d]
        out = np.zeros(n, np.uint16)
        mask = np.zeros(n, np.uint8)
        mine = [(sp // 4 + so, (dp - d * DST_BASE) // 2 + do, size, ss, ds, cnt)
                for (sp, dp, so, do, size, ss, ds, cnt) in chunks if dp // DST_BASE == d]
        ors.apply_element_chunks(flat, out, mine, cast_bf16=True)
        for (_, do, size, _, ds, cnt) in mine:
          for c in range(max(cnt, 1)):
            mask[do + c * ds: do + c * ds + size] += 1
        dist.send(torch.from_numpy(out.view(np.int16)), dst=half + d)
        dist.send(torch.from_numpy(mask), dst=half + d)
    else:
      n = descs[rank]
      buf = np.zeros(n, np.uint16)
      cover = np.zeros(n, np.int64)
      for s in range(half):
        vals = torch.empty(n, dtype=torch.int16)
        mask = torch.empty(n, dtype=torch.uint8)
        dist.recv(vals, src=s)
        dist.recv(mask, src=s)
        m = mask.numpy().astype(bool)
        buf[m] = vals.numpy().view(np.uint16)[m]
        cover += mask.numpy()
      assert (cover == 1).all(), f"rank {rank}: coverage {np.bincount(cover)}"
      want = torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.dst_mesh)[v.dst_box_of(idx)])
                        .reshape(-1) for vi, v in enumerate(specs)])
      want = want.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
      np.testing.assert_array_equal(buf, want)
    # the bench's timing reduction: the max over ranks
    t = torch.tensor([float(rank + 1)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    assert t.item() == float(world)
  except BaseException as e:  # reported to the parent, which fails the test
    errors.put(f"rank {rank}: {type(e).__name__}: {e}")
    raise
  finally:
    dist.destroy_process_group()


def _free_port():
  with socket.socket() as s:
    s.bind(("127.0.0.1", 0))
    return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_weight_sync_across_ranks(world):
  import torch.multiprocessing as tmp
  ctx = tmp.get_context("spawn")
  errors = ctx.Queue()
  port = _free_port()
  procs = [ctx.Process(target=_rank_main, args=(r, world, port, errors)) for r in range(world)]
  for p in procs:
    p.start()
  for p in procs:
    p.join(timeout=180)
  alive = [p for p in procs if p.is_alive()]
  for p in alive:
    p.kill()
    p.join()
  msgs = []
  while not errors.empty():
    msgs.append(errors.get())
  assert not alive, "ranks did not finish"
  assert not msgs, msgs
  assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


@pytest.mark.parametrize("n_src,n_dst", [(1, 1), (1, 2), (2, 1), (2, 2), (4, 4), (2, 4)])
def test_staged_pull_chunks_cover_each_sampler_exactly_once(n_src, n_dst):
  """The staged pull's receiver chunk lists (workloads.weight_sync_pull_chunks,
  what bench.py hands to ops.PullReceiver): applied by the oracle from the
  trainers' flat fp32 buffers (the staging holds their bf16 casts in the same
  element layout), every element of a sampler's buffer is written exactly
  once and equals its TP shards of the global tensors."""
  specs = workloads.weight_sync_specs(n_src, n_dst, PARAMS)
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, n_src, n_dst)
  full = _global_tensors()
  flats = [torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.src_mesh)[v.src_box_of(s)])
                      .reshape(-1) for vi, v in enumerate(specs)]).numpy()
           for s in range(n_src)]
  for d in range(n_dst):
    chunks = workloads.weight_sync_pull_chunks(plan, layout, d, 0, n_src)
    n = layout[1][d][1]
    out = np.zeros(n, np.uint16)
    cover = np.zeros(n, np.int64)
    for s in range(n_src):
      mine = [(so, dp // 2 + do, size, ss, ds, cnt)
              for (t, dp, so, do, size, ss, ds, cnt) in chunks if t == s]
      for (so, _, size, ss, _, cnt) in mine:  # inside the sender's staging
        assert so + (cnt - 1) * ss + size <= layout[0][s][1]
      ors.apply_element_chunks(flats[s], out, mine, cast_bf16=True)
      for (_, do, size, _, ds, cnt) in mine:
        for c in range(max(cnt, 1)):
          cover[do + c * ds: do + c * ds + size] += 1
    assert (cover == 1).all(), (d, np.unique(cover))
    want = torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.dst_mesh)[v.dst_box_of(d)])
                      .reshape(-1) for vi, v in enumerate(specs)]).to(torch.bfloat16)
    np.testing.assert_array_equal(out, want.view(torch.int16).numpy().view(np.uint16))


@pytest.mark.parametrize("n", [2, 4])
def test_hybrid_split_covers_each_sampler_exactly_once(n):
  """The hybrid weight sync of bench.py (n -> n): sampler d pulls only what
  trainer d holds for it (weight_sync_pull_chunks with src_slots={d}), and
  every other trainer pushes its slices for d (weight_sync_chunks with
  dst_slots={d}).  Together they write every element of d's buffer exactly
  once, equal to its TP shards."""
  specs = workloads.weight_sync_specs(n, n, PARAMS)
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, n, n)
  full = _global_tensors()
  flats = [torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.src_mesh)[v.src_box_of(s)])
                      .reshape(-1) for vi, v in enumerate(specs)]).numpy() for s in range(n)]
  for d in range(n):
    size = layout[1][d][1]
    out = np.zeros(size, np.uint16)
    cover = np.zeros(size, np.int64)
    parts = []
    for (t, dp, so, do, sz, ss, ds, cnt) in workloads.weight_sync_pull_chunks(
        plan, layout, d, 0, n, src_slots={d}):
      assert t == d
      parts.append((t, (so, dp // 2 + do, sz, ss, ds, cnt)))
    for t in range(n):
      if t == d:
        continue
      for (sp, dp, so, do, sz, ss, ds, cnt) in workloads.weight_sync_chunks(
          plan, layout, t, 0, {e: e * DST_BASE for e in range(n)}, dst_slots={d}):
        assert dp // DST_BASE == d
        parts.append((t, (sp // 4 + so, (dp - d * DST_BASE) // 2 + do, sz, ss, ds, cnt)))
    for t, c in parts:
      ors.apply_element_chunks(flats[t], out, [c], cast_bf16=True)
      so, do, sz, ss, ds, cnt = c
      for r in range(max(cnt, 1)):
        cover[do + r * ds: do + r * ds + sz] += 1
    assert (cover == 1).all(), (d, np.unique(cover))
    want = torch.cat([_box(full[vi], rp.shard_boxes(v.shape, v.dst_mesh)[v.dst_box_of(d)])
                      .reshape(-1) for vi, v in enumerate(specs)]).to(torch.bfloat16)
    np.testing.assert_array_equal(out, want.view(torch.int16).numpy().view(np.uint16))

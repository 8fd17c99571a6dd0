"""GPU parity of the pool reshard executor (one kernel per source unit).

Plans come from the product planner; every source unit's program runs on
cuda:0 and stores into destination storages (here on the same GPU; the
NVLink peer case is in test_gpu_multi.py).  The destination bytes are
compared with the oracle's application of the same plan
(oracle/pool_reshard.apply_plan) -- bit-exact, untouched bytes included.
"""

import random

import numpy as np
import pytest
import torch

from oracle import pool_reshard as opr
from oracle import reshard as ors
from tpu_sync_b200 import ops, workloads
from tpu_sync_b200.pool_reshard import PoolReshardProgram, build_pool_reshard_plan

from test_cpu_pool_reshard import _random_request

pytestmark = pytest.mark.gpu


def gpu():
  if not torch.cuda.is_available():
    pytest.skip("needs a GPU")
  return torch.device("cuda", 0)


def oracle_plan(plan):
  return {"schedules": {u: [(e.src_block_id, e.dst_block_id, e.src_offset_bytes,
                             e.dst_offset_bytes, e.size_bytes, e.pool_group) for e in es]
                        for u, es in plan.schedules.items()},
          "groups": [{"pool_indices": g.pool_indices} for g in plan.pool_groups]}


def storage_bytes(pools):
  return max(p.base_offset_bytes + p.num_blocks * p.block_stride_bytes for p in pools)


def test_random_plans_match_oracle():
  dev = gpu()
  rng = random.Random(5)
  g = torch.Generator().manual_seed(5)
  done = 0
  while done < 25:
    src_pools, dst_pools, tags, ids, decls, kw = _random_request(rng)
    try:
      plan = build_pool_reshard_plan(src_pools, dst_pools, tags, ids, decls, **kw)
    except ValueError:
      continue
    nu = len(src_pools)
    sb, db = storage_bytes(src_pools[0]), storage_bytes(dst_pools)
    srcs = [torch.randint(0, 256, (sb,), generator=g, dtype=torch.uint8) for _ in range(nu)]
    dst = torch.randint(0, 256, (db,), generator=g, dtype=torch.uint8)
    want = dst.numpy().copy()
    d_dev = dst.to(dev)
    spare = torch.zeros(16, dtype=torch.uint8, device=dev)  # storage index not used by a side
    progs = []
    for u in range(nu):
      s_dev = srcs[u].to(dev)
      # source pools live in storage 0, destination pools in storage 1
      prog = PoolReshardProgram(plan, u, [s_dev, spare], [spare, d_dev])
      prog.launch()
      progs.append((prog, s_dev))
      opr.apply_plan(oracle_plan(plan), u, [p.to_dict() for p in src_pools[u]],
                     [p.to_dict() for p in dst_pools], [srcs[u].numpy(), None], [None, want])
    torch.cuda.synchronize()
    np.testing.assert_array_equal(d_dev.cpu().numpy(), want)
    done += 1


def test_c3_handoff_plan_matches_relayout_kernel():
  dev = gpu()
  rng = np.random.default_rng(9)
  n_st, n_seqs, T, H, HB = 4, 3, 512, 2, 256
  sbps, dbps = T // 16, T // 64
  st = rng.permutation(n_seqs * sbps + 5)[:n_seqs * sbps].reshape(n_seqs, sbps).astype(np.int32)
  dt = rng.permutation(n_seqs * dbps + 3)[:n_seqs * dbps].reshape(n_seqs, dbps).astype(np.int32)
  src_pools, dst_pools, dst_ids, r = workloads.handoff_pool_plan_inputs(n_st, st, dt, H, HB)
  plan = build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids, [(0, r)])
  sbb, dbb = 16 * H * HB, 64 * H * HB
  n_sb, n_db = int(st.max()) + 1, int(dt.max()) + 1
  g = torch.Generator().manual_seed(1)
  src = [torch.randint(0, 256, (n_sb, sbb), generator=g, dtype=torch.uint8).to(dev)
         for _ in range(n_st)]
  via_plan = [torch.zeros((n_db, dbb), dtype=torch.uint8, device=dev) for _ in range(n_st)]
  via_relayout = [torch.zeros((n_db, dbb), dtype=torch.uint8, device=dev) for _ in range(n_st)]
  prog = PoolReshardProgram(plan, 0, src, via_plan)
  # merged rows: one task per (source page, head), 16 head vectors each
  assert prog.n_tasks == n_st * n_seqs * sbps * H and prog.bytes == n_st * n_seqs * T * H * HB
  prog.launch()
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  ops.kv_relayout(src, via_relayout, sg, dg, torch.from_numpy(st), torch.from_numpy(dt), T,
                  device=dev)
  torch.cuda.synchronize()
  for s in range(n_st):
    want = np.zeros((n_db, dbb), np.uint8)
    ors.relayout(src[s].cpu().numpy(), want, sg, dg, st, dt, T)
    np.testing.assert_array_equal(via_plan[s].cpu().numpy(), want)
    assert torch.equal(via_plan[s], via_relayout[s])


def test_program_rejects_storages_smaller_than_pools():
  dev = gpu()
  src_pools, dst_pools, dst_ids, r = workloads.handoff_pool_plan_inputs(
      1, np.arange(4, dtype=np.int32).reshape(1, 4), np.arange(1, dtype=np.int32).reshape(1, 1),
      2, 64)
  plan = build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids, [(0, r)])
  src = torch.zeros((4, 16 * 2 * 64), dtype=torch.uint8, device=dev)
  small = torch.zeros((64 * 2 * 64) - 1, dtype=torch.uint8, device=dev)
  with pytest.raises(RuntimeError, match="destination pool kv exceeds storage bytes"):
    PoolReshardProgram(plan, 0, [src], [small])


def test_received_plan_with_repeating_entries_matches_relayout():
  """A controller-style plan (entries with count / strides, as
  ShardPushEntryProto carries them) validated on both ends and executed."""
  from tpu_sync_b200.pool_reshard import plan_from_received
  dev = gpu()
  rng = np.random.default_rng(12)
  n_st, n_seqs, T, H, HB = 2, 2, 256, 2, 128
  sbps, dbps = T // 16, T // 64
  st = rng.permutation(n_seqs * sbps).reshape(n_seqs, sbps).astype(np.int32)
  dt = rng.permutation(n_seqs * dbps).reshape(n_seqs, dbps).astype(np.int32)
  src_pools, dst_pools, _, _ = workloads.handoff_pool_plan_inputs(n_st, st, dt, H, HB)
  entries = []
  for q in range(n_seqs):
    for p in range(sbps):
      for h in range(H):
        entries.append(dict(dst_peer="decode:0", dst_shard_idx=0, src_block_id=int(st[q, p]),
                            dst_block_id=int(dt[q, p // 4]), src_offset_bytes=h * 16 * HB,
                            dst_offset_bytes=(p % 4) * 16 * H * HB + h * HB, size_bytes=HB,
                            src_stride_bytes=HB, dst_stride_bytes=H * HB, count=16,
                            pool_group=0))
  recv = {"transfer_pool_indices": list(range(n_st)), "pool_dtype_tags": [""] * n_st,
          "parallelism": 1,
          "pool_groups": [{"pool_indices": list(range(n_st)),
                           "dst_device_block_ids": [int(x) for x in dt.reshape(-1)],
                           "dst_expected_extent_bytes": [64 * H * HB] * (n_seqs * dbps),
                           "expected_pushes": 1, "order_rank": 0}],
          "shard_push_schedules": {0: entries}}
  plan = plan_from_received(recv, src_pools, dst_pools, [int(x) for x in st.reshape(-1)],
                            [int(x) for x in dt.reshape(-1)])
  g = torch.Generator().manual_seed(3)
  src = [torch.randint(0, 256, (n_seqs * sbps, 16 * H * HB), generator=g,
                       dtype=torch.uint8).to(dev) for _ in range(n_st)]
  dst = [torch.zeros((n_seqs * dbps, 64 * H * HB), dtype=torch.uint8, device=dev)
         for _ in range(n_st)]
  PoolReshardProgram(plan, 0, src, dst).launch()
  torch.cuda.synchronize()
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  for s in range(n_st):
    want = np.zeros((n_seqs * dbps, 64 * H * HB), np.uint8)
    ors.relayout(src[s].cpu().numpy(), want, sg, dg, st, dt, T)
    np.testing.assert_array_equal(dst[s].cpu().numpy(), want)

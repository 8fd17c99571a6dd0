"""Two-GPU parity of the NVLink paths (skipped with fewer than two GPUs).

* in one process: reshard and relayout kernels on cuda:0 store into
  tensors on cuda:1 through peer pointers;
* across two processes: the sampler process exports its destination
  tensors (CUDA IPC), the trainer process maps them and pushes its fp32
  shards as bf16; the sampler checks every element bit-exact.
"""

import multiprocessing as mp

import numpy as np
import pytest
import torch

from oracle import reshard as ors
from tpu_sync_b200 import ops, workloads
from tpu_sync_b200 import reshard_plan as rp

pytestmark = pytest.mark.gpu


def two_gpus():
  if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two GPUs")


def small_params():
  return [("embed", (320, 64), "vocab"), ("q", (64, 64), "col"), ("o", (64, 64), "row"),
          ("down", (64, 160), "row"), ("norm", (64,), "rep")]


def globals_for(params):
  g = torch.Generator().manual_seed(3)
  return [(torch.randn(shape, generator=g) * 0.02) for _, shape, _ in params]


def test_peer_reshard_and_relayout_in_process():
  two_gpus()
  from tpu_sync_b200.weight_synchronizer import WeightSynchronizer
  params = small_params()
  specs = [rp.VariableSpec(n, s, workloads.mesh_for(s, "fsdp", 2), workloads.mesh_for(s, sp, 2),
                           layer_idx=i) for i, (n, s, sp) in enumerate(params)]
  plan = rp.build_plan(specs)
  full = globals_for(params)
  grid = [[full[i][tuple(slice(a, b) for a, b in box)].contiguous().cuda(0)
           for box in rp.shard_boxes(v.shape, v.src_mesh)] for i, v in enumerate(specs)]
  dest = {(vi, d): torch.zeros(rp.local_shape(box), dtype=torch.bfloat16, device="cuda:1")
          for vi, v in enumerate(specs) for d, box in enumerate(rp.shard_boxes(v.shape, v.dst_mesh))}
  WeightSynchronizer(grid).push_weights_resharded(plan, {0: 0, 1: 1}, dest).Await()
  torch.cuda.synchronize(1)
  for (vi, d), t in dest.items():
    box = rp.shard_boxes(specs[vi].shape, specs[vi].dst_mesh)[d]
    want = full[vi].to(torch.bfloat16)[tuple(slice(a, b) for a, b in box)]
    assert torch.equal(t.cpu().view(torch.int16), want.view(torch.int16))
  # relayout into the peer
  sg = dict(block_tokens=16, heads=2, head_bytes=256, head_major=1)
  dg = dict(block_tokens=64, heads=2, head_bytes=256, head_major=0)
  rng = np.random.default_rng(1)
  st = rng.permutation(16).reshape(2, 8).astype(np.int32)
  dt = rng.permutation(4).reshape(2, 2).astype(np.int32)
  src = torch.from_numpy(rng.integers(0, 256, (16, 8192), dtype=np.uint8)).cuda(0)
  dst = torch.zeros((4, 32768), dtype=torch.uint8, device="cuda:1")
  from tpu_sync_b200.weight_synchronizer import enable_peer_access
  enable_peer_access(0, 1)
  ops.kv_relayout([src], [dst], sg, dg, torch.from_numpy(st), torch.from_numpy(dt), 128,
                  device="cuda:0")
  torch.cuda.synchronize(0)
  want = np.zeros((4, 32768), np.uint8)
  ors.relayout(src.cpu().numpy(), want, sg, dg, st, dt, 128)
  np.testing.assert_array_equal(dst.cpu().numpy(), want)


@pytest.mark.parametrize("engine", ["sm", "copy"])
def test_peer_reshard_both_directions(engine):
  """Source shard i on GPU i, destination shard d on GPU 1 - d: every chunk
  crosses NVLink, the column-split variables as strided rows (the 2 -> 2
  weight sync's pattern), pushed by the SM kernel or the copy engines."""
  two_gpus()
  from tpu_sync_b200.weight_synchronizer import WeightSynchronizer
  params = small_params()
  specs = [rp.VariableSpec(n, s, workloads.mesh_for(s, "fsdp", 2), workloads.mesh_for(s, sp, 2),
                           layer_idx=i) for i, (n, s, sp) in enumerate(params)]
  plan = rp.build_plan(specs)
  assert any(cnt > 1 and (ss != size or ds != size)
             for cs in plan.for_source(0).values() for (_, _, size, ss, ds, cnt) in cs)
  full = globals_for(params)
  grid = [[full[i][tuple(slice(a, b) for a, b in box)].contiguous().cuda(s)
           for s, box in enumerate(rp.shard_boxes(v.shape, v.src_mesh))]
          for i, v in enumerate(specs)]
  dest = {(vi, d): torch.zeros(rp.local_shape(box), dtype=torch.bfloat16, device=f"cuda:{1 - d}")
          for vi, v in enumerate(specs) for d, box in enumerate(rp.shard_boxes(v.shape, v.dst_mesh))}
  fut = WeightSynchronizer(grid).push_weights_resharded(plan, {0: 0, 1: 1}, dest, engine=engine)
  fut.Await()
  torch.cuda.synchronize(0)
  torch.cuda.synchronize(1)
  for (vi, d), t in dest.items():
    box = rp.shard_boxes(specs[vi].shape, specs[vi].dst_mesh)[d]
    want = full[vi].to(torch.bfloat16)[tuple(slice(a, b) for a, b in box)]
    assert torch.equal(t.cpu().view(torch.int16), want.view(torch.int16)), (vi, d)


def _sampler(q_out, q_in, result):
  import torch
  from tpu_sync_b200 import reshard_plan as rp, workloads
  from tpu_sync_b200.weight_synchronizer import export_destinations
  torch.cuda.set_device(1)
  params = small_params()
  specs = [rp.VariableSpec(n, s, workloads.mesh_for(s, "fsdp", 1), workloads.mesh_for(s, sp, 1),
                           layer_idx=i) for i, (n, s, sp) in enumerate(params)]
  dest = {(vi, 0): torch.zeros(v.shape, dtype=torch.bfloat16, device="cuda:1")
          for vi, v in enumerate(specs)}
  q_out.put(export_destinations(dest))
  q_in.get(timeout=120)  # trainer finished its push
  full = globals_for(params)
  ok = all(torch.equal(dest[(vi, 0)].cpu().view(torch.int16),
                       full[vi].to(torch.bfloat16).view(torch.int16)) for vi in range(len(specs)))
  result.put(ok)


def _trainer(q_in, q_out):
  import torch
  from tpu_sync_b200 import reshard_plan as rp, workloads
  from tpu_sync_b200.weight_synchronizer import WeightSynchronizer, import_destinations
  torch.cuda.set_device(0)
  params = small_params()
  specs = [rp.VariableSpec(n, s, workloads.mesh_for(s, "fsdp", 1), workloads.mesh_for(s, sp, 1),
                           layer_idx=i) for i, (n, s, sp) in enumerate(params)]
  plan = rp.build_plan(specs)
  full = globals_for(params)
  grid = [[t.cuda(0)] for t in full]
  dest = import_destinations(q_in.get(timeout=120))
  WeightSynchronizer(grid).push_weights_resharded(plan, {0: 0}, dest).Await()
  torch.cuda.synchronize(0)
  q_out.put("done")


def test_cross_process_ipc_reshard():
  two_gpus()
  ctx = mp.get_context("spawn")
  to_trainer, to_sampler, result = ctx.Queue(), ctx.Queue(), ctx.Queue()
  ps = ctx.Process(target=_sampler, args=(to_trainer, to_sampler, result))
  pt = ctx.Process(target=_trainer, args=(to_trainer, to_sampler))
  ps.start()
  pt.start()
  pt.join(timeout=180)
  ok = result.get(timeout=180)
  ps.join(timeout=60)
  assert pt.exitcode == 0 and ps.exitcode == 0
  assert ok


def test_pool_reshard_plan_into_peer_gpu():
  """C3-shaped pool plan executed on cuda:0, storing into cuda:1's pages."""
  two_gpus()
  from tpu_sync_b200.pool_reshard import PoolReshardProgram, build_pool_reshard_plan
  rng = np.random.default_rng(4)
  n_st, n_seqs, T, H, HB = 3, 2, 512, 2, 256
  sbps, dbps = T // 16, T // 64
  st = rng.permutation(n_seqs * sbps).reshape(n_seqs, sbps).astype(np.int32)
  dt = rng.permutation(n_seqs * dbps).reshape(n_seqs, dbps).astype(np.int32)
  src_pools, dst_pools, dst_ids, r = workloads.handoff_pool_plan_inputs(n_st, st, dt, H, HB)
  plan = build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids, [(0, r)])
  g = torch.Generator().manual_seed(2)
  src = [torch.randint(0, 256, (n_seqs * sbps, 16 * H * HB), generator=g,
                       dtype=torch.uint8).cuda(0) for _ in range(n_st)]
  dst = [torch.zeros((n_seqs * dbps, 64 * H * HB), dtype=torch.uint8, device="cuda:1")
         for _ in range(n_st)]
  PoolReshardProgram(plan, 0, src, dst).launch()
  torch.cuda.synchronize(0)
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  for s in range(n_st):
    want = np.zeros((n_seqs * dbps, 64 * H * HB), np.uint8)
    ors.relayout(src[s].cpu().numpy(), want, sg, dg, st, dt, T)
    np.testing.assert_array_equal(dst[s].cpu().numpy(), want)


def test_block_handoff_across_gpus():
  """register_read / start_read between managers on two GPUs: in one process
  (peer pointers) and across processes (CUDA IPC), the consumer's kernel
  loading the producer's blocks over NVLink."""
  two_gpus()
  from tpu_sync_b200 import KVCacheManager
  from test_gpu_handoff import poll_until, pool, run_cross_process
  src, dst = pool(1, torch.device("cuda", 0)), pool(2, torch.device("cuda", 1))
  prod = KVCacheManager([[t] for t in src], host_blocks_to_allocate=4)
  cons = KVCacheManager([[t] for t in dst], host_blocks_to_allocate=4)
  prod.register_read("peer", 3, [7, 8, 9])
  cons.start_read("peer", 3, prod.get_local_endpoints(), [7, 8, 9], [60, 61, 62])
  assert "peer" in poll_until(cons, 1, "peer")
  torch.cuda.synchronize(1)
  for l in range(len(src)):
    assert torch.equal(dst[l][60:63].cpu(), src[l][7:10].cpu())
  assert "peer" in poll_until(prod, 0, "peer")
  prod.close()
  cons.close()
  run_cross_process(0, 1)


def _pull_case(n_src, n_dst):
  specs = workloads.weight_sync_specs(n_src, n_dst, small_params())
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, n_src, n_dst)
  return specs, plan, layout


def _pull_expected(plan, layout, flats, d, n_src):
  out = np.zeros(layout[1][d][1], np.uint16)
  chunks = workloads.weight_sync_pull_chunks(plan, layout, d, 0, n_src)
  for s in range(n_src):
    ors.apply_element_chunks(flats[s], out, [(so, dp // 2 + do, size, ss, ds, cnt)
                                             for (t, dp, so, do, size, ss, ds, cnt) in chunks
                                             if t == s], cast_bf16=True)
  return out


def test_staged_pull_across_gpus_in_process():
  """Trainers' staging on cuda:0, samplers on cuda:1 reading it over NVLink
  (peer pointers in one process), two generations, oracle-exact."""
  two_gpus()
  import os
  specs, plan, layout = _pull_case(2, 2)
  srcs = [torch.empty(layout[0][s][1], dtype=torch.float32, device="cuda:0") for s in range(2)]
  senders = [ops.PullSender(f"tsb_multi_pull_{os.getpid()}_{s}", srcs[s], groups=4)
             for s in range(2)]
  dsts = [torch.zeros(layout[1][d][1], dtype=torch.bfloat16, device="cuda:1") for d in range(2)]
  recv = [ops.PullReceiver([x.name for x in senders],
                           workloads.weight_sync_pull_chunks(plan, layout, d, dsts[d].data_ptr(), 2),
                           torch.device("cuda:1")) for d in range(2)]
  try:
    for gen in range(2):
      g = torch.Generator().manual_seed(40 + gen)
      flats = [(torch.randn(layout[0][s][1], generator=g) * 0.02).float() for s in range(2)]
      for s in range(2):
        srcs[s].copy_(flats[s])
        senders[s].stage(torch.cuda.current_stream(0))
      for r in recv:
        r.pull(torch.cuda.current_stream(1))
      torch.cuda.synchronize(0)
      torch.cuda.synchronize(1)
      for d in range(2):
        got = dsts[d].view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got, _pull_expected(plan, layout,
                                                          [f.numpy() for f in flats], d, 2))
  finally:
    for r in recv:
      r.close()
    for x in senders:
      x.close()


def _pull_sender_proc(mailbox, n, seed, q_ready, q_go):
  import torch as t
  from tpu_sync_b200 import ops as o
  t.cuda.set_device(0)
  g = t.Generator().manual_seed(seed)
  src = (t.randn(n, generator=g) * 0.02).float().to("cuda:0")
  snd = o.PullSender(mailbox, src, groups=5)
  q_ready.put("READY")
  assert q_go.get(timeout=120) == "GO"
  snd.stage()
  snd.wait()
  q_ready.put("STAGED")
  assert q_go.get(timeout=120) == "EXIT"
  snd.close()
  q_ready.put("BYE")


def test_staged_pull_from_a_sender_process_on_the_other_gpu():
  """Trainer process on cuda:0, sampler (this process) on cuda:1: the
  staging crosses processes by CUDA IPC and GPUs over NVLink."""
  two_gpus()
  import os
  specs, plan, layout = _pull_case(1, 1)
  n = layout[0][0][1]
  mailbox = f"tsb_multi_pullx_{os.getpid()}"
  ctx = mp.get_context("spawn")
  q_ready, q_go = ctx.Queue(), ctx.Queue()
  p = ctx.Process(target=_pull_sender_proc, args=(mailbox, n, 91, q_ready, q_go))
  p.start()
  try:
    assert q_ready.get(timeout=180) == "READY"
    dst = torch.zeros(layout[1][0][1], dtype=torch.bfloat16, device="cuda:1")
    rcv = ops.PullReceiver([mailbox], workloads.weight_sync_pull_chunks(plan, layout, 0,
                                                                        dst.data_ptr(), 1),
                           torch.device("cuda:1"))
    q_go.put("GO")
    rcv.pull(torch.cuda.current_stream(1), timeout_ms=60000)
    torch.cuda.synchronize(1)
    assert q_ready.get(timeout=120) == "STAGED"
    g = torch.Generator().manual_seed(91)
    flat = (torch.randn(n, generator=g) * 0.02).float().numpy()
    np.testing.assert_array_equal(dst.view(torch.int16).cpu().numpy().view(np.uint16),
                                  _pull_expected(plan, layout, [flat], 0, 1))
    rcv.close()
    q_go.put("EXIT")
    assert q_ready.get(timeout=120) == "BYE"
    p.join(timeout=60)
  finally:
    if p.is_alive():
      p.kill()
      p.join()

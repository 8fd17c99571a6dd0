#!/usr/bin/env python
"""Benchmark of the KV offload/reload hot path (config C1, Llama-3-8B KV tier).

One step = offload one 512-block batch (extract kernel HBM pages -> HBM
staging, copy-engine DMA -> pinned host tier) and reload another 512-block
batch (DMA host tier -> staging, insert kernel -> HBM pages), both directions
in flight together.  A block is 2 MiB (32 layers x K/V x 16 tokens x 8 heads x
128 x bf16), so a step moves 1 GiB each way over PCIe.

  value      offload + reload bytes of all ranks / device time (CUDA events,
             max over ranks), through the C ABI manager with the pool resident
             in HBM and block lists prepared before the timed region
  e2e        the same through the Python KVCacheManager.d2h/h2d API from
             Python lists, Await() on each step, host wall clock
  roofline   the kernel with the most live device time (the reload's insert
             kernel pulling the mapped host tier): host-tier bytes it moved /
             its device time, CUDA events around every launch in the timed
             region, against the pinned-memcpy peak of its direction
  pcie       achieved D2H / H2D GB/s of the step against pinned-memcpy peaks
             measured in this run (at N > 1 with all ranks copying at once)
             and the Gen5 x16 spec (64 GB/s)
  cpu_baseline  the reference's host copy loops restated in C (oracle/cpu_ref.c)
             on this box's host cores, on a bounded sample of the workload

`--impl reference` times that CPU restatement alone (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KV offload/reload GB/s per GPU vs PCIe peak; extract HBM GB/s; 8B weight-sync s"
GIB = 1 << 30
# C1 geometry (Llama-3-8B KV): 32 layers x K/V storages of 16-token blocks of
# 8 heads x 128 bf16.  Stated here so the CPU reference arm needs nothing from
# the product package; the GPU arm checks the package's C1 against it.
C1_STORAGES = 32 * 2
C1_STORAGE_BLOCK_BYTES = 16 * 8 * 128 * 2     # 32 KiB
C1_BLOCK_BYTES = C1_STORAGES * C1_STORAGE_BLOCK_BYTES  # 2 MiB
PCIE_SPEC_GBS = 64.0
# DRAM bytes per 2 MiB block moved by the insert kernel, from
# profiles/insert_kernel_c1_256blocks.md (mean of the two captured launches).
INSERT_TRAFFIC_PER_BLOCK = 1019588608 / 256
# DRAM bytes per 2 MiB block moved by the extract kernel (HBM pool -> HBM
# staging): the 16-byte vector kernel (profiles/extract_kernel_c1_256blocks.md)
# and the bulk-copy kernel (profiles/bulk_copy_kernel_c1_256blocks.md), mean
# of the two captured launches each.
VEC_EXTRACT_TRAFFIC_PER_BLOCK = 1018413568 / 256
BULK_EXTRACT_TRAFFIC_PER_BLOCK = 1026581632 / 256
# DRAM bytes per 2 MiB block of the insert kernel pulling from the mapped host
# tier (reload direct), from profiles/insert_direct_kernel_c1_256blocks.md
# (HBM writes; its host reads cross PCIe, not DRAM).
INSERT_DIRECT_TRAFFIC_PER_BLOCK = 477387264 / 256


def parse():
  p = argparse.ArgumentParser()
  p.add_argument("--gpus", type=int, default=1)
  p.add_argument("--steps", type=int, default=10)
  p.add_argument("--warmup", type=int, default=3)
  p.add_argument("--impl", choices=["ours", "reference"], default="ours")
  p.add_argument("--batch", type=int, default=512)
  p.add_argument("--pool-blocks", type=int, default=32768)
  p.add_argument("--host-blocks", type=int, default=0, help="0 = size to host RAM")
  p.add_argument("--cpu-sample-s", type=float, default=10.0)
  p.add_argument("--no-cpu-baseline", action="store_true")
  p.add_argument("--no-exchange", action="store_true",
                 help="skip the N>=2 weight-sync and hand-off measurements")
  p.add_argument("--mode", default="direct_h2d",
                 choices=["staged", "direct_d2h", "direct_h2d", "direct"],
                 help="C1 manager transfer mode (staged: copy-engine DMAs through HBM "
                      "staging; direct*: SM-driven PCIe to the mapped host tier).  "
                      "direct_h2d (reloads pulled by the insert kernel, offloads by copy "
                      "engine) measured fastest with both directions in flight")
  p.add_argument("--copy-streams", type=int, default=2)
  p.add_argument("--chunk-blocks", type=int, default=0, help="0 = manager default")
  p.add_argument("--max-ctas", type=int, default=0, help="kernel grid cap, 0 = default")
  p.add_argument("--sched", default="offload_priority,reload_per_piece,bulk_copy",
                 help="comma-separated manager sched flags: offload_priority, "
                      "reload_per_piece, reload_overlap, bulk_copy ('' = none)")
  p.add_argument("--reload-staged-every", type=int, default=0,
                 help="direct reloads: every n-th chunk through the copy engines (0 = none)")
  p.add_argument("--kernel-case", default="",
                 choices=["", "extract", "insert", "extract_fp8", "insert_fp8", "pool_reshard",
                          "insert_direct", "relayout", "manager_extract",
                          "manager_insert", "reshard_cast", "reshard_copy"],
                 help="run a few launches of one kernel on a small case (for ncu)")
  return p.parse_args()


def peaks():
  try:
    return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
  except Exception:
    return {}


def mem_available_bytes() -> int:
  try:
    for line in open("/proc/meminfo"):
      if line.startswith("MemAvailable:"):
        return int(line.split()[1]) * 1024
  except OSError:
    pass
  return 64 * GIB


def cpu_model() -> str:
  try:
    for line in open("/proc/cpuinfo"):
      if line.startswith("model name"):
        return line.split(":", 1)[1].strip()
  except OSError:
    pass
  return "unknown"


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
  """nvidia-smi clock / throttle samples (every 50 ms) around a timed region.

  start() returns once the first sample has arrived, so the sampler is live
  before the region begins; begin() / end() bracket the region; stop() waits
  for one sample after the region and summarises those taken inside it (plus
  that one)."""
  QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

  def __init__(self, device_index: int):
    self.dev = device_index
    self.proc = None
    self.lines = []  # (monotonic time, csv line)
    self.t0 = self.t1 = None

  def start(self):
    try:
      self.proc = subprocess.Popen(
          ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
           "-lms", "50", "-i", str(self.dev)], stdout=subprocess.PIPE,
          stderr=subprocess.DEVNULL, text=True)
      self.thread = threading.Thread(target=self._read, daemon=True)
      self.thread.start()
    except OSError:
      self.proc = None
      return
    deadline = time.monotonic() + 10.0
    while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
      time.sleep(0.01)

  def begin(self):
    self.t0 = time.monotonic()

  def end(self):
    self.t1 = time.monotonic()

  def _read(self):
    for line in self.proc.stdout:
      self.lines.append((time.monotonic(), line.strip()))

  def stop(self):
    if self.proc is None:
      return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
    t1 = self.t1 if self.t1 is not None else time.monotonic()
    t0 = self.t0 if self.t0 is not None else t1
    deadline = time.monotonic() + 2.0
    while (not any(t > t1 for t, _ in self.lines) and time.monotonic() < deadline
           and self.proc.poll() is None):
      time.sleep(0.01)
    self.proc.terminate()
    try:
      self.proc.wait(timeout=5)
    except subprocess.TimeoutExpired:
      self.proc.kill()
    after = [t for t, _ in self.lines if t > t1]
    t_hi = min(after) if after else t1
    window = [l for t, l in self.lines if t0 <= t <= t_hi]
    sm, smax, reasons = [], None, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    for line in window:
      f = [x.strip() for x in line.split(",")]
      if len(f) < 9:
        continue
      try:
        sm.append(float(f[1]))
        smax = float(f[2])
      except ValueError:
        continue
      for name, val in zip(names, f[5:9]):
        if val.lower() == "active":
          reasons.add(name)
    return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
            "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU arms (oracle restatement of the reference host loops)
# ---------------------------------------------------------------------------

def c1_plans(rank: int, host_blocks: int, pool_blocks: int, batch: int, n_steps: int,
             source: str = "product"):
  """Step plans of the C1 trace (see run_ours): per step (offload device ids,
  offload host ids, reload host ids, reload device ids).

  source "product": the trace runs through the product's tier-2 store;
  "reference": through the reference's own LRU and block allocator compiled
  from source (oracle/_ref/store_trace_ref), which imports nothing from the
  product.  Both give the same plans (tests/test_cpu_store.py)."""
  if source == "reference":
    from oracle import store_trace
    trace = store_trace.zipf_trace(seed=10 + rank)
    batches, stats = store_trace.transfer_streams(trace, host_blocks, pool_blocks, batch)
  else:
    from tpu_sync_b200 import workloads
    trace = workloads.zipf_trace(seed=10 + rank)
    batches, stats = workloads.store_transfer_streams(trace, host_blocks, pool_blocks, batch)
  half_pool = pool_blocks // 2
  # A step gathers consecutive access batches, in trace order, until `batch`
  # reloads (or offloads) are pending: its offloads and reloads go out
  # together (a reload that depends on an offload of the same step waits for
  # it inside the manager).
  steps, cur_s, cur_l = [], [], []
  for sv, ld in batches[len(batches) // 2:]:
    cur_s += sv
    cur_l += ld
    if len(cur_l) >= batch or len(cur_s) >= batch:
      steps.append((cur_s, cur_l))
      cur_s, cur_l = [], []
  if len(steps) < n_steps:
    raise RuntimeError(f"C1 trace yields {len(steps)} steps, {n_steps} requested")
  plans = []
  for sv, ld in steps[:n_steps]:
    plans.append((np.array([d % half_pool for d, _ in sv], np.int64),
                  np.array([h for _, h in sv], np.int64),
                  np.array([h for h, _ in ld], np.int64),
                  np.array([half_pool + d % half_pool for _, d in ld], np.int64)))
  return plans, stats


def c1_host_blocks(args, world: int) -> int:
  """Host tier blocks of the C1 configuration: as many as requested (default
  32768 = 64 GiB), bounded by this box's RAM share per local rank: 45 % of
  the available RAM for one rank, 30 % in total when ranks share the host
  (with eight ranks pinning 45 % of a 1 TB host, later pinned allocations
  of the run were refused)."""
  want = args.host_blocks or 32768
  local_ranks = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
  share = 0.45 if local_ranks <= 1 else 0.30
  fit = int(share * mem_available_bytes() / max(local_ranks, 1) // C1_BLOCK_BYTES)
  return max(4 * args.batch, min(want, fit))


def host_memory_state() -> dict:
  """Host memory figures that bound pinned allocations (GiB)."""
  out = {}
  try:
    for line in open("/proc/meminfo"):
      k, v = line.split(":", 1)
      if k in ("MemTotal", "MemAvailable", "Mlocked", "Unevictable"):
        out[k] = round(int(v.split()[0]) / 2**20, 1)
  except OSError:
    pass
  for name in ("memory.current", "memory.max"):
    try:
      v = open(f"/sys/fs/cgroup/{name}").read().strip()
      out[name] = v if v == "max" else round(int(v) / 2**30, 1)
    except (OSError, ValueError):
      pass
  return out


def make_manager(KVCacheManager, grid, attempts: int = 6, **kw):
  """A manager whose pinned host tier may be refused for a moment right after
  another leg freed a large one (seen with eight ranks on one host): retries
  a few times, and on the last failure reports the host memory state."""
  for i in range(attempts):
    try:
      return KVCacheManager(grid, **kw)
    except RuntimeError as e:
      if "cudaHostAlloc" not in str(e) or i == attempts - 1:
        raise RuntimeError(f"{e} (host memory: {host_memory_state()})") from e
      time.sleep(2.0)


def c1_config(args, host_blocks: int, plans, trace_stats, world: int) -> dict:
  """The `config` of both arms' JSON lines (same workload, same plans)."""
  pitch = C1_BLOCK_BYTES
  pool_bytes = args.pool_blocks * pitch
  return {
      "workload": ("C1 Llama-3-8B KV tier: 32 layers x K/V, 16-token blocks of "
                   "8 heads x 128 bf16 (2 MiB per block); per step the offloads "
                   "(misses) and reloads (hits) of consecutive 512-access batches "
                   "of the Zipf trace until 512 reloads are pending, both "
                   "directions in flight"),
      "blocks_per_step": round(sum(len(p[0]) + len(p[2]) for p in plans[args.warmup:])
                               / args.steps, 1),
      "pool_blocks": args.pool_blocks, "pool_gib": round(pool_bytes / GIB, 1),
      "host_tier_blocks": host_blocks,
      "host_tier_gib": round(host_blocks * pitch / GIB, 1),
      "batch": args.batch,
      "l2": "inputs larger than L2 (~1 GiB of scattered 2 MiB blocks per step)",
      "trace": ("100k accesses Zipf(1.1) over 200k prefix ids (seed 10+rank), batches "
                "of 512, through the tier-2 store (reference LRU + host block "
                "allocator); steps from the middle of the trace"),
      "trace_hit_rate": trace_stats["hit_rate"],
      "parallelism": f"replicas x{world}"}


def cpu_offload_reload(plans, seconds: float, steps: int = 0, warmup: int = 0):
  """Times the reference host loops (restated in C) on the C1 step plans.

  The reference's CPU client keeps its "device" buffers in host memory, so a
  host-resident pool stands in for HBM; block ids are folded into a
  2048-block pool and a 2048-block host tier (every copy stays a 32 KiB run
  per storage, as in the real layout).
  """
  from oracle import cpu_ref
  S, bb = C1_STORAGES, C1_STORAGE_BLOCK_BYTES
  nb = 2048
  threads = cpu_ref.host_threads()
  dev = [np.empty(nb * bb, np.uint8) for _ in range(S)]
  host = [np.empty(nb * bb, np.uint8) for _ in range(S)]
  for a in dev + host:
    a.fill(1)
  folded = [tuple(np.asarray(x) % nb for x in p) for p in plans]

  def one_step(p):
    ones_s = np.ones(len(p[0]), np.int64)
    ones_l = np.ones(len(p[2]), np.int64)
    cpu_ref.copy_runs(host, dev, [bb] * S, p[0], p[1], ones_s, threads)   # D2H
    cpu_ref.copy_runs(dev, host, [bb] * S, p[2], p[3], ones_l, threads)   # H2D

  for i in range(warmup):
    one_step(folded[i % len(folded)])
  times, moved = [], 0
  t_end = time.perf_counter() + seconds
  i = 0
  while (steps and len(times) < steps) or (not steps and (time.perf_counter() < t_end or
                                                          len(times) < 2)):
    p = folded[(warmup + i) % len(folded)]
    t0 = time.perf_counter()
    one_step(p)
    times.append(time.perf_counter() - t0)
    moved += (len(p[0]) + len(p[2])) * C1_BLOCK_BYTES
    i += 1
  total = sum(times)
  return {"value": round(moved / total / 1e9, 3), "unit": "GB/s", "cores": threads,
          "ms_per_step": total / len(times) * 1e3, "steps": len(times),
          "sample": (f"{len(times)} steps of the C1 trace plans (offloads + reloads of one "
                     f"512-access batch each, 2 MiB blocks) between a {nb}-block "
                     f"host-resident pool and a {nb}-block host tier, memcpy per (storage, "
                     f"run) as DispatchD2hWork/DispatchH2dWork on the CPU client"),
          "cpu": cpu_model()}


def _timed_loop(fn, seconds: float, min_iters: int = 2):
  """Runs fn() for about `seconds` (at least min_iters times); returns (iters, s)."""
  t0 = time.perf_counter()
  n = 0
  while n < min_iters or time.perf_counter() - t0 < seconds:
    fn()
    n += 1
  return n, time.perf_counter() - t0


def cpu_c2_fp8(seconds: float):
  """C2 offload on the host cores: gather + per-(block, storage) absmax scale
  + e4m3 cast of 256 random blocks of the 80-layer x K/V shard (the C
  restatement, all threads), from a 512-block host-resident sample pool."""
  from oracle import cpu_ref
  from tpu_sync_b200 import workloads
  g = workloads.C2
  n_st, blocks, B = g.storages, 256, workloads.C2_BATCH
  elems = g.storage_block_bytes // 2
  rng = np.random.default_rng(20)
  # 40 distinct 4 MiB storages (160 MiB, more than a host L3) cycled over the
  # 160 storage slots keeps the set-up short
  distinct = [(rng.standard_normal((blocks, elems), np.float32).view(np.uint32) >> 16)
              .astype(np.uint16) for _ in range(40)]
  pool = [distinct[i % len(distinct)] for i in range(n_st)]
  ids = rng.permutation(blocks).astype(np.int64)
  offs = [s * elems for s in range(n_st)]  # fp8 payload: elems bytes per storage
  scale_off = n_st * elems
  pitch = scale_off + 4 * n_st
  staging = np.zeros((B, pitch), np.uint8)
  threads = cpu_ref.host_threads()
  n, sec = _timed_loop(lambda: cpu_ref.extract_fp8(pool, ids, staging, pitch, offs, scale_off,
                                                   threads), seconds)
  return {"value": round(n * B * g.block_bytes / sec / 1e9, 2), "unit": "GB/s of bf16 offloaded",
          "cores": threads, "kind": "port",
          "sample": f"{n} offloads of 256 blocks in random order (gather + absmax scale + e4m3 "
                    "cast, oracle/cpu_ref.c) of the C2 geometry, 160 MiB of distinct host data"}


def cpu_c3_relayout(seconds: float):
  """C3 permute on the host cores: one of the 8 sequences (1 GiB of the 8 GiB
  per pair), 64 storages, head-major 16-token pages -> token-major 64-token."""
  from oracle import cpu_ref
  n_st, T, H, HB = 64, 32768, 2, 256
  rng = np.random.default_rng(30)
  st = rng.permutation(T // 16).reshape(1, -1).astype(np.int32)
  dt = rng.permutation(T // 64).reshape(1, -1).astype(np.int32)
  src = [rng.integers(0, 256, (T // 16) * 16 * H * HB, dtype=np.uint8) for _ in range(n_st)]
  dst = [np.empty((T // 64) * 64 * H * HB, np.uint8) for _ in range(n_st)]
  threads = cpu_ref.host_threads()
  n, sec = _timed_loop(lambda: cpu_ref.relayout(src, dst, H, HB, 16, 64, st, dt, T, threads),
                       seconds)
  moved = n_st * T * H * HB
  return {"value": round(n * moved / sec / 1e9, 2), "unit": "GB/s", "cores": threads,
          "kind": "port",
          "sample": f"{n} relayouts of one 32768-token sequence x 64 storages x 2 heads "
                    "(1 GiB; oracle/cpu_ref.c, a 256-byte memcpy per head vector)"}


def cpu_c4_reshard(plan, specs, seconds: float):
  """C4 on the host cores: the planner's chunks of the first decoder layer
  (q, k, v, o, gate, up, down, 2 norms) applied fp32 -> bf16 (RNE) with all
  threads, source shard 0 to every destination shard."""
  import math
  from oracle import cpu_ref
  from tpu_sync_b200 import reshard_plan as rp
  chosen = [i for i, v in enumerate(specs) if v.name.startswith("layers.0.")]
  src_sizes = {v: math.prod(rp.local_shape(
      rp.shard_boxes(specs[v].shape, specs[v].src_mesh)[specs[v].src_box_of(0)])) for v in chosen}
  src_off, tot = {}, 0
  for v in chosen:
    src_off[v], tot = tot, tot + src_sizes[v]
  chunks, dst_off, dtot = [], {}, 0
  for (vi, d), cs in plan.for_source(0).items():
    if vi not in src_off:
      continue
    n_dst = math.prod(rp.local_shape(
        rp.shard_boxes(specs[vi].shape, specs[vi].dst_mesh)[specs[vi].dst_box_of(d)]))
    if (vi, d) not in dst_off:
      dst_off[(vi, d)], dtot = dtot, dtot + n_dst
    for (so, do, size, ss, ds, cnt) in cs:
      chunks.append((src_off[vi] + so, dst_off[(vi, d)] + do, size, ss, ds, cnt))
  rng = np.random.default_rng(3)
  src = (rng.standard_normal(tot, np.float32) * np.float32(0.02))
  dst = np.empty(dtot, np.uint16)
  threads = cpu_ref.host_threads()
  n, sec = _timed_loop(lambda: cpu_ref.reshard_f32_bf16(src, dst, chunks, threads), seconds)
  return {"value": round(n * 2 * dtot / sec / 1e9, 2), "unit": "GB/s of bf16 written",
          "cores": threads, "kind": "port",
          "sample": f"{n} pushes of decoder layer 0 ({tot / 1e6:.0f} M params, "
                    f"{len(chunks)} chunks; oracle/cpu_ref.c fp32 -> bf16 RNE)"}


def run_reference(args):
  rank = int(os.environ.get("RANK", "0"))
  if rank != 0:
    return
  world = int(os.environ.get("WORLD_SIZE", "1"))
  host_blocks = c1_host_blocks(args, world)
  try:
    plans, stats = c1_plans(0, host_blocks, args.pool_blocks, args.batch,
                            args.warmup + args.steps, source="reference")
  except (OSError, RuntimeError) as e:
    print(json.dumps({"impl": "reference",
                      "unavailable": f"reference store trace driver unavailable: {e}"}))
    return
  r = cpu_offload_reload(plans, 0.0, steps=args.steps, warmup=args.warmup)
  line = {"impl": "reference", "metric": METRIC, "value": r["value"], "unit": "GB/s",
          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
          "ms_per_step": round(r["ms_per_step"], 3), "higher_is_better": True,
          "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
          "data": "synthetic (host-resident pool standing in for the CPU client's device)",
          "config": c1_config(args, host_blocks, plans, stats, world),
          "cpu_baseline": {"value": r["value"], "unit": "GB/s", "cores": r["cores"],
                           "kind": "port", "sample": r["sample"]},
          "e2e": {"value": r["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                  "d2h_bytes_per_step": 0}}
  print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def c1_seed_host_blocks(plans, executed, half_pool):
  """Host blocks the executed steps reload before any of them offloads
  there (blocks the trace saved before the steps that run): host block h ->
  pool block h mod half_pool, which an untimed offload puts there before
  the warm-up, so every reload moves known bytes."""
  written, seed = set(), {}
  for i in executed:
    off_d, off_h, ld_h, ld_d = plans[i]
    written.update(off_h.tolist())
    for h in ld_h.tolist():
      if h not in written and h not in seed:
        seed[h] = h % half_pool
  return seed


def c1_expected_sources(plans, executed, seed=None):
  """The pool block whose bytes each reloaded pool block must hold after the
  steps `executed` (plan indices, in order) over a host tier seeded as
  `seed` says: a step's offloads go before its reloads (the manager orders
  a reload after an earlier call's offload of the same host block), and
  within a call the last copy to a block wins.  Offloads read the pool's
  first half, which nothing writes, and reloads write its second half.  A
  reload of a host block of unknown content is left out."""
  host_src, dev_src = dict(seed or {}), {}
  for i in executed:
    off_d, off_h, ld_h, ld_d = plans[i]
    for d, h in zip(off_d.tolist(), off_h.tolist()):
      host_src[h] = d
    for h, d in zip(ld_h.tolist(), ld_d.tolist()):
      dev_src[d] = host_src.get(h)
  return {d: s for d, s in dev_src.items() if s is not None}


def c1_blocks_differ(torch, full, expected, device, batch=512) -> int:
  """Pool blocks (all layers, K and V) that differ bitwise from the block
  `expected` names; `full` is the [layers, 2, blocks, ...] bf16 pool."""
  if not expected:
    return 0
  dst = torch.tensor(sorted(expected), dtype=torch.int64, device=device)
  src = torch.tensor([expected[int(d)] for d in dst.tolist()], dtype=torch.int64, device=device)
  bad = torch.zeros(dst.numel(), dtype=torch.bool, device=device)
  bits = full.view(torch.int16)
  for l in range(full.shape[0]):
    for k0 in range(0, dst.numel(), batch):
      d_, s_ = dst[k0:k0 + batch], src[k0:k0 + batch]
      a = bits[l].index_select(1, d_)
      b = bits[l].index_select(1, s_)
      bad[k0:k0 + batch] |= (a != b).flatten(2).any(dim=2).any(dim=0)
  return int(bad.sum().item())


def measure_pcie(torch, device, nbytes=GIB, barrier=None):
  """Best-of-3 pinned cudaMemcpyAsync D2H, H2D and both at once (GB/s).

  With `barrier` (N > 1) every trial starts on all ranks together, so the
  figures are per-GPU peaks with all N GPUs copying at once: the host link
  and host memory they share are part of the measured peak."""
  d = torch.empty(nbytes, dtype=torch.uint8, device=device)
  d2 = torch.empty(nbytes, dtype=torch.uint8, device=device)
  h = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
  h2 = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
  s1, s2 = torch.cuda.Stream(device), torch.cuda.Stream(device)
  out = {}
  for name in ("d2h", "h2d", "duplex"):
    best = 0.0
    for _ in range(3):
      torch.cuda.synchronize(device)
      if barrier is not None:
        barrier()
      e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      e2 = torch.cuda.Event(enable_timing=True)
      e0.record(s1)
      s2.wait_event(e0)
      if name in ("d2h", "duplex"):
        with torch.cuda.stream(s1):
          h.copy_(d, non_blocking=True)
      if name in ("h2d", "duplex"):
        with torch.cuda.stream(s2):
          d2.copy_(h2, non_blocking=True)
      e2.record(s2)
      s1.wait_event(e2)
      e1.record(s1)
      torch.cuda.synchronize(device)
      ms = e0.elapsed_time(e1)
      moved = nbytes * (2 if name == "duplex" else 1)
      best = max(best, moved / (ms * 1e-3) / 1e9)
    out[name] = round(best, 2)
  del d, d2, h, h2
  return out


def c4_shards_exact(torch, device, params, half, d, flat):
  """Sampler d's bf16 TP shards against their definition, recomputed with
  torch on this GPU (no product planner or kernel): each trainer t's fp32
  FSDP buffer is regenerated from its seed (3 + t; the same CUDA generator
  stream the trainer drew), every parameter's global tensor is reassembled
  from the trainers' dim-0 slices, and sampler d's shard is the dim-0
  (column-parallel, vocab) or dim-1 (row-parallel) slice d of `half`, or the
  whole tensor (replicated norms), cast to bf16 round-to-nearest-even.
  Returns the names of the parameters whose bytes differ."""
  import math
  sizes = [math.prod(shape) // half for _, shape, _ in params]
  total = sum(sizes)
  trainers = []
  for t in range(half):
    x = torch.empty(total, dtype=torch.float32, device=device)
    x.normal_(0.0, 0.02, generator=torch.Generator(device=device).manual_seed(3 + t))
    trainers.append(x)
  bad, soff, doff = [], 0, 0
  for (name, shape, split), n in zip(params, sizes):
    rows = shape[0] // half
    full = torch.cat([trainers[t][soff:soff + n].view((rows,) + tuple(shape[1:]))
                      for t in range(half)])
    if split in ("col", "vocab"):
      want = full[d * (shape[0] // half):(d + 1) * (shape[0] // half)]
    elif split == "row":
      want = full[:, d * (shape[1] // half):(d + 1) * (shape[1] // half)]
    else:
      want = full
    want = want.to(torch.bfloat16).contiguous()
    got = flat[doff:doff + want.numel()].view(want.shape)
    if not torch.equal(got.view(torch.int16), want.view(torch.int16)):
      bad.append(name)
    soff += n
    doff += want.numel()
  if doff != flat.numel():
    bad.append(f"<layout: {doff} of {flat.numel()} elements>")
  del trainers
  torch.cuda.empty_cache()
  return bad


def run_weight_sync(torch, dist, rank, world, device, steps, warmup):
  """C4: Llama-3-8B fp32 FSDP shards on ranks [0, half) -> TP bf16 shards on
  ranks [half, 2*half), one reshard kernel per trainer rank storing straight
  into the sampler ranks' memory (CUDA IPC mappings, NVLink P2P stores)."""
  import math
  from tpu_sync_b200 import ops, reshard_plan as rp, workloads
  from tpu_sync_b200.weight_synchronizer import (close_imports, export_destinations,
                                                 import_destinations)
  half = world // 2
  is_src = rank < half
  idx = rank if is_src else rank - half
  params = workloads.llama3_8b_params()
  specs = workloads.weight_sync_specs(half, half, params)
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, half, half)
  src_total = layout[0][idx][1] if is_src else 0
  dst_offs = layout[1]
  if is_src:
    flat = torch.empty(src_total, dtype=torch.float32, device=device)
    flat.normal_(0.0, 0.02, generator=torch.Generator(device=device).manual_seed(3 + idx))
    desc = None
  else:
    flat = torch.zeros(dst_offs[idx][1], dtype=torch.bfloat16, device=device)
    desc = export_destinations({0: flat})
  descs = [None] * world
  dist.all_gather_object(descs, desc)
  per_push_ms, prog, prog_ce, ce_error = 0.0, None, None, ""
  if is_src:
    dsts = {d: import_destinations(descs[half + d], kernel_device=device.index)[0]
            for d in range(half)}
    chunks = workloads.weight_sync_chunks(plan, layout, idx, flat.data_ptr(),
                                          {d: dsts[d].data_ptr() for d in range(half)})
    prog = ops.ReshardProgram(chunks, torch.float32, torch.bfloat16, device)
    for _ in range(warmup):
      prog.launch()
    # the copy-engine leg is a comparison: a launch error there is reported
    # in the line instead of ending the run
    try:
      prog_ce = ops.ReshardCopyEngineProgram(chunks, torch.float32, torch.bfloat16, device)
      for _ in range(warmup):
        prog_ce.launch()
    except RuntimeError as e:
      ce_error = str(e).splitlines()[0][:200]
      prog_ce = None
    torch.cuda.synchronize(device)
  ok = torch.tensor([0 if ce_error else 1], dtype=torch.int32, device=device)
  dist.all_reduce(ok, op=dist.ReduceOp.MIN)
  if not int(ok.item()) and not ce_error:
    ce_error = "failed on another trainer rank"
  dist.barrier()
  ce_ms = 0.0
  mismatched = {}
  for which in (("sm", "copy") if not ce_error else ("sm",)):
    if is_src:
      p_ = prog if which == "sm" else prog_ce
      e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      e0.record()
      for _ in range(steps):
        p_.launch()
      e1.record()
      torch.cuda.synchronize(device)
      if which == "sm":
        per_push_ms = e0.elapsed_time(e1) / steps
      else:
        ce_ms = e0.elapsed_time(e1) / steps
    dist.barrier()
    # after each engine's pushes the samplers check every byte they received,
    # then clear their buffers for the next engine
    if not is_src:
      mismatched[which] = c4_shards_exact(torch, device, params, half, idx, flat)
      flat.zero_()
      torch.cuda.synchronize(device)
    dist.barrier()
  # Staged pull: each trainer casts into its bf16 staging group by group and
  # publishes the groups in a /dev/shm mailbox; each sampler's kernels read
  # the staging over NVLink as the groups appear.  Hybrid (N >= 4): each
  # sampler pulls only from its own-index trainer, and each trainer pushes
  # its slices for the other samplers (the SM push kernel) while it casts, so
  # every trainer has one reader and every sampler one source to read.
  # Timed per rank from one barrier over `steps` back-to-back pushes (a
  # trainer's next stage waits for its readers to finish the previous pull),
  # max over ranks.
  token = [f"{os.getpid()}_{int(time.time() * 1e3) % 10**9}" if rank == 0 else None]
  dist.broadcast_object_list(token, src=0)

  def staged_engine(kind):
    names = [f"tsb_bench_w{kind}_{token[0]}_{t_}" for t_ in range(half)]
    sender = receiver = cross = None
    err, ms = "", 0.0
    side = torch.cuda.Stream(device)
    try:
      if is_src:
        sender = ops.PullSender(names[idx], flat, groups=16)
        if kind == "hybrid":
          cross = ops.ReshardProgram(
              workloads.weight_sync_chunks(plan, layout, idx, flat.data_ptr(),
                                           {d: dsts[d].data_ptr() for d in range(half)},
                                           dst_slots=set(range(half)) - {idx}),
              torch.float32, torch.bfloat16, device)
    except Exception as e:  # reported in the line, never ends the run
      err = str(e).splitlines()[0][:200]
    ok_ = torch.tensor([0 if err else 1], dtype=torch.int32, device=device)
    dist.all_reduce(ok_, op=dist.ReduceOp.MIN)
    if int(ok_.item()):
      try:
        if not is_src:
          srcs_ = {idx} if kind == "hybrid" else None
          pulls = workloads.weight_sync_pull_chunks(plan, layout, idx, flat.data_ptr(), half,
                                                    src_slots=srcs_)
          if kind == "hybrid":
            receiver = ops.PullReceiver([names[idx]], [(0,) + tuple(c[1:]) for c in pulls],
                                        device)
          else:
            receiver = ops.PullReceiver(names, pulls, device)
      except Exception as e:  # reported in the line, never ends the run
        err = str(e).splitlines()[0][:200]
      ok_ = torch.tensor([0 if err else 1], dtype=torch.int32, device=device)
      dist.all_reduce(ok_, op=dist.ReduceOp.MIN)
    if int(ok_.item()):
      def one_push():
        if is_src:
          if cross is not None:  # the cross slices go out while the trainer casts
            side.wait_stream(torch.cuda.current_stream(device))
            cross.launch(side)
          sender.stage(timeout_ms=60000)
          if cross is not None:
            torch.cuda.current_stream(device).wait_stream(side)
        else:
          receiver.pull(timeout_ms=60000)
      def pushes(n):
        try:
          for _ in range(n):
            one_push()
          torch.cuda.synchronize(device)
          return ""
        except Exception as e:  # reported in the line, never ends the run
          torch.cuda.synchronize(device)
          return str(e).splitlines()[0][:200]

      # every rank takes the same collective steps, failed or not
      err = pushes(warmup)
      ok_ = torch.tensor([0 if err else 1], dtype=torch.int32, device=device)
      dist.all_reduce(ok_, op=dist.ReduceOp.MIN)
      if int(ok_.item()):
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        err = pushes(steps)
        e1.record()
        torch.cuda.synchronize(device)
        ms = e0.elapsed_time(e1) / steps
        ok_ = torch.tensor([0 if err else 1], dtype=torch.int32, device=device)
        dist.all_reduce(ok_, op=dist.ReduceOp.MIN)
      if not int(ok_.item()) and not err:
        err = "failed on another rank"
      dist.barrier()
      if not is_src and not err:
        mismatched[kind] = c4_shards_exact(torch, device, params, half, idx, flat)
        flat.zero_()
        torch.cuda.synchronize(device)
    elif not err:
      err = "failed on another rank"
    if receiver is not None:
      receiver.close()  # the samplers' mappings go before the trainers' staging
    dist.barrier()
    if sender is not None:
      sender.close()
    return (0.0 if err else ms), err

  pull_ms, pull_error = staged_engine("pull")
  hyb_ms, hyb_error = staged_engine("hybrid") if half >= 2 else (0.0, "")
  exact = torch.tensor([0 if any(mismatched.values()) else 1], dtype=torch.int32, device=device)
  dist.all_reduce(exact, op=dist.ReduceOp.MIN)
  t = torch.tensor([per_push_ms, ce_ms, pull_ms, hyb_ms], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  sm_s, ce_s, pull_s, hyb_s = (float(t[k].item()) / 1e3 for k in range(4))
  runs = {"sm": sm_s, "copy": ce_s, "pull": pull_s, "hybrid": hyb_s}
  engine = min((k for k, v in runs.items() if v > 0), key=lambda k: runs[k])
  push_s = runs[engine]
  recv_bytes = max(2 * plan.elements_to(d) for d in range(half))
  total_params = sum(math.prod(v.shape) for v in specs)
  del prog
  if prog_ce is not None:
    prog_ce.close()
  if is_src:
    dsts = None
    close_imports(device.index)
  dist.barrier()
  return {"config": f"C4 Llama-3-8B fp32 FSDP {half} ranks -> bf16 TP={half} ({half}->{half})",
          "params": total_params, "seconds": round(push_s, 5),
          "bytes_per_dst_gpu": recv_bytes,
          "nvlink_gbs_per_dst_gpu": round(recv_bytes / push_s / 1e9, 1) if push_s else None,
          "frac_of_nvlink_770": round(recv_bytes / push_s / 1e9 / 770.0, 3) if push_s else None,
          "engine": engine,
          "engines": {"sm": {"how": "one kernel per trainer GPU casting and storing into the "
                                    "samplers' memory over NVLink", "seconds": round(sm_s, 5)},
                      "copy": {"how": "the kernel casts into local staging, the copy engines "
                                      "move each chunk (cudaMemcpy2DAsync), 16 pipelined groups",
                               "seconds": round(ce_s, 5) if not ce_error else None,
                               **({"error": ce_error} if ce_error else {})},
                      "pull": {"how": "each trainer casts into local bf16 staging in 16 groups "
                                      "published through a /dev/shm mailbox; each sampler's "
                                      "kernels load the staging over NVLink as groups appear "
                                      "(back-to-back pushes, each waiting for the previous "
                                      "pull to finish)",
                               "seconds": round(pull_s, 5) if not pull_error else None,
                               **({"error": pull_error} if pull_error else {})},
                      **({"hybrid": {
                          "how": "each sampler pulls from its own-index trainer's staging "
                                 "(as pull); each trainer pushes its slices for the other "
                                 "samplers with the SM kernel while it casts",
                          "seconds": round(hyb_s, 5) if not hyb_error else None,
                          **({"error": hyb_error} if hyb_error else {})}} if half >= 2 else {})},
          "chunks_per_src": len(plan.for_source(0)),
          "exact": bool(int(exact.item())),
          "exact_how": ("every sampler's bf16 TP shards of all parameters, after each "
                        "engine's pushes, equal their definition recomputed with torch "
                        "(global tensors from the trainers' seeded fp32 shards, TP slice, "
                        "RNE cast)")}


def run_pull(torch, dist, rank, world, device, steps, warmup):
  """Block hand-off through the managers' pull protocol (register_read on
  rank i, start_read on rank i + N/2): 512 C1 blocks (1 GiB) per pair and
  step, the consumer's kernel loading the producer's pool over NVLink
  (CUDA IPC).  Device time of the copy on the consumer's stream."""
  from tpu_sync_b200 import KVCacheManager, workloads
  half = world // 2
  is_src = rank < half
  g = workloads.C1
  n_blocks, B = 2048, 512
  full = torch.empty((g.layers, g.kv, n_blocks, g.block_tokens, g.heads, g.head_dim),
                     dtype=torch.bfloat16, device=device)
  full.normal_(generator=torch.Generator(device=device).manual_seed(50 + rank))
  storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]
  mgr = make_manager(KVCacheManager, [[t] for t in storages], host_blocks_to_allocate=4)
  ep = mgr.get_local_endpoints() if is_src else None
  eps = [None] * world
  dist.all_gather_object(eps, ep)
  rng = np.random.default_rng(60)
  ms, host_ms = [], []
  for it in range(warmup + steps):
    src_ids = rng.choice(n_blocks, B, replace=False).tolist()
    dst_ids = rng.choice(n_blocks, B, replace=False).tolist()
    if is_src:
      assert mgr.register_read(f"pull-{it}", 1000 + it, src_ids)
      t0 = time.time()
      while mgr.read_state(1000 + it) != "ready":  # the blocks are written
        if time.time() - t0 > 10:
          raise RuntimeError("registered blocks never became ready")
        time.sleep(0.0002)
    dist.barrier()
    if not is_src:
      s = torch.cuda.current_stream(device)
      e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      # ~5 ms of GPU sleep ahead of e0 keeps the host's start_read (checks,
      # pair upload, launch; its wall time is reported as host_ms) out of the
      # timed window
      torch.cuda._sleep(10_000_000)
      e0.record(s)
      h0 = time.perf_counter()
      mgr.start_read(f"pull-{it}", 1000 + it, eps[rank - half], src_ids, dst_ids)
      h1 = time.perf_counter()
      e1.record(s)
      t0 = time.time()
      while f"pull-{it}" not in mgr.poll_stats()[1]:
        if time.time() - t0 > 30:
          raise RuntimeError("pull did not complete")
      torch.cuda.synchronize(device)
      if it >= warmup:
        ms.append(e0.elapsed_time(e1))
        host_ms.append((h1 - h0) * 1e3)
    else:
      t0 = time.time()
      while f"pull-{it}" not in mgr.poll_stats()[0]:
        if time.time() - t0 > 30:
          raise RuntimeError("pull was not consumed")
        time.sleep(0.001)
    dist.barrier()
  t = torch.tensor([statistics.median(ms) if ms else 0.0,
                    statistics.median(host_ms) if host_ms else 0.0],
                   dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  step_ms, start_read_ms = float(t[0].item()), float(t[1].item())
  moved = B * g.block_bytes
  mgr.close()
  # The last read's destination blocks hold the producer's source blocks,
  # the producer's pool regenerated here from its seed (50 + its rank).
  exact = True
  if not is_src:
    prod = torch.empty_like(full)
    prod.normal_(generator=torch.Generator(device=device).manual_seed(50 + rank - half))
    si = torch.tensor(src_ids, dtype=torch.int64, device=device)
    di = torch.tensor(dst_ids, dtype=torch.int64, device=device)
    exact = bool(torch.equal(full[:, :, di].view(torch.int16), prod[:, :, si].view(torch.int16)))
    del prod
  ok = torch.tensor([1 if exact else 0], dtype=torch.int32, device=device)
  dist.all_reduce(ok, op=dist.ReduceOp.MIN)
  del full, storages
  return {"config": f"{B} C1 blocks (2 MiB each) per pair, {half} pairs (GPU i -> i+{half}), "
                    "register_read / start_read / poll_stats over CUDA IPC",
          "bytes_per_pair": moved, "ms": round(step_ms, 3),
          "exact": bool(int(ok.item())),
          "exact_how": "the last read's 512 destination blocks equal the producer's source "
                       "blocks, its pool regenerated from its seed",
          "start_read_host_ms": round(start_read_ms, 3),
          "nvlink_gbs_per_pair": round(moved / (step_ms * 1e-3) / 1e9, 1) if step_ms else None,
          "frac_of_nvlink_770": round(moved / (step_ms * 1e-3) / 1e9 / 770.0, 3)
          if step_ms else None}


def c3_expected_pages(torch, device, src_rank, n_st, n_seqs, sbps, dbps, H, HB, st_tab, dt_tab):
  """The consumer's pages after the hand-off, recomputed with torch (no
  product kernel or planner): the producer's pages regenerated from its seed
  (40 + its rank), each sequence's 16-token head-major source pages gathered
  in order by its source page table, laid out token-major ([token][head]),
  four to a 64-token page, and scattered by the destination page table."""
  E = HB // 2  # bf16 elements of one head vector
  src = torch.empty((n_st, n_seqs * sbps, 16 * H * E), dtype=torch.bfloat16, device=device)
  src.normal_(generator=torch.Generator(device=device).manual_seed(40 + src_rank))
  sidx = torch.from_numpy(st_tab.reshape(-1).astype(np.int64)).to(device)
  didx = torch.from_numpy(dt_tab.reshape(-1).astype(np.int64)).to(device)
  g = src[:, sidx].view(n_st, n_seqs, sbps, H, 16, E)       # [st][seq][page][head][tok]
  g = g.permute(0, 1, 2, 4, 3, 5).reshape(n_st, n_seqs * dbps, 64 * H * E)
  del src
  out = torch.zeros((n_st, n_seqs * dbps, 64 * H * E), dtype=torch.bfloat16, device=device)
  out[:, didx] = g
  return out


def run_handoff(torch, dist, rank, world, device, steps, warmup):
  """C3: 8 sequences x 32768 tokens of Llama-3-8B KV (2 heads per GPU) move
  from rank i (16-token head-major pages) to rank i+half (64-token
  token-major pages): one relayout kernel per producer storing into the
  consumer's pages (CUDA IPC mapping, NVLink P2P stores)."""
  import numpy as np
  from tpu_sync_b200 import ops
  from tpu_sync_b200.weight_synchronizer import (close_imports, export_destinations,
                                                 import_destinations)
  half = world // 2
  is_src = rank < half
  n_st, n_seqs, T, H, HB = 64, 8, 32768, 2, 256
  sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
  dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
  sbps, dbps = T // 16, T // 64
  rng = np.random.default_rng(30 + (rank % half))
  st_tab = rng.permutation(n_seqs * sbps).reshape(n_seqs, sbps).astype(np.int32)
  dt_tab = rng.permutation(n_seqs * dbps).reshape(n_seqs, dbps).astype(np.int32)
  sbb, dbb = 16 * H * HB, 64 * H * HB
  if is_src:
    pages = torch.empty((n_st, n_seqs * sbps, sbb // 2), dtype=torch.bfloat16, device=device)
    pages.normal_(generator=torch.Generator(device=device).manual_seed(40 + rank))
    desc = None
  else:
    pages = torch.zeros((n_st, n_seqs * dbps, dbb // 2), dtype=torch.bfloat16, device=device)
    desc = export_destinations({0: pages})
  descs = [None] * world
  dist.all_gather_object(descs, desc)
  ms = 0.0
  if is_src:
    peer = import_destinations(descs[rank + half], kernel_device=device.index)[0]
    srcs = [pages[s] for s in range(n_st)]
    storage_bytes = n_seqs * dbps * dbb
    dsts = [peer.data_ptr() + s * storage_bytes for s in range(n_st)]
    st_t, dt_t = torch.from_numpy(st_tab), torch.from_numpy(dt_tab)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    for _ in range(warmup):
      ops.kv_relayout(srcs, dsts, sg, dg, st_t, dt_t, T, device=device,
                      dst_pages=n_seqs * dbps, err=err)
    torch.cuda.synchronize(device)
    if int(err.item()) != 0:
      raise RuntimeError("kv_relayout: a page table entry is out of range")
  dist.barrier()
  if is_src:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
      ops.kv_relayout(srcs, dsts, sg, dg, st_t, dt_t, T, device=device,
                      dst_pages=n_seqs * dbps, err=err)
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
  dist.barrier()
  t = torch.tensor([ms], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  ms = float(t.item())
  moved = n_st * n_seqs * T * H * HB
  # After each variant the consumer compares every page with the pages
  # recomputed from their definition, then clears them for the next one.
  expected = (c3_expected_pages(torch, device, rank - half, n_st, n_seqs, sbps, dbps, H, HB,
                                st_tab, dt_tab) if not is_src else None)
  exact = {}

  def check(label):
    if not is_src:
      torch.cuda.synchronize(device)
      exact[label] = bool(torch.equal(pages.view(torch.int16), expected.view(torch.int16)))
      pages.zero_()
      torch.cuda.synchronize(device)
    dist.barrier()

  check("push")

  # The same relayout pulled by the consumer (the reference's StartRead
  # direction): the decode GPU's kernel loads the prefill GPU's pages over
  # NVLink and stores into its own pages.
  src_desc = export_destinations({0: pages}) if is_src else None
  sdescs = [None] * world
  dist.all_gather_object(sdescs, src_desc)
  pull_ms = 0.0
  if not is_src:
    peer_src = import_destinations(sdescs[rank - half], kernel_device=device.index)[0]
    src_storage_bytes = n_seqs * sbps * sbb
    psrcs = [peer_src.data_ptr() + s * src_storage_bytes for s in range(n_st)]
    pdsts = [pages[s] for s in range(n_st)]
    pst_t, pdt_t = torch.from_numpy(st_tab), torch.from_numpy(dt_tab)
    perr = torch.zeros(1, dtype=torch.int32, device=device)
    for _ in range(warmup):
      ops.kv_relayout(psrcs, pdsts, sg, dg, pst_t, pdt_t, T, device=device,
                      src_pages=n_seqs * sbps, err=perr)
    torch.cuda.synchronize(device)
    if int(perr.item()) != 0:
      raise RuntimeError("kv_relayout (pull): a page table entry is out of range")
  dist.barrier()
  if not is_src:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
      ops.kv_relayout(psrcs, pdsts, sg, dg, pst_t, pdt_t, T, device=device,
                      src_pages=n_seqs * sbps, err=perr)
    e1.record()
    torch.cuda.synchronize(device)
    pull_ms = e0.elapsed_time(e1) / steps
  dist.barrier()
  t = torch.tensor([pull_ms], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  pull_ms = float(t.item())
  check("pull")
  if not is_src:
    peer_src = psrcs = None
    close_imports(device.index)
  dist.barrier()

  # The same hand-off through the pool reshard planner: pools + span
  # declarations -> plan entries -> one program launch per source GPU.
  plan_ms = prog_ms = 0.0
  n_tasks = 0
  if is_src:
    from tpu_sync_b200 import pool_reshard, workloads
    t0 = time.perf_counter()
    src_pools, dst_pools, dst_ids, reg = workloads.handoff_pool_plan_inputs(
        n_st, st_tab, dt_tab, H, HB)
    plan = pool_reshard.build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids,
                                                [(0, reg)])
    plan_ms = (time.perf_counter() - t0) * 1e3

    class _Peer:  # one destination storage inside the imported mapping
      def __init__(self, ptr, dev, nbytes):
        self._p, self.device, self.dtype, self.shape = ptr, dev, torch.uint8, (nbytes,)

      def data_ptr(self):
        return self._p

    peer = import_destinations(descs[rank + half], kernel_device=device.index)[0]
    dst_st = [_Peer(peer.data_ptr() + s * storage_bytes, peer.device, storage_bytes)
              for s in range(n_st)]
    prog = pool_reshard.PoolReshardProgram(plan, 0, srcs, dst_st)
    n_tasks = prog.n_tasks
    for _ in range(warmup):
      prog.launch()
    torch.cuda.synchronize(device)
  dist.barrier()
  if is_src:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
      prog.launch()
    e1.record()
    torch.cuda.synchronize(device)
    prog_ms = e0.elapsed_time(e1) / steps
  dist.barrier()
  t = torch.tensor([prog_ms, plan_ms], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  prog_ms, plan_ms = float(t[0].item()), float(t[1].item())
  check("pool_plan")
  if is_src:
    prog.close()
    plan.close()
    peer = None
    close_imports(device.index)
  dist.barrier()

  # The planner's program pulled: launched on the consumer, its tasks load
  # the producer's pages over NVLink.
  pull_prog_ms = 0.0
  if not is_src:
    from tpu_sync_b200 import pool_reshard, workloads
    src_pools, dst_pools, dst_ids, reg = workloads.handoff_pool_plan_inputs(
        n_st, st_tab, dt_tab, H, HB)
    plan = pool_reshard.build_pool_reshard_plan([src_pools], dst_pools, ["kv"], dst_ids,
                                                [(0, reg)])

    class _Remote:  # one source storage inside the imported mapping
      def __init__(self, ptr, dev, nbytes):
        self._p, self.device, self.dtype, self.shape = ptr, dev, torch.uint8, (nbytes,)

      def data_ptr(self):
        return self._p

    peer_src = import_destinations(sdescs[rank - half], kernel_device=device.index)[0]
    src_storage_bytes = n_seqs * sbps * sbb
    src_st = [_Remote(peer_src.data_ptr() + s * src_storage_bytes, peer_src.device,
                      src_storage_bytes) for s in range(n_st)]
    prog = pool_reshard.PoolReshardProgram(plan, 0, src_st, [pages[s] for s in range(n_st)],
                                           device=device.index)
    for _ in range(warmup):
      prog.launch()
    torch.cuda.synchronize(device)
  dist.barrier()
  if not is_src:
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
      prog.launch()
    e1.record()
    torch.cuda.synchronize(device)
    pull_prog_ms = e0.elapsed_time(e1) / steps
  dist.barrier()
  t = torch.tensor([pull_prog_ms], dtype=torch.float64, device=device)
  dist.all_reduce(t, op=dist.ReduceOp.MAX)
  pull_prog_ms = float(t.item())
  check("pool_plan_pull")
  ok = torch.tensor([1 if all(exact.values()) else 0], dtype=torch.int32, device=device)
  dist.all_reduce(ok, op=dist.ReduceOp.MIN)
  expected = None
  torch.cuda.empty_cache()
  if not is_src:
    prog.close()
    plan.close()
    peer_src = src_st = None
    close_imports(device.index)
  dist.barrier()
  def rate(t_ms):
    return {"ms": round(t_ms, 3),
            "nvlink_gbs_per_pair": round(moved / (t_ms * 1e-3) / 1e9, 1) if t_ms else None,
            "frac_of_nvlink_770": round(moved / (t_ms * 1e-3) / 1e9 / 770.0, 3) if t_ms else None}

  return {"config": "C3 8 seqs x 32768 tok, 2 KV heads/GPU, 16-tok head-major -> 64-tok "
                    f"token-major, {half} pairs (GPU i -> i+{half})",
          "bytes_per_pair": moved,
          "exact": bool(int(ok.item())),
          "exact_how": ("after each of the four variants every consumer's 8 GiB of pages "
                        "equal the producer's regenerated pages relaid out by torch indexing "
                        "(page tables applied by definition)"),
          "how": ("relayout kernel on the consumer (the reference's pull direction): loads "
                  "the producer's pages over NVLink (CUDA IPC), stores its own pages"),
          **rate(pull_ms),
          "push": dict(how="the same kernel on the producer, storing into the consumer's "
                           "pages over NVLink", **rate(ms)),
          "pool_plan": {"how": "pool reshard planner (span declarations -> entries) + one "
                               "program launch per source GPU",
                        "plan_ms_cpu": round(plan_ms, 1), "tasks": n_tasks,
                        "ms": round(prog_ms, 3),
                        "nvlink_gbs_per_pair": round(moved / (prog_ms * 1e-3) / 1e9, 1)
                        if prog_ms else None,
                        "frac_of_nvlink_770": round(moved / (prog_ms * 1e-3) / 1e9 / 770.0, 3)
                        if prog_ms else None,
                        "pull": dict(how="the same program launched on the consumer",
                                     **rate(pull_prog_ms))}}


def run_c2_fp8(torch, rank, device, steps, warmup, max_over_ranks, cpu_seconds=0.0):
  """C2: Llama-3-70B TP8 KV shard (80 layers x K/V, 64-token blocks of 1 head
  x 128 bf16 = 16 KiB per storage block) on an fp8 host tier: per step 256
  random blocks (seed 20+rank) offloaded (fused bf16 -> e4m3 + per-block
  scale) while the previous step's 256 are reloaded (dequantised) into other
  blocks, both directions in flight.  GB/s counts the bf16 bytes moved."""
  from tpu_sync_b200 import KVCacheManager, workloads
  g = workloads.C2
  B, nblk, host_blocks = workloads.C2_BATCH, 4096, 1024
  full = torch.empty((g.layers, g.kv, nblk, g.block_tokens, g.heads, g.head_dim),
                     dtype=torch.bfloat16, device=device)
  gen = torch.Generator(device=device).manual_seed(20 + rank)
  for l in range(g.layers):
    full[l].normal_(generator=gen)
  storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]
  mgr = make_manager(KVCacheManager, [[t] for t in storages], host_blocks_to_allocate=host_blocks,
                     fp8=True)
  rng = np.random.default_rng(20 + rank)
  n = warmup + steps + 1
  out_ids = [rng.choice(nblk // 2, B, replace=False).astype(np.int64) for _ in range(n)]
  in_ids = [nblk // 2 + rng.choice(nblk // 2, B, replace=False).astype(np.int64) for _ in range(n)]
  host = [((np.arange(B) + i * B) % host_blocks).astype(np.int64) for i in range(n)]
  stream = torch.cuda.Stream(device)

  def step(i):
    f1 = mgr.d2h(out_ids[i + 1], host[i + 1], stream=stream)
    f2 = mgr.h2d(host[i], in_ids[i], stream=stream)
    f1.stream_wait(stream)
    f2.stream_wait(stream)
    return f1, f2

  mgr.d2h(out_ids[0], host[0], stream=stream).Await()
  for i in range(warmup):
    for f in step(i):
      f.Await()
  torch.cuda.synchronize(device)
  mgr.set_profiling(True)
  mgr.kernel_stats("extract")
  mgr.kernel_stats("insert")
  e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  e0.record(stream)
  futs = []
  for i in range(warmup, warmup + steps):
    futs.extend(step(i))
  e1.record(stream)
  torch.cuda.synchronize(device)
  for f in futs:
    f.Await()
  ms = max_over_ranks(e0.elapsed_time(e1)) / steps
  ext, ins = mgr.kernel_stats("extract"), mgr.kernel_stats("insert")
  mgr.close()
  # The last step reloaded into in_ids[last] what the step before offloaded
  # from out_ids[last]: the fp8 round trip of those blocks, recomputed here
  # with torch from its definition (per (layer, K/V, block) scale =
  # amax / 448, q = e4m3 RN of x / scale, x' = bf16 RN of q * scale).
  last = warmup + steps - 1
  sid = torch.from_numpy(out_ids[last]).to(device)
  did = torch.from_numpy(in_ids[last]).to(device)
  x = full[:, :, sid].float()
  amax = x.abs().amax(dim=(3, 4, 5), keepdim=True)
  # a tensor divisor keeps torch's true (round-to-nearest) division on the
  # GPU; a Python-scalar divisor would be applied as a reciprocal multiply
  scale = torch.where(amax == 0, torch.ones_like(amax), amax / torch.full_like(amax, 448.0))
  want = ((x / scale).to(torch.float8_e4m3fn).float() * scale).to(torch.bfloat16)
  exact = bool(torch.equal(full[:, :, did].view(torch.int16), want.view(torch.int16)))
  del x, amax, scale, want
  bf16_bytes = 2 * B * g.block_bytes
  wire = 2 * B * mgr.host_block_pitch

  def kgbs(st):
    return round(st["bytes"] / (st["ms"] * 1e-3) / 1e9, 1) if st["ms"] > 0 else None

  cpu = cpu_c2_fp8(cpu_seconds) if cpu_seconds > 0 else None
  return {"config": "C2 Llama-3-70B TP8 KV (80 layers x K/V, 64 tok x 1 head x 128 bf16 "
                    f"blocks), {nblk}-block pool, fp8 e4m3 host tier of {host_blocks} blocks, "
                    f"{B} offloads + {B} reloads per step",
          "cpu_baseline": cpu,
          "ms_per_step": round(ms, 3),
          "bf16_gbs": round(bf16_bytes / (ms * 1e-3) / 1e9, 2),
          "pcie_gbs": round(wire / (ms * 1e-3) / 1e9, 2),
          "extract_fp8_kernel_gbs": kgbs(ext), "insert_fp8_kernel_gbs": kgbs(ins),
          "kernel_launches": ext["launches"] + ins["launches"],
          "exact": exact,
          "exact_how": ("the last step's 256 reloaded blocks (all 160 storages) equal the fp8 "
                        "round trip of the blocks offloaded before them, recomputed with torch")}


def noalloc_offload_figure(torch, device, storages, table, id_sets, n, pitch):
  """D2H GB/s of ts_kv_offload_noalloc (no device allocation, 64 MiB static
  staging) at the C1 geometry: n random pool blocks into n consecutive host
  blocks of a pinned buffer, CUDA events on the call's stream, median of 5."""
  import ctypes
  from tpu_sync_b200 import _native
  arr = (_native.BlockStorage * len(storages))()
  for i, t in enumerate(storages):
    nbytes = t.numel() * t.element_size()
    arr[i].dev_ptr, arr[i].block_bytes = t.data_ptr(), nbytes // t.shape[0]
    arr[i].dev_bytes, arr[i].stage_off = nbytes, table.stage_offs[i]
  host = torch.empty((n, pitch), dtype=torch.uint8, pin_memory=True)
  stream = torch.cuda.Stream(device)
  dst = _native.i64_array(np.arange(n))
  ms = []
  for i in range(8):
    src = _native.i64_array(id_sets[i % len(id_sets)])
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    _native.check(_native.lib().ts_kv_offload_noalloc(
        device.index, arr, len(storages), _native.i64_ptr(src), _native.i64_ptr(dst), n,
        ctypes.c_void_p(host.data_ptr()), pitch, n, ctypes.c_void_p(stream.cuda_stream)))
    b.record(stream)
    stream.synchronize()
    if i >= 3:
      ms.append(a.elapsed_time(b))
  del host
  med = statistics.median(ms)
  return {"gbs": round(n * pitch / (med * 1e-3) / 1e9, 2), "ms": round(med, 3), "blocks": n,
          "how": "ts_kv_offload_noalloc, 2 MiB C1 blocks from the HBM pool to pinned host "
                 "memory through the 64 MiB static staging (32 blocks per chunk)"}


def run_ours(args):
  import torch
  import torch.distributed as dist

  from tpu_sync_b200 import KVCacheManager, ops, workloads

  world = int(os.environ.get("WORLD_SIZE", "1"))
  rank = int(os.environ.get("RANK", "0"))
  local = int(os.environ.get("LOCAL_RANK", "0"))
  torch.cuda.set_device(local)
  device = torch.device("cuda", local)
  if world > 1:
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                            device_id=device)

  def barrier():
    if world > 1:
      dist.barrier()

  def max_over_ranks(x: float) -> float:
    if world == 1:
      return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())

  g = workloads.C1
  if (g.storages, g.storage_block_bytes) != (C1_STORAGES, C1_STORAGE_BLOCK_BYTES):
    raise RuntimeError("workloads.C1 does not match the C1 geometry stated in bench.py")
  B = args.batch
  pool_blocks = args.pool_blocks
  # Pool: [layers, K/V, blocks, 16, 8, 128] bf16, N(0,1) generated on device.
  gen = torch.Generator(device=device).manual_seed(10 + rank)
  full = torch.empty((g.layers, g.kv, pool_blocks, g.block_tokens, g.heads, g.head_dim),
                     dtype=torch.bfloat16, device=device)
  for l in range(g.layers):
    full[l].normal_(generator=gen)
  storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]

  # Host tier: as large as requested, bounded by this box's RAM share.
  pitch = g.block_bytes
  host_blocks = c1_host_blocks(args, world)
  mgr = make_manager(KVCacheManager, [[t] for t in storages], host_blocks_to_allocate=host_blocks,
                     mode=args.mode, copy_streams=args.copy_streams,
                     chunk_blocks=args.chunk_blocks, max_ctas=args.max_ctas,
                     reload_staged_every=args.reload_staged_every,
                     sched=tuple(f for f in args.sched.split(",") if f))

  pcie = measure_pcie(torch, device, barrier=barrier if world > 1 else None)
  pcie["gpus_copying_at_once"] = world

  # Step plans from the C1 access trace: 100k accesses Zipf(1.1) over 200k
  # prefix ids, in batches of 512, run through the tier-2 store (LRU index +
  # host block allocator with the reference's policies) over this host tier.
  # A step moves what one access batch needs: its misses offloaded (saved)
  # and its hits reloaded, both directions in flight; steps follow the trace
  # from its middle (tier full, evicting).  Device ids: offloads read the
  # first half of the pool, reloads write the second half.
  plans, trace_stats = c1_plans(rank, host_blocks, pool_blocks, B, args.warmup + args.steps)
  # The CPU reference arm takes its plans from the reference's own LRU and
  # allocator; the two must agree for its number to be comparable.
  plans_match = None
  if rank == 0:
    try:
      ref_plans, _ = c1_plans(rank, host_blocks, pool_blocks, B, args.warmup + args.steps,
                              source="reference")
      plans_match = all(all(np.array_equal(a, b) for a, b in zip(p, q))
                        for p, q in zip(plans, ref_plans))
    except (OSError, RuntimeError):
      plans_match = None
  plan_bytes = [(len(p[0]) + len(p[2])) * pitch for p in plans]
  bench_stream = torch.cuda.Stream(device)

  def step(plan, stream):
    f1 = mgr.d2h(plan[0], plan[1], stream=stream)
    f2 = mgr.h2d(plan[2], plan[3], stream=stream)
    f1.stream_wait(stream)
    f2.stream_wait(stream)
    return f1, f2

  # Untimed: the host blocks the steps reload before offloading there get
  # known bytes (the trace saved them before the steps that run), so the
  # end-of-run check can name what every reloaded block must hold.
  executed = list(range(args.warmup + args.steps)) + list(range(args.warmup,
                                                                args.warmup + args.steps))
  seed = c1_seed_host_blocks(plans, executed, pool_blocks // 2)
  if seed:
    seed_h = sorted(seed)
    mgr.d2h([seed[h] for h in seed_h], seed_h).Await()

  # ---- device-timed steps (value) ----
  for i in range(args.warmup):
    for f in step(plans[i], bench_stream):
      f.Await()
  torch.cuda.synchronize(device)
  clocks = ClockSampler(device.index)
  clocks.start()  # live before the barrier, so every rank's region is sampled
  barrier()
  torch.cuda.synchronize(device)
  mgr.set_profiling(True)
  mgr.kernel_stats("extract")
  mgr.kernel_stats("insert")
  clocks.begin()
  e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
  e0.record(bench_stream)
  futs = []
  for i in range(args.warmup, args.warmup + args.steps):
    futs.extend(step(plans[i], bench_stream))
  e1.record(bench_stream)
  torch.cuda.synchronize(device)
  clocks.end()
  clock_info = clocks.stop()
  barrier()
  for f in futs:
    f.Await()
  dev_ms = e0.elapsed_time(e1)
  mgr.set_profiling(False)
  ext = mgr.kernel_stats("extract")
  ins = mgr.kernel_stats("insert")
  max_ms = max_over_ranks(dev_ms)
  ms_per_step = max_ms / args.steps
  timed_bytes = sum(plan_bytes[args.warmup:])
  timed_d2h = sum(len(p[0]) for p in plans[args.warmup:]) * pitch
  timed_h2d = sum(len(p[2]) for p in plans[args.warmup:]) * pitch
  value = world * timed_bytes / (max_ms * 1e-3) / 1e9

  # ---- standalone extract of a whole batch in one launch (HBM GB/s) ----
  table = ops.StorageTable(storages)
  staging = table.new_staging(B)
  one_rng = np.random.default_rng(7)
  one_ids = [one_rng.choice(pool_blocks, B, replace=False).astype(np.int64) for _ in range(5)]
  big_ids = torch.from_numpy(one_ids[0]).to(device)
  for _ in range(3):
    ops.kv_extract(table, big_ids, staging)
  torch.cuda.synchronize(device)
  xs = []
  for i in range(5):
    ids_i = torch.from_numpy(one_ids[i]).to(device)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    ops.kv_extract(table, ids_i, staging)
    b.record()
    torch.cuda.synchronize(device)
    xs.append(a.elapsed_time(b))
  extract_one_launch_gbs = 2 * B * pitch / (statistics.median(xs) * 1e-3) / 1e9
  del staging
  noalloc = noalloc_offload_figure(torch, device, storages, table, one_ids, B, pitch)

  # ---- end to end through the public Python API ----
  barrier()
  lists = [[p[0].tolist(), p[1].tolist(), p[2].tolist(), p[3].tolist()] for p in plans]
  torch.cuda.synchronize(device)
  t0 = time.perf_counter()
  for i in range(args.warmup, args.warmup + args.steps):
    a = mgr.d2h(lists[i][0], lists[i][1])
    b = mgr.h2d(lists[i][2], lists[i][3])
    a.Await()
    b.Await()
  wall = time.perf_counter() - t0
  wall = max_over_ranks(wall)
  e2e_value = world * timed_bytes / wall / 1e9

  # ---- every reloaded block checked against its definition ----
  expected = c1_expected_sources(plans, executed, seed)
  c1_bad = c1_blocks_differ(torch, full, expected, device)
  c1_exact = torch.tensor([0 if c1_bad else 1], dtype=torch.int32, device=device)
  if world > 1:
    dist.all_reduce(c1_exact, op=dist.ReduceOp.MIN)
  c1_exact = bool(int(c1_exact.item()))

  # ---- roofline of the dominant kernel (by live device time) ----
  pk = peaks()
  hbm_peak = pk.get("hbm_gbs")
  peak_src = "measured (MEASURED_PEAKS.json hbm_gbs)"
  if not hbm_peak:
    hbm_peak, peak_src = 6650.0, "fallback"
  kern = {}
  direct = {"extract": args.mode in ("direct_d2h", "direct"),
            "insert": args.mode in ("direct_h2d", "direct")}
  bulk = "bulk_copy" in args.sched.split(",")
  for name, st in (("extract", ext), ("insert", ins)):
    # the manager runs HBM -> HBM chunks on the bulk-copy kernel when asked
    kname = "block_copy_bulk_kernel" if bulk and not direct[name] else "block_copy_vec_kernel"
    kern[name] = {
        "kernel": f"{kname}<{'true' if name == 'extract' else 'false'}> ({name})",
        "path": (("HBM pool -> mapped host tier over PCIe" if name == "extract" else
                  "mapped host tier over PCIe -> HBM pool") if direct[name] else
                 ("HBM pool -> HBM staging" if name == "extract" else
                  "HBM staging -> HBM pool")),
        "launches": st["launches"], "total_ms": round(st["ms"], 3),
        "bytes_per_launch": int(st["bytes"] / max(st["launches"], 1)),
        "avg_launch_us": round(st["ms"] * 1e3 / max(st["launches"], 1), 2),
        "achieved_gbs": round(st["bytes"] / (st["ms"] * 1e-3) / 1e9, 1) if st["ms"] > 0 else 0.0}
    if direct[name] and st["ms"] > 0:
      # half of the kernel's bytes (the host side) cross the link
      kern[name]["pcie_gbs"] = round(st["bytes"] / 2 / (st["ms"] * 1e-3) / 1e9, 2)
  tot_ms = sum(k["total_ms"] for k in kern.values()) or 1.0
  for k in kern.values():
    k["share"] = round(k["total_ms"] / tot_ms, 3)
  dom = max(kern, key=lambda n: kern[n]["total_ms"])
  # DRAM traffic per block from ncu captures of the same kernels on the
  # small kernel case (profiles/*_kernel_c1_256blocks.md), scaled to this
  # run's launches by the blocks they move.
  traffic_per_block = {"extract": (BULK_EXTRACT_TRAFFIC_PER_BLOCK if bulk
                                   else VEC_EXTRACT_TRAFFIC_PER_BLOCK),
                       "insert": (INSERT_DIRECT_TRAFFIC_PER_BLOCK if direct["insert"]
                                  else INSERT_TRAFFIC_PER_BLOCK)}
  if direct["extract"]:
    traffic_per_block["extract"] = None
  blocks_per_launch = kern[dom]["bytes_per_launch"] / (2 * pitch)
  tpb = traffic_per_block.get(dom)
  if direct[dom]:
    # a kernel that pulls (pushes) the host tier over PCIe is bound by the
    # link, not by HBM: its roofline is the pinned-memcpy peak of that
    # direction measured in this run
    pdir = "h2d" if dom == "insert" else "d2h"
    roof = {"bound": "pcie", "kernel": kern[dom]["kernel"],
            "achieved": kern[dom]["pcie_gbs"], "peak": pcie.get(pdir), "unit": "GB/s",
            "frac": round(kern[dom]["pcie_gbs"] / pcie[pdir], 3) if pcie.get(pdir) else None,
            "peak_source": f"measured in this run: pinned 1 GiB cudaMemcpyAsync {pdir.upper()}",
            "achieved_def": "host-tier bytes the kernel moved over PCIe per launch / its "
                            "CUDA-event duration (the HBM side moves the same bytes)"}
  else:
    roof = {"bound": "hbm", "kernel": kern[dom]["kernel"],
            "achieved": kern[dom]["achieved_gbs"], "peak": hbm_peak, "unit": "GB/s",
            "frac": round(kern[dom]["achieved_gbs"] / hbm_peak, 3), "peak_source": peak_src}
  roof.update({
      "traffic": int(tpb * blocks_per_launch) if tpb else None,
      "traffic_source": "ncu DRAM read+write bytes of the small kernel case, scaled per block"
      if tpb else None,
      "note": ("live: launched in 64-block chunks concurrently with the other direction's "
               "kernel and the DMAs"),
      "kernels": kern})
  hbm_side = [n for n in kern if not direct[n] and kern[n]["launches"]]
  if direct[dom] and hbm_side:
    n = max(hbm_side, key=lambda k: kern[k]["total_ms"])
    roof["hbm_kernel"] = {"kernel": kern[n]["kernel"], "bound": "hbm",
                          "achieved": kern[n]["achieved_gbs"], "peak": hbm_peak,
                          "frac": round(kern[n]["achieved_gbs"] / hbm_peak, 3),
                          "peak_source": peak_src,
                          "note": ("live, each launch timed from its start event: the "
                                   "gather waits for SM slots that the reload's CTAs hold "
                                   "while they wait on PCIe; the extract_hbm_gbs_one_launch "
                                   "figure is a 512-block extract alone")}
  # ---- CPU baseline (rank 0, N=1) ----
  cpu = None
  if rank == 0 and world == 1 and not args.no_cpu_baseline:
    cpu = cpu_offload_reload(plans, args.cpu_sample_s)

  d2h_gbs = timed_d2h / (max_ms * 1e-3) / 1e9
  h2d_gbs = timed_h2d / (max_ms * 1e-3) / 1e9
  line = None
  if rank == 0:
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic N(0,1) bf16 KV pool generated on device (seed 10+rank)",
        "config": dict(c1_config(args, host_blocks, plans, trace_stats, world),
                       plans_match_reference_store=plans_match),
        "transfer": {"mode": args.mode, "copy_streams": args.copy_streams,
                     "max_ctas": args.max_ctas or None,
                     "reload_staged_every": args.reload_staged_every or None,
                     "sched": [f for f in args.sched.split(",") if f]},
        "per_gpu_gbs": round(value / world, 3),
        "pcie": {"offload_d2h_gbs": round(d2h_gbs, 2), "reload_h2d_gbs": round(h2d_gbs, 2),
                 "measured_peak": pcie, "spec_gbs_per_dir": PCIE_SPEC_GBS,
                 "frac_of_measured_duplex": round((d2h_gbs + h2d_gbs) / pcie["duplex"], 3)
                 if pcie.get("duplex") else None,
                 "reload_frac_of_measured_h2d": round(h2d_gbs / pcie["h2d"], 3)
                 if pcie.get("h2d") else None,
                 "frac_of_spec_busier_dir": round(max(d2h_gbs, h2d_gbs) / PCIE_SPEC_GBS, 3)},
        "roofline": roof,
        "extract_hbm_gbs_one_launch": round(extract_one_launch_gbs, 1),
        "noalloc_offload": noalloc,
        "exact": c1_exact,
        "exact_how": (f"after the warm-up, timed and end-to-end steps, each of the "
                      f"{len(expected)} pool blocks the reloads wrote equals, bitwise, the "
                      f"pool block whose bytes the host block it last read held (offloaded "
                      f"by an earlier step, or before the warm-up for the "
                      f"{len(seed)} host blocks the trace had saved earlier); torch on "
                      f"the device, a step's offloads before its reloads, the last copy "
                      f"to a block winning"),
        "e2e": {"value": round(e2e_value, 3), "unit": "GB/s",
                "h2d_bytes_per_step": int(timed_h2d / args.steps),
                "d2h_bytes_per_step": int(timed_d2h / args.steps),
                "how": "KVCacheManager.d2h/h2d from Python lists, Await() per step, wall clock"},
        "gpu_launches": ext["launches"] + ins["launches"],
        "clocks": clock_info,
        "cpu_baseline": None if cpu is None else {
            "value": cpu["value"], "unit": "GB/s", "cores": cpu["cores"], "kind": "port",
            "sample": cpu["sample"], "cpu": cpu["cpu"]},
    }
  host_after_c1 = host_memory_state()
  mgr.close()
  del mgr, full, storages, table
  torch.cuda.empty_cache()
  if hasattr(torch._C, "_host_emptyCache"):  # torch's cached pinned buffers
    torch._C._host_emptyCache()
  if rank == 0:
    line["host_memory"] = {"during_c1": host_after_c1, "after_c1": host_memory_state()}
  c2 = run_c2_fp8(torch, rank, device, 5, 3, max_over_ranks,
                  cpu_seconds=5.0 if (rank == 0 and world == 1 and not args.no_cpu_baseline)
                  else 0.0)
  torch.cuda.empty_cache()
  if world > 1:  # every rank's check must hold
    ok = torch.tensor([1 if c2["exact"] else 0], dtype=torch.int32, device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    c2["exact"] = bool(int(ok.item()))
  c2["gpus_concurrent"] = world
  if rank == 0:
    line["c2_fp8"] = c2
  exchange = {}
  if world >= 2 and world % 2 == 0 and not args.no_exchange:
    exchange["weight_sync"] = run_weight_sync(torch, dist, rank, world, device, 3, 2)
    torch.cuda.empty_cache()
    exchange["handoff"] = run_handoff(torch, dist, rank, world, device, 3, 2)
    torch.cuda.empty_cache()
    exchange["pull"] = run_pull(torch, dist, rank, world, device, 5, 2)
    torch.cuda.empty_cache()
    if rank == 0 and not args.no_cpu_baseline:
      # the same exchanges on the host cores (bounded samples; the other
      # ranks wait at the closing barrier)
      from tpu_sync_b200 import reshard_plan as rp
      half = world // 2
      specs = workloads.weight_sync_specs(half, half)
      exchange["weight_sync"]["cpu_baseline"] = cpu_c4_reshard(rp.build_plan(specs), specs, 5.0)
      exchange["handoff"]["cpu_baseline"] = cpu_c3_relayout(5.0)
  if rank == 0:
    line.update(exchange)
    print(json.dumps(line), flush=True)
  if world > 1:
    dist.barrier()
    dist.destroy_process_group()


def run_kernel_case(args):
  """A few launches of one kernel on a case of a few GB (inputs > L2), for
  ncu captures: 1024-block C1 pool (2 GiB), 256 blocks per launch
  (512 MiB read + 512 MiB written), 4 launches."""
  import torch

  from tpu_sync_b200 import ops, workloads
  device = torch.device("cuda", 0)
  if args.kernel_case == "pool_reshard":
    # C3 hand-off plan for 16 of the 64 storages, destination on this GPU:
    # 2 GiB read + 2 GiB written per launch, 4 launches.
    from tpu_sync_b200 import pool_reshard
    n_st, n_seqs, T, H, HB = 16, 8, 32768, 2, 256
    rng = np.random.default_rng(30)
    st = rng.permutation(n_seqs * T // 16).reshape(n_seqs, -1).astype(np.int32)
    dt = rng.permutation(n_seqs * T // 64).reshape(n_seqs, -1).astype(np.int32)
    sp, dp, ids, reg = workloads.handoff_pool_plan_inputs(n_st, st, dt, H, HB)
    plan = pool_reshard.build_pool_reshard_plan([sp], dp, ["kv"], ids, [(0, reg)])
    src = [torch.randint(0, 256, (n_seqs * T // 16, 16 * H * HB), dtype=torch.uint8,
                         device=device) for _ in range(n_st)]
    dst = [torch.empty((n_seqs * T // 64, 64 * H * HB), dtype=torch.uint8, device=device)
           for _ in range(n_st)]
    prog = pool_reshard.PoolReshardProgram(plan, 0, src, dst)
    ms = []
    for i in range(4):
      a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      a.record()
      prog.launch()
      b.record()
      torch.cuda.synchronize()
      ms.append(a.elapsed_time(b))
    print(json.dumps({"kernel_case": "pool_reshard", "tasks": prog.n_tasks, "bytes": prog.bytes,
                      "ms": [round(x, 3) for x in ms],
                      "hbm_gbs": round(2 * prog.bytes / (min(ms) * 1e-3) / 1e9, 1)}))
    return
  if args.kernel_case == "relayout":
    # The C3 relayout kernel on the pool_reshard case's geometry (16 of the 64
    # storages, 8 x 32768 tokens, 16-token head-major -> 64-token token-major
    # pages), destination on this GPU: 2 GiB read + 2 GiB written, 4 launches.
    n_st, n_seqs, T, H, HB = 16, 8, 32768, 2, 256
    rng = np.random.default_rng(30)
    st = rng.permutation(n_seqs * T // 16).reshape(n_seqs, -1).astype(np.int32)
    dt = rng.permutation(n_seqs * T // 64).reshape(n_seqs, -1).astype(np.int32)
    src = [torch.randint(0, 256, (n_seqs * T // 16, 16 * H * HB), dtype=torch.uint8,
                         device=device) for _ in range(n_st)]
    dst = [torch.empty((n_seqs * T // 64, 64 * H * HB), dtype=torch.uint8, device=device)
           for _ in range(n_st)]
    sg = dict(block_tokens=16, heads=H, head_bytes=HB, head_major=1)
    dg = dict(block_tokens=64, heads=H, head_bytes=HB, head_major=0)
    st_t, dt_t = torch.from_numpy(st).to(device), torch.from_numpy(dt).to(device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    ms = []
    for _ in range(4):
      a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      a.record()
      ops.kv_relayout(src, dst, sg, dg, st_t, dt_t, T, device=device, err=err)
      b.record()
      torch.cuda.synchronize()
      ms.append(a.elapsed_time(b))
    assert int(err.item()) == 0
    moved = n_st * n_seqs * T * H * HB
    print(json.dumps({"kernel_case": "relayout", "bytes": moved,
                      "ms": [round(x, 3) for x in ms],
                      "hbm_gbs": round(2 * moved / (min(ms) * 1e-3) / 1e9, 1)}))
    return
  if args.kernel_case in ("reshard_cast", "reshard_copy"):
    # The weight-sync reshard kernel on trainer 0's chunks of the C4 4 -> 4
    # plan for decoder layers 0-7 of Llama-3-8B (a 436 M-parameter FSDP
    # slice of their 1.74 G), every destination on this GPU:
    # reshard_cast = fp32 -> bf16 (the push kernel's arithmetic and the
    # staged pull's sender cast), reshard_copy = bf16 -> bf16 (the staged
    # pull's receiver copy).  4 launches, CUDA events.
    from tpu_sync_b200 import reshard_plan as rp
    params = [p for p in workloads.llama3_8b_params()
              if p[0].startswith(tuple(f"layers.{i}." for i in range(8)))]
    specs = workloads.weight_sync_specs(4, 4, params)
    plan = rp.build_plan(specs)
    layout = workloads.weight_sync_layout(specs, 4, 4)
    cast = args.kernel_case == "reshard_cast"
    sdt = torch.float32 if cast else torch.bfloat16
    src = torch.empty(layout[0][0][1], dtype=sdt, device=device).normal_(0.0, 0.02)
    dsts = {d: torch.empty(layout[1][d][1], dtype=torch.bfloat16, device=device)
            for d in range(4)}
    chunks = workloads.weight_sync_chunks(plan, layout, 0, src.data_ptr(),
                                          {d: dsts[d].data_ptr() for d in range(4)},
                                          src_itemsize=src.element_size())
    prog = ops.ReshardProgram(chunks, sdt, torch.bfloat16, device)
    elems = sum(c[4] * c[7] for c in chunks)
    ms = []
    for _ in range(4):
      a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
      a.record()
      prog.launch()
      b.record()
      torch.cuda.synchronize()
      ms.append(a.elapsed_time(b))
    moved = elems * (src.element_size() + 2)
    print(json.dumps({"kernel_case": args.kernel_case, "chunks": len(chunks), "elements": elems,
                      "bytes": moved, "ms": [round(x, 3) for x in ms],
                      "hbm_gbs": round(moved / (min(ms) * 1e-3) / 1e9, 1)}))
    return
  if args.kernel_case == "insert_direct":
    # The insert kernel pulling 256 blocks (512 MiB) per launch from the
    # manager's mapped host tier into a 1024-block C1 pool (2 GiB), 4 launches.
    from tpu_sync_b200 import KVCacheManager
    g = workloads.C1
    full = torch.empty((g.layers, g.kv, 1024, g.block_tokens, g.heads, g.head_dim),
                       dtype=torch.bfloat16, device=device)
    full.normal_(generator=torch.Generator(device=device).manual_seed(1))
    storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]
    mgr = KVCacheManager([[t] for t in storages], host_blocks_to_allocate=256,
                         mode="direct_h2d", chunk_blocks=256)
    rng = np.random.default_rng(5)
    mgr.d2h(list(range(256)), rng.permutation(256).tolist()).Await()
    for i in range(4):
      mgr.h2d(rng.permutation(256).tolist(), rng.choice(1024, 256, replace=False).tolist()).Await()
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": args.kernel_case, "blocks_per_launch": 256,
                      "bytes_per_block": g.block_bytes}))
    mgr.close()
    return
  if args.kernel_case in ("manager_extract", "manager_insert"):
    # The manager's staged extract (HBM pool -> HBM staging) or insert kernel,
    # 256 random C1 blocks (512 MiB each way) per launch on a 1024-block pool,
    # with the kernel the --sched flags select (bulk_copy: the bulk-copy
    # kernel); CUDA-event device time of each launch from the manager.
    from tpu_sync_b200 import KVCacheManager
    g = workloads.C1
    full = torch.empty((g.layers, g.kv, 1024, g.block_tokens, g.heads, g.head_dim),
                       dtype=torch.bfloat16, device=device)
    full.normal_(generator=torch.Generator(device=device).manual_seed(1))
    storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]
    mgr = KVCacheManager([[t] for t in storages], host_blocks_to_allocate=256, mode="staged",
                         chunk_blocks=256, sched=tuple(f for f in args.sched.split(",") if f))
    rng = np.random.default_rng(5)
    extract = args.kernel_case == "manager_extract"
    if not extract:
      mgr.d2h(list(range(256)), list(range(256))).Await()
    for i in range(8):
      if i == 3:
        mgr.set_profiling(True)
        mgr.kernel_stats("extract")
        mgr.kernel_stats("insert")
      ids = rng.choice(1024, 256, replace=False).tolist()
      (mgr.d2h(ids, rng.permutation(256).tolist()) if extract
       else mgr.h2d(rng.permutation(256).tolist(), ids)).Await()
    st = mgr.kernel_stats("extract" if extract else "insert")
    mgr.close()
    print(json.dumps({"kernel_case": args.kernel_case, "sched": args.sched,
                      "launches": st["launches"],
                      "us_per_launch": round(st["ms"] * 1e3 / max(st["launches"], 1), 1),
                      "hbm_gbs": round(st["bytes"] / (st["ms"] * 1e-3) / 1e9, 1)}))
    return
  g = workloads.C1 if not args.kernel_case.endswith("fp8") else workloads.C2
  blocks = 1024 if g is workloads.C1 else 2048
  full = torch.empty((g.layers, g.kv, blocks, g.block_tokens, g.heads, g.head_dim),
                     dtype=torch.bfloat16, device=device)
  full.normal_(generator=torch.Generator(device=device).manual_seed(1))
  storages = [full[l, k] for l in range(g.layers) for k in range(g.kv)]
  table = ops.StorageTable(storages, fp8=args.kernel_case.endswith("fp8"))
  n = 256
  staging = table.new_staging(n)
  rng = np.random.default_rng(5)
  for i in range(4):
    ids = torch.from_numpy(rng.choice(blocks, n, replace=False).astype(np.int64)).to(device)
    if args.kernel_case.startswith("extract"):
      ops.kv_extract(table, ids, staging)
    else:
      if i == 0:  # fill the staging with real blocks (and fp8 scales)
        ops.kv_extract(table, ids, staging)
      ops.kv_insert(table, ids, staging)
  torch.cuda.synchronize()
  print(json.dumps({"kernel_case": args.kernel_case, "blocks_per_launch": n,
                    "bytes_per_block": table.pitch}))


def main():
  args = parse()
  if args.kernel_case:
    run_kernel_case(args)
    return
  if args.impl == "reference":
    run_reference(args)
  else:
    run_ours(args)


if __name__ == "__main__":
  main()

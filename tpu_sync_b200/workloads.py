"""Seeded synthetic workloads with the shapes of the benchmark configurations.

There is no dataset behind the hot path: KV caches and weights are random
values of the model shapes named in the configurations (Llama-3-8B / -70B
shaped KV pools, Llama-3-8B shaped weights).

  C0  paged KV [layers=4, K/V=2, blocks=1024, 16 tokens, 8 heads, 128] bf16,
      N(0,1) from seed 0; extract 128 distinct ids (seed 1), insert at 128
      other distinct ids (seed 2).
  C1  Llama-3-8B KV tier: 32 layers x K/V, 16-token blocks of 8 heads x 128
      bf16 (32 KiB per storage block, 2 MiB per block over all 64 storages),
      32768-block pool, 512-block offload/reload batches.
  C2  Llama-3-70B TP8 KV: 80 layers x K/V, 64-token blocks of 1 head x 128
      bf16 (16 KiB per storage block), 256 random blocks per rank
      (seed 20 + rank), stored as fp8 e4m3 + per-block scale.
  C3  hand-off: C1 geometry, 8 sequences x 32768 tokens, 2 heads per GPU,
      16-token head-major pages -> 64-token token-major pages.
  C4  Llama-3-8B weights fp32 N(0, 0.02) seed 3, FSDP dim-0 split over 4
      trainer ranks -> TP=4 bf16 sampler layout.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Tuple

import numpy as np
import torch


def bf16_normal(shape, seed: int, device="cpu", chunk_elems: int = 1 << 26) -> torch.Tensor:
  """N(0,1) fp32 from torch.Generator(seed), rounded to bf16 (RNE).

  Generated in chunks on the CPU generator so the values do not depend on
  the device; large pools are filled chunk by chunk straight into `device`.
  """
  g = torch.Generator().manual_seed(seed)
  out = torch.empty(shape, dtype=torch.bfloat16, device=device)
  flat = out.view(-1)
  n = flat.numel()
  for s in range(0, n, chunk_elems):
    e = min(n, s + chunk_elems)
    flat[s:e].copy_(torch.randn(e - s, generator=g, dtype=torch.float32).to(torch.bfloat16))
  return out


def distinct_ids(n: int, high: int, seed: int) -> np.ndarray:
  """n distinct block ids drawn uniformly from [0, high)."""
  return np.random.default_rng(seed).choice(high, size=n, replace=False).astype(np.int64)


@dataclass(frozen=True)
class KVGeometry:
  layers: int
  kv: int
  block_tokens: int
  heads: int
  head_dim: int
  itemsize: int = 2

  @property
  def storages(self) -> int:
    return self.layers * self.kv

  @property
  def storage_block_bytes(self) -> int:
    return self.block_tokens * self.heads * self.head_dim * self.itemsize

  @property
  def block_bytes(self) -> int:
    """Bytes of one block over all storages (one host block)."""
    return self.storages * self.storage_block_bytes


C0 = KVGeometry(layers=4, kv=2, block_tokens=16, heads=8, head_dim=128)
C0_BLOCKS = 1024
C0_IDS = 128

C1 = KVGeometry(layers=32, kv=2, block_tokens=16, heads=8, head_dim=128)
C1_POOL_BLOCKS = 32768
C1_BATCH = 512

C2 = KVGeometry(layers=80, kv=2, block_tokens=64, heads=1, head_dim=128)
C2_BATCH = 256


def kv_pool(geom: KVGeometry, num_blocks: int, seed: int, device) -> List[torch.Tensor]:
  """One [num_blocks, tokens, heads, head_dim] bf16 storage per (layer, K/V).

  Values are N(0,1) drawn in the order of the 6-D tensor
  [layers, K/V, blocks, tokens, heads, head_dim].
  """
  full = bf16_normal((geom.layers, geom.kv, num_blocks, geom.block_tokens, geom.heads,
                      geom.head_dim), seed, device=device)
  return [full[l, k] for l in range(geom.layers) for k in range(geom.kv)]


# ---------------------------------------------------------------------------
# Llama-3-8B weights (C4)
# ---------------------------------------------------------------------------

HIDDEN, FFN, VOCAB, N_LAYERS = 4096, 14336, 128256, 32
Q_DIM, KV_DIM = 4096, 1024


def llama3_8b_params() -> List[Tuple[str, Tuple[int, ...], str]]:
  """(name, shape, tp_split) in document order; tp_split in {col,row,vocab,rep}.

  col = column-parallel (dim-0 split), row = row-parallel (dim-1 split),
  vocab = vocab-sharded (dim 0), rep = replicated.
  """
  out = [("embed_tokens", (VOCAB, HIDDEN), "vocab")]
  for i in range(N_LAYERS):
    p = f"layers.{i}."
    out += [
        (p + "q_proj", (Q_DIM, HIDDEN), "col"),
        (p + "k_proj", (KV_DIM, HIDDEN), "col"),
        (p + "v_proj", (KV_DIM, HIDDEN), "col"),
        (p + "o_proj", (HIDDEN, Q_DIM), "row"),
        (p + "gate_proj", (FFN, HIDDEN), "col"),
        (p + "up_proj", (FFN, HIDDEN), "col"),
        (p + "down_proj", (HIDDEN, FFN), "row"),
        (p + "input_layernorm", (HIDDEN,), "rep"),
        (p + "post_attention_layernorm", (HIDDEN,), "rep"),
    ]
  out += [("norm", (HIDDEN,), "rep"), ("lm_head", (VOCAB, HIDDEN), "vocab")]
  return out


def mesh_for(shape, split: str, n: int) -> Tuple[int, ...]:
  """Mesh shape of a parameter sharded `split` over n ranks."""
  if split in ("col", "vocab", "fsdp"):
    return (n,) + (1,) * (len(shape) - 1)
  if split == "row":
    return (1, n) + (1,) * (len(shape) - 2)
  return (1,) * len(shape)


def weight_sync_specs(n_src: int, n_dst: int, params=None):
  """C4 reshard variables: fp32 FSDP dim-0 shards on n_src trainer ranks ->
  bf16 tensor-parallel shards on n_dst sampler ranks.  A replicated
  parameter (the norms) is held whole by every sampler rank, so each of them
  receives it (every trainer rank sends its FSDP slice to each)."""
  from tpu_sync_b200 import reshard_plan as rp
  out = []
  for i, (name, shape, split) in enumerate(params if params is not None else
                                           llama3_8b_params()):
    out.append(rp.VariableSpec(name, tuple(shape), mesh_for(shape, "fsdp", n_src),
                               mesh_for(shape, split, n_dst), layer_idx=i,
                               dst_holders=[0] * n_dst if split == "rep" else None))
  return out


def _cumsum(sizes):
  out, acc = [], 0
  for n in sizes:
    out.append(acc)
    acc += int(n)
  return out, acc


def weight_sync_layout(specs, n_src: int, n_dst: int):
  """Flat-buffer layout of a weight sync: every trainer slot holds its
  source boxes of all variables back to back (variable order), every
  sampler slot its destination boxes.  Returns (src, dst): per slot a pair
  (element offset of each variable, total elements)."""
  import math

  from tpu_sync_b200 import reshard_plan as rp
  src_sizes = [[math.prod(rp.local_shape(rp.shard_boxes(v.shape, v.src_mesh)[v.src_box_of(r)]))
                for v in specs] for r in range(n_src)]
  dst_sizes = [[math.prod(rp.local_shape(rp.shard_boxes(v.shape, v.dst_mesh)[v.dst_box_of(r)]))
                for v in specs] for r in range(n_dst)]
  return [_cumsum(x) for x in src_sizes], [_cumsum(x) for x in dst_sizes]


def weight_sync_chunks(plan, layout, src_slot: int, src_base: int, dst_bases,
                       src_itemsize: int = 4, dst_itemsize: int = 2, dst_slots=None):
  """One trainer slot's chunks over the flat buffers, in the form of
  ops.ReshardProgram: (src address, dst address, src element offset, dst
  element offset, size, src stride, dst stride, count), addresses being each
  variable's start (`src_base` / `dst_bases[d]` plus its byte offset).
  dst_slots: only the chunks into these sampler slots (None: all)."""
  src, dst = layout
  out = []
  for (vi, d), cs in plan.for_source(src_slot).items():
    if dst_slots is not None and d not in dst_slots:
      continue
    sp = src_base + src_itemsize * src[src_slot][0][vi]
    dp = dst_bases[d] + dst_itemsize * dst[d][0][vi]
    for (so, do, size, ss, ds, cnt) in cs:
      out.append((sp, dp, so, do, size, ss, ds, cnt))
  return out


def weight_sync_pull_chunks(plan, layout, dst_slot: int, dst_base: int, n_src: int,
                            dst_itemsize: int = 2, src_slots=None):
  """One sampler slot's chunks for the staged pull (ops.PullReceiver):
  (trainer slot, dst address, src element offset in that trainer's flat
  buffer, dst element offset, size, src stride, dst stride, count).
  src_slots: only the chunks from these trainer slots (None: all)."""
  src, dst = layout
  out = []
  for s in range(n_src):
    if src_slots is not None and s not in src_slots:
      continue
    for (vi, d), cs in plan.for_source(s).items():
      if d != dst_slot:
        continue
      dp = dst_base + dst_itemsize * dst[d][0][vi]
      for (so, do, size, ss, ds, cnt) in cs:
        out.append((s, dp, src[s][0][vi] + so, do, size, ss, ds, cnt))
  return out


# ---------------------------------------------------------------------------
# C1 access trace driving the tier-2 store
# ---------------------------------------------------------------------------

def zipf_trace(n_access: int = 100_000, n_ids: int = 200_000, s: float = 1.1,
               seed: int = 10) -> np.ndarray:
  """n_access block accesses drawn Zipf(s) over n_ids prefix ids.

  Rank r (1-based) has probability proportional to r^-s; ranks map to ids
  through a seeded permutation, so popularity is not correlated with id.
  """
  rng = np.random.default_rng(seed)
  p = np.arange(1, n_ids + 1, dtype=np.float64) ** (-s)
  p /= p.sum()
  ranks = rng.choice(n_ids, size=n_access, p=p)
  return rng.permutation(n_ids)[ranks].astype(np.int64)


def store_transfer_streams(trace: np.ndarray, host_blocks: int, device_blocks: int,
                           batch: int = 512):
  """Runs the access trace through a host-only KVCacheStore.

  Every access gets a device block (a ring over the HBM pool); a hit is
  looked up and loaded into it, a miss is inserted from it and saved.  The
  store's LRU and host block allocator (the reference's policies) choose the
  host ids.  Returns (batches, stats): per access batch, (saves, loads) with
  saves = [(device id, host id)] and loads = [(host id, device id)].  Within a
  batch the two lists never share a host block (loaded blocks are pinned, so
  the save's allocator cannot evict them); a load can depend on an earlier
  batch's save.
  """
  from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId
  store = KVCacheStore(capacity=host_blocks, host_blocks=host_blocks)
  batches = []
  ring = 0
  hits = misses = 0
  for b0 in range(0, len(trace), batch):
    seen, hit_h, hit_dev, miss_h, miss_dev = set(), [], [], [], []
    saves, loads = [], []
    for x in trace[b0:b0 + batch]:
      h = int(x).to_bytes(8, "little")
      if h in seen:
        continue
      seen.add(h)
      d = ring % device_blocks
      ring += 1
      r = store.lookup([h])
      if r:
        hit_h.append(h)
        hit_dev.append(d)
        loads.append((r[0][1].host_block_id, d))
      else:
        miss_h.append(h)
        miss_dev.append(d)
    hits += len(hit_h)
    misses += len(miss_h)
    if hit_h:
      store.load(hit_h, hit_dev)
    if miss_h and store.insert(miss_h, [RaidenBlockId(device_block_id=d, status=BlockStatus.HBM)
                                        for d in miss_dev]):
      if store.save(miss_h):
        store.poll_save_status()
        for h, d in zip(miss_h, miss_dev):
          saves.append((d, store.lookup([h], pin_found=False)[0][1].host_block_id))
      else:
        store.release(miss_h)
    store.poll_load_status()
    store.poll_save_status()
    batches.append((saves, loads))
  stats = {"accesses": int(len(trace)), "hits": hits, "misses": misses,
           "hit_rate": round(hits / max(hits + misses, 1), 4)}
  store.close()
  return batches, stats


# ---------------------------------------------------------------------------
# C3 hand-off as pools + byte-span declarations
# ---------------------------------------------------------------------------

def handoff_pool_plan_inputs(n_storages: int, src_table: np.ndarray, dst_table: np.ndarray,
                             heads: int, head_bytes: int, src_tokens: int = 16,
                             dst_tokens: int = 64):
  """Pools and span declarations of the prefill -> decode KV hand-off.

  One pool per (layer, K/V) storage, all tagged "kv": source pages of
  `src_tokens` tokens, head-major ([head][token][head_bytes]); destination
  pages of `dst_tokens` tokens, token-major ([token][head][head_bytes]).
  src_table[q, p] / dst_table[q, P] are sequence q's page ids.  The single
  source unit declares, per source page and head, one span of src_tokens
  rows (one head vector each) at the head-major source stride and the
  token-major destination stride, page-indexed (dst_space_version 0).
  Returns (src_pools, dst_pools, dst_block_ids, registration).
  """
  from tpu_sync_b200.pool_layout import PoolSpec, RegionSpec
  from tpu_sync_b200.pool_reshard import PoolByteSpan, PoolSpanRegistration
  n_seqs, sbps = src_table.shape
  dbps = dst_table.shape[1]
  per = dst_tokens // src_tokens
  sbb, dbb = src_tokens * heads * head_bytes, dst_tokens * heads * head_bytes
  n_src_blocks = int(src_table.max()) + 1
  n_dst_blocks = int(dst_table.max()) + 1
  src_pools = [PoolSpec("kv", s, 0, sbb, n_src_blocks, (RegionSpec("page", 0, sbb, sbb, 1),))
               for s in range(n_storages)]
  dst_pools = [PoolSpec("kv", s, 0, dbb, n_dst_blocks, (RegionSpec("page", 0, dbb, dbb, 1),))
               for s in range(n_storages)]
  spans = []
  for q in range(n_seqs):
    for p in range(sbps):
      for h in range(heads):
        spans.append(PoolByteSpan(
            src_block_ordinal=q * sbps + p, src_offset_bytes=h * src_tokens * head_bytes,
            dst_block_index=q * dbps + p // per,
            dst_offset_bytes=(p % per) * src_tokens * heads * head_bytes + h * head_bytes,
            size_bytes=head_bytes, src_stride_bytes=head_bytes,
            dst_stride_bytes=heads * head_bytes, count=src_tokens))
  reg = PoolSpanRegistration("kv", [int(x) for x in src_table.reshape(-1)], spans)
  return src_pools, dst_pools, [int(x) for x in dst_table.reshape(-1)], reg

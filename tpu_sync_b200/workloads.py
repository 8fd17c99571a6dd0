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

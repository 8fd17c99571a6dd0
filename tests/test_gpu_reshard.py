"""GPU parity of the weight-sync reshard executor and the KV hand-off relayout
kernel against the CPU oracle (bit-exact, fp32 -> bf16 round-to-nearest-even)."""

import textwrap

import numpy as np
import pytest
import torch

from oracle import fp8 as ofp8
from oracle import reshard as ors
from tpu_sync_b200 import ops, workloads
from tpu_sync_b200 import reshard_plan as rp
from tpu_sync_b200.weight_synchronizer import WeightSynchronizer

pytestmark = pytest.mark.gpu


def small_llama(hidden=256, ffn=640, vocab=1000, layers=2, kv=64):
  """Llama-3-8B-shaped parameter list scaled down (same splits)."""
  out = [("embed_tokens", (vocab, hidden), "vocab")]
  for i in range(layers):
    p = f"layers.{i}."
    out += [(p + "q_proj", (hidden, hidden), "col"), (p + "k_proj", (kv, hidden), "col"),
            (p + "v_proj", (kv, hidden), "col"), (p + "o_proj", (hidden, hidden), "row"),
            (p + "gate_proj", (ffn, hidden), "col"), (p + "up_proj", (ffn, hidden), "col"),
            (p + "down_proj", (hidden, ffn), "row"),
            (p + "input_layernorm", (hidden,), "rep"),
            (p + "post_attention_layernorm", (hidden,), "rep")]
  out += [("norm", (hidden,), "rep"), ("lm_head", (vocab, hidden), "vocab")]
  return out


def execute_specs(cuda, specs, n_src_slots, n_dst_slots, src_dtype=torch.float32,
                  dst_dtype=torch.bfloat16, seed=3, engine="sm"):
  """Runs the plan of `specs` on cuda:0 (source slot s = local shard s of one
  synchronizer, destination slot d = its own tensors) and checks that every
  destination slot holds exactly its box of every variable."""
  g = torch.Generator().manual_seed(seed)
  globals_ = [(torch.randn(v.shape, generator=g) * 0.02).to(src_dtype) for v in specs]
  plan = rp.build_plan(specs)
  grid = []
  for v, full in zip(specs, globals_):
    boxes = rp.shard_boxes(v.shape, v.src_mesh)
    grid.append([full[tuple(slice(a, b) for a, b in boxes[v.src_box_of(s)])].contiguous().to(cuda)
                 for s in range(n_src_slots)])
  ws = WeightSynchronizer(grid)
  dest = {}
  for vi, v in enumerate(specs):
    boxes = rp.shard_boxes(v.shape, v.dst_mesh)
    for d in range(n_dst_slots):
      dest[(vi, d)] = torch.zeros(rp.local_shape(boxes[v.dst_box_of(d)]), dtype=dst_dtype,
                                  device=cuda)
  fut = ws.push_weights_resharded(plan, {s: s for s in range(n_src_slots)}, dest, engine=engine)
  fut.Await()
  torch.cuda.synchronize()
  for vi, v in enumerate(specs):
    want_full = globals_[vi].to(dst_dtype)
    boxes = rp.shard_boxes(v.shape, v.dst_mesh)
    for d in range(n_dst_slots):
      want = want_full[tuple(slice(a, b) for a, b in boxes[v.dst_box_of(d)])]
      got = dest[(vi, d)].cpu()
      assert torch.equal(got.view(torch.int16) if dst_dtype == torch.bfloat16 else got,
                         want.view(torch.int16) if dst_dtype == torch.bfloat16 else want), \
          (v.name, d)
  return plan


def run_reshard(cuda, n_src, n_dst, params, src_dtype=torch.float32, dst_dtype=torch.bfloat16,
                engine="sm"):
  specs = workloads.weight_sync_specs(n_src, n_dst, params)
  return execute_specs(cuda, specs, n_src, n_dst, src_dtype, dst_dtype, engine=engine)


def test_replicated_sources_and_destinations(cuda):
  """Units on named meshes (the reference's sharding specs): trainer units
  on (fsdp=2, tp=2) hold dim-0 halves replicated over tp; sampler units on
  (fsdp=1, tp=4) hold tp quarters of dim 1, or the whole tensor for a
  replicated norm.  Each destination slot gets its box from one holder
  (slot mod holders), the result is exact on every slot."""
  specs = []
  for i, (name, shape, dst_spec, dst_mesh) in enumerate([
      ("o_proj", (64, 96), ["", "tp"], [1, 4]),
      ("norm", (96,), [""], [1]),
      ("emb", (40, 24), ["tp", ""], [4, 1])]):
    src_spec, src_mesh = (["fsdp", ""], [2, 1]) if len(shape) == 2 else (["fsdp"], [2])
    sh = rp.slot_holders(4, src_mesh, src_spec, ["fsdp", "tp"], [2, 2])
    dh = rp.slot_holders(4, dst_mesh, dst_spec, ["fsdp", "tp"], [1, 4])
    specs.append(rp.VariableSpec(name, shape, tuple(src_mesh), tuple(dst_mesh), i, sh, dh))
  assert specs[0].src_holders == [0, 0, 1, 1] and specs[1].dst_holders == [0, 0, 0, 0]
  plan = execute_specs(cuda, specs, 4, 4)
  # de-duplicated: a destination slot takes each source box from one holder
  for vi in range(len(specs)):
    pairs = [(s, d) for (v, s, d) in plan.chunks if v == vi]
    for d in range(4):
      srcs = [s for s, dd in pairs if dd == d]
      boxes = [specs[vi].src_box_of(s) for s in srcs]
      assert len(boxes) == len(set(boxes)), (vi, d, srcs)


@pytest.mark.parametrize("engine", ["sm", "copy"])
@pytest.mark.parametrize("n_src,n_dst", [(4, 4), (1, 1), (1, 2), (2, 4)])
def test_llama_shaped_reshard_fp32_to_bf16(cuda, n_src, n_dst, engine):
  run_reshard(cuda, n_src, n_dst, small_llama(), engine=engine)


def test_copy_engine_program_relaunch_and_identity(cuda):
  """Relaunching reuses the staging only after the previous launch's copies
  left it; same-dtype chunks copy straight from the source; the result is
  exact after every launch."""
  from tpu_sync_b200 import ops
  g = torch.Generator().manual_seed(11)
  src = (torch.randn(512, 96, generator=g) * 0.02).to(cuda)
  dst = torch.zeros(96, 512, dtype=torch.bfloat16, device=cuda)
  # even source rows written transposed: 96 one-element rows at stride 512
  chunks = [(src, dst, r * 96, r, 1, 1, 512, 96) for r in range(0, 512, 2)]
  chunks += [(src, dst, 96, 1, 32, 192, 1024, 0)]  # count 0: nothing
  prog = ops.ReshardCopyEngineProgram(chunks, torch.float32, torch.bfloat16, cuda, groups=5)
  assert prog.groups >= 5 and prog.staging_bytes == 256 * 96 * 2
  want = torch.zeros(96, 512, dtype=torch.bfloat16)
  want[:, 0::2] = src[0::2].cpu().t().to(torch.bfloat16)
  for _ in range(3):
    dst.zero_()
    prog.launch()
    torch.cuda.synchronize()
    assert torch.equal(dst.cpu().view(torch.int16), want.view(torch.int16))
  b_src = torch.randint(0, 256, (4096,), dtype=torch.uint8, device=cuda)
  b_dst = torch.zeros(8192, dtype=torch.uint8, device=cuda)
  ident = ops.ReshardCopyEngineProgram([(b_src, b_dst, 7, 100, 33, 64, 200, 20)],
                                       torch.uint8, torch.uint8, cuda)
  assert ident.staging_bytes == 0
  ident.launch()
  torch.cuda.synchronize()
  want = np.zeros(8192, np.uint8)
  ors.apply_byte_entries(b_src.cpu().numpy(), want, [(7, 100, 33, 64, 200, 20)])
  np.testing.assert_array_equal(b_dst.cpu().numpy(), want)
  # a chunk that would end past its destination is refused before any launch
  with pytest.raises(ValueError, match="chunk 0 ends past its destination"):
    ops.ReshardCopyEngineProgram([(b_src, b_dst, 7, 100, 33, 64, 1000, 20)],
                                 torch.uint8, torch.uint8, cuda)
  with pytest.raises(ValueError, match="chunk 0 ends past its source"):
    ops.ReshardProgram([(b_src, b_dst, 4000, 0, 200, 0, 0, 1)], torch.uint8, torch.uint8, cuda)


def test_reshard_identity_dtype_odd_shapes(cuda):
  params = [("a", (37, 29), "col"), ("b", (13, 51), "row"), ("c", (7,), "rep"),
            ("d", (9, 4, 6), "col")]
  run_reshard(cuda, 3, 2, params, torch.float32, torch.float32)
  run_reshard(cuda, 2, 3, params, torch.bfloat16, torch.bfloat16)


def test_bf16_cast_matches_oracle_rne(cuda):
  v = np.concatenate([np.random.default_rng(4).standard_normal(4097).astype(np.float32),
                      np.array([0.0, -0.0, 3.4e38, 1e-40, np.inf, -np.inf], np.float32)])
  src = torch.from_numpy(v).to(cuda)
  dst = torch.empty(v.size, dtype=torch.bfloat16, device=cuda)
  prog = ops.ReshardProgram([(src, dst, 0, 0, v.size, 0, 0, 1)], torch.float32,
                            torch.bfloat16, cuda)
  prog.launch()
  torch.cuda.synchronize()
  np.testing.assert_array_equal(dst.view(torch.int16).cpu().numpy().view(np.uint16),
                                ofp8.f32_to_bf16_bits_rne(v))


GEOM_SRC = dict(block_tokens=16, heads=2, head_bytes=256, head_major=1)
GEOM_DST = dict(block_tokens=64, heads=2, head_bytes=256, head_major=0)


@pytest.mark.parametrize("seq_tokens", [256, 200, 17])
def test_relayout_head_major16_to_token_major64(cuda, seq_tokens):
  n_seqs, n_st = 3, 4
  rng = np.random.default_rng(7)
  sbps = (seq_tokens + 15) // 16
  dbps = (seq_tokens + 63) // 64
  n_src_blocks, n_dst_blocks = n_seqs * sbps + 5, n_seqs * dbps + 3
  src_table = rng.permutation(n_src_blocks)[:n_seqs * sbps].reshape(n_seqs, sbps).astype(np.int32)
  dst_table = rng.permutation(n_dst_blocks)[:n_seqs * dbps].reshape(n_seqs, dbps).astype(np.int32)
  sbb, dbb = 16 * 2 * 256, 64 * 2 * 256
  srcs = [torch.from_numpy(rng.integers(0, 256, (n_src_blocks, sbb), dtype=np.uint8)).to(cuda)
          for _ in range(n_st)]
  dsts = [torch.zeros((n_dst_blocks, dbb), dtype=torch.uint8, device=cuda) for _ in range(n_st)]
  err = ops.kv_relayout(srcs, dsts, GEOM_SRC, GEOM_DST, torch.from_numpy(src_table),
                        torch.from_numpy(dst_table), seq_tokens, device=cuda)
  torch.cuda.synchronize()
  assert int(err.item()) == 0
  for s, d in zip(srcs, dsts):
    want = np.zeros((n_dst_blocks, dbb), np.uint8)
    ors.relayout(s.cpu().numpy(), want, GEOM_SRC, GEOM_DST, src_table, dst_table, seq_tokens)
    np.testing.assert_array_equal(d.cpu().numpy(), want)


@pytest.mark.parametrize("sg,dg,seq_tokens", [
    # power-of-two geometries (fast kernel): every head-major combination
    ((16, 4, 128, 1), (32, 4, 128, 1), 100), ((16, 4, 128, 0), (64, 4, 128, 1), 130),
    ((8, 8, 256, 0), (16, 8, 256, 0), 77), ((32, 1, 16, 1), (8, 1, 16, 0), 65),
    # not powers of two (generic kernel): 3 heads, 48-byte heads, 24-token pages,
    # a token wider than the CTA (heads x vectors > 256)
    ((16, 3, 128, 1), (64, 3, 128, 0), 90), ((24, 2, 48, 0), (16, 2, 48, 1), 51),
    ((16, 2, 256, 1), (24, 2, 256, 0), 70), ((4, 16, 512, 1), (8, 16, 512, 0), 19)])
def test_relayout_geometries_match_oracle(cuda, sg, dg, seq_tokens):
  sgd = dict(zip(("block_tokens", "heads", "head_bytes", "head_major"), sg))
  dgd = dict(zip(("block_tokens", "heads", "head_bytes", "head_major"), dg))
  n_seqs = 3
  rng = np.random.default_rng(sum(sg) + sum(dg) + seq_tokens)
  sbps = -(-seq_tokens // sg[0])
  dbps = -(-seq_tokens // dg[0])
  n_sb, n_db = n_seqs * sbps + 2, n_seqs * dbps + 2
  st = rng.permutation(n_sb)[:n_seqs * sbps].reshape(n_seqs, sbps).astype(np.int32)
  dt = rng.permutation(n_db)[:n_seqs * dbps].reshape(n_seqs, dbps).astype(np.int32)
  sbb, dbb = sg[0] * sg[1] * sg[2], dg[0] * dg[1] * dg[2]
  srcs = [torch.from_numpy(rng.integers(0, 256, (n_sb, sbb), dtype=np.uint8)).to(cuda)
          for _ in range(2)]
  dsts = [torch.zeros((n_db, dbb), dtype=torch.uint8, device=cuda) for _ in range(2)]
  err = ops.kv_relayout(srcs, dsts, sgd, dgd, torch.from_numpy(st), torch.from_numpy(dt),
                        seq_tokens, device=cuda)
  torch.cuda.synchronize()
  assert int(err.item()) == 0
  for s, d in zip(srcs, dsts):
    want = np.zeros((n_db, dbb), np.uint8)
    ors.relayout(s.cpu().numpy(), want, sgd, dgd, st, dt, seq_tokens)
    np.testing.assert_array_equal(d.cpu().numpy(), want)


def test_relayout_out_of_range_pages_are_skipped_and_flagged(cuda):
  """A page id past a storage (either table) is skipped: nothing lands
  outside the storages, the other pages still move, the flag is set."""
  rng = np.random.default_rng(9)
  T, n_src, n_dst = 128, 8, 2
  st = np.arange(8, dtype=np.int32).reshape(1, 8)
  dt = np.array([[0, 1]], np.int32)
  src = torch.from_numpy(rng.integers(0, 256, (n_src + 1, 16 * 2 * 256), dtype=np.uint8)).to(cuda)
  # storages are views of the first rows; the extra row is a guard band
  dst_full = torch.zeros((n_dst + 1, 64 * 2 * 256), dtype=torch.uint8, device=cuda)
  bad_src = st.copy()
  bad_src[0, 5] = n_src          # one source page past the storage
  err = ops.kv_relayout([src[:n_src]], [dst_full[:n_dst]], GEOM_SRC, GEOM_DST,
                        torch.from_numpy(bad_src), torch.from_numpy(dt), T, device=cuda)
  torch.cuda.synchronize()
  assert int(err.item()) == 1
  want = np.zeros((n_dst + 1, 64 * 2 * 256), np.uint8)
  ors.relayout(src.cpu().numpy(), want, GEOM_SRC, GEOM_DST, st, dt, T)
  got = dst_full.cpu().numpy()
  # tokens 80..95 (source page 5) stay zero; everything else moved
  page5 = np.zeros_like(want)
  ors.relayout(np.where(np.arange(n_src + 1)[:, None] == 5, src.cpu().numpy(), 0).astype(np.uint8),
               page5, GEOM_SRC, GEOM_DST, st, dt, T)
  np.testing.assert_array_equal(got, np.where(page5 != 0, 0, want))
  assert not got[n_dst].any()
  bad_dst = dt.copy()
  bad_dst[0, 1] = n_dst          # one destination page past the storage
  dst_full.zero_()
  err = ops.kv_relayout([src[:n_src]], [dst_full[:n_dst]], GEOM_SRC, GEOM_DST,
                        torch.from_numpy(st), torch.from_numpy(bad_dst), T, device=cuda)
  torch.cuda.synchronize()
  assert int(err.item()) == 1
  got = dst_full.cpu().numpy()
  np.testing.assert_array_equal(got[0], want[0])
  assert not got[1].any() and not got[n_dst].any()


def test_relayout_round_trip(cuda):
  """token-major 64 -> head-major 16 inverts the forward relayout."""
  n_seqs, T = 2, 128
  rng = np.random.default_rng(8)
  st = rng.permutation(20)[:16].reshape(2, 8).astype(np.int32)
  dt = rng.permutation(6)[:4].reshape(2, 2).astype(np.int32)
  src = torch.from_numpy(rng.integers(0, 256, (20, 16 * 2 * 256), dtype=np.uint8)).to(cuda)
  mid = torch.zeros((6, 64 * 2 * 256), dtype=torch.uint8, device=cuda)
  back = torch.zeros_like(src)
  ops.kv_relayout([src], [mid], GEOM_SRC, GEOM_DST, torch.from_numpy(st), torch.from_numpy(dt),
                  T, device=cuda)
  ops.kv_relayout([mid], [back], GEOM_DST, GEOM_SRC, torch.from_numpy(dt), torch.from_numpy(st),
                  T, device=cuda)
  torch.cuda.synchronize()
  used = st.reshape(-1)
  assert torch.equal(back[used], src[used])


# ---------------------------------------------------------------------------
# Controller-made byte schedules (WeightSynchronizerBase::PushWeightsResharded)
# ---------------------------------------------------------------------------

def _entry(**kw):
  e = dict(dst_peer="sampler:0", dst_shard_idx=0, src_offset_bytes=0, dst_offset_bytes=0,
           size_bytes=0, src_stride_bytes=0, dst_stride_bytes=0, count=1, layer_idx=0)
  e.update(kw)
  return e


def _byte_ws(cuda, nbytes, layers=1, fill=0xAB):
  src = [torch.full((nbytes,), fill, dtype=torch.uint8, device=cuda) for _ in range(layers)]
  dst = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda) for _ in range(layers)]
  ws = WeightSynchronizer([[t] for t in src], layer_names=[f"l{i}" for i in range(layers)])
  return ws, src, {("sampler:0", i, 0): dst[i] for i in range(layers)}, dst


def test_entries_exact_boundary_and_zero_bytes(cuda):
  """weight_synchronizer_test.cc:184-272: a whole-slice entry copies every
  byte; a zero-byte entry copies none."""
  ws, _, dests, dst = _byte_ws(cuda, 16384)
  ws.push_weights_resharded_entries({0: [_entry(size_bytes=0)]}, dests).Await()
  assert int(dst[0].count_nonzero()) == 0
  ws.push_weights_resharded_entries({0: [_entry(size_bytes=16384)]}, dests).Await()
  assert bool((dst[0] == 0xAB).all())


def test_entries_errors_match_reference(cuda):
  """:274-360: source range past the shard, layer index past the layers,
  an empty schedule; and the layer-name fallback (:362-460)."""
  ws, _, dests, dst = _byte_ws(cuda, 1024, layers=2)
  with pytest.raises(ValueError, match="^Push range out of bounds$"):
    ws.push_weights_resharded_entries({0: [_entry(src_offset_bytes=500, size_bytes=600)]},
                                      dests)
  with pytest.raises(ValueError, match="^Layer index out of bounds: 2$"):
    ws.push_weights_resharded_entries({0: [_entry(size_bytes=16, layer_idx=2)]}, dests)
  with pytest.raises(ValueError, match="^Push range out of bounds$"):  # a late repeat
    ws.push_weights_resharded_entries({0: [_entry(size_bytes=100, src_stride_bytes=300,
                                                  dst_stride_bytes=100, count=5)]}, dests)
  with pytest.raises(ValueError, match="^Push destination range out of bounds$"):
    ws.push_weights_resharded_entries({0: [_entry(dst_offset_bytes=1000, size_bytes=64)]},
                                      dests)
  ws.push_weights_resharded_entries({}, dests).Await()
  ws.push_weights_resharded_entries({0: []}, dests).Await()
  assert int(dst[0].count_nonzero()) == 0 and int(dst[1].count_nonzero()) == 0
  no_layer = _entry(size_bytes=32)
  del no_layer["layer_idx"]
  with pytest.raises(LookupError, match="Layer name not found in WeightSynchronizer: x"):
    ws.push_weights_resharded_entries({0: [no_layer]}, dests, src_data_name="x")
  ws.push_weights_resharded_entries({0: [no_layer]}, dests, src_data_name="l1").Await()
  assert int(dst[1][:32].ne(0xAB).sum()) == 0 and int(dst[1][32:].count_nonzero()) == 0


def test_entries_strided_repeats_match_oracle(cuda):
  """Random strided entries (counts, strides, odd offsets) against the
  oracle's entry expansion (weight_synchronizer_base.cc:606-667)."""
  rng = np.random.default_rng(17)
  nbytes = 1 << 16
  g = torch.Generator().manual_seed(4)
  src_host = torch.randint(0, 256, (nbytes,), generator=g, dtype=torch.uint8)
  src = src_host.to(cuda)
  dst = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
  ws = WeightSynchronizer([[src]])
  want = np.zeros(nbytes, np.uint8)
  entries, used = [], np.zeros(nbytes, bool)
  while len(entries) < 40:
    size = int(rng.integers(1, 300))
    count = int(rng.integers(1, 6))
    ss = size + int(rng.integers(0, 50)) if count > 1 else 0
    ds = size + int(rng.integers(0, 50)) if count > 1 else 0
    so = int(rng.integers(0, nbytes - (count * max(ss, size) + size)))
    do = int(rng.integers(0, nbytes - (count * max(ds, size) + size)))
    span = [(do + c * (ds if count > 1 else size), size) for c in range(count)]
    if any(used[a:a + n].any() for a, n in span):
      continue  # destinations of one push are disjoint
    for a, n in span:
      used[a:a + n] = True
    entries.append(_entry(src_offset_bytes=so, dst_offset_bytes=do, size_bytes=size,
                          src_stride_bytes=ss, dst_stride_bytes=ds, count=count))
    ors.apply_byte_entries(src_host.numpy(), want,
                           [(so, do, size, ss, ds, count)])
  ws.push_weights_resharded_entries({0: entries}, {("sampler:0", 0, 0): dst}).Await()
  np.testing.assert_array_equal(dst.cpu().numpy(), want)


# ---------------------------------------------------------------------------
# push_weights to "ipc:" endpoints (PushWeights, weight_synchronizer_base.cc:541-556)
# ---------------------------------------------------------------------------

def _grid(cuda, seed, fill=None):
  g = torch.Generator().manual_seed(seed)
  shapes = [[(64, 33), (64, 33)], [(17,), (17,)], [(8, 4, 2), (8, 4, 2)]]
  out = []
  for layer in shapes:
    row = []
    for shp in layer:
      t = torch.randn(shp, generator=g).to(torch.bfloat16)
      row.append((t if fill is None else torch.full(shp, fill, dtype=torch.bfloat16)).to(cuda))
    out.append(row)
  return out


def test_push_weights_to_ipc_endpoint_same_process(cuda):
  src_grid, dst_grid = _grid(cuda, 1), _grid(cuda, 2, fill=0.0)
  src, dst = WeightSynchronizer(src_grid), WeightSynchronizer(dst_grid)
  ep = dst.get_local_endpoint()
  assert ep.startswith("ipc:") and dst.get_local_endpoint() == ep
  src.push_weights([ep])
  for a, b in zip(src_grid, dst_grid):
    for x, y in zip(a, b):
      assert torch.equal(x, y)
  with pytest.raises(ValueError, match="only same-node 'ipc:' endpoints"):
    src.push_weights(["10.0.0.1:8000"])
  other = WeightSynchronizer([[t[:32] for t in src_grid[0]]])
  with pytest.raises(RuntimeError, match="is torch.bfloat16 \\(64, 33\\)"):
    other.push_weights([ep])
  dst.close()
  with pytest.raises(RuntimeError, match="no weight synchronizer endpoint"):
    src.push_weights([ep])


_RECEIVER = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    sys.path.insert(0, {tests!r})
    import torch
    from test_gpu_reshard import _grid
    from tpu_sync_b200.weight_synchronizer import WeightSynchronizer
    dev = torch.device("cuda", 0)
    grid = _grid(dev, 2, fill=0.0)
    ws = WeightSynchronizer(grid)
    print(ws.get_local_endpoint(), flush=True)
    sys.stdin.readline()          # the pusher is done
    want = _grid(dev, 1)
    ok = all(torch.equal(x, y) for a, b in zip(grid, want) for x, y in zip(a, b))
    print("MATCH" if ok else "DIFF", flush=True)
    ws.close()
""")


def test_push_weights_to_ipc_endpoint_other_process(cuda):
  import subprocess, sys
  from pathlib import Path
  here = Path(__file__).resolve().parent
  p = subprocess.Popen([sys.executable, "-c", _RECEIVER.format(root=str(here.parent),
                                                               tests=str(here))],
                       stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                       text=True)
  try:
    ep = p.stdout.readline().strip()
    assert ep.startswith("ipc:"), p.stderr.read()[-3000:]
    WeightSynchronizer(_grid(cuda, 1)).push_weights([ep])
    out, err = p.communicate("done\n", timeout=120)
    assert "MATCH" in out, (out, err[-3000:])
  finally:
    if p.poll() is None:
      p.kill()
      p.wait()

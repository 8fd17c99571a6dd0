"""GPU parity of the staged-pull weight sync (ts_wpull_src_* / ts_wpull_dst_*,
ops.PullSender / ops.PullReceiver): the trainers cast their fp32 shards into
bf16 staging group by group and publish each group in a /dev/shm mailbox;
the samplers read the staging with the reshard kernel as groups appear.

Every sampler buffer is checked bit-exact against the CPU oracle's
application of the same plan (oracle/reshard.py: the reference's entry
expansion, weight_synchronizer_base.cc:606-667, plus the RNE cast), over
several generations, in one process and with the trainer in another process;
the protocol's failures (nothing staged, a receiver that never pulled, a
chunk past the staging) end in errors within the given timeouts."""

import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reshard as ors
from tpu_sync_b200 import _native, ops, workloads
from tpu_sync_b200 import reshard_plan as rp

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def small_params(hidden=256, ffn=640, vocab=1000, layers=2, kv=64):
  """Llama-3-8B-shaped parameters scaled down (the same splits)."""
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


def trainer_flat(n, seed):
  g = torch.Generator().manual_seed(seed)
  return (torch.randn(n, generator=g) * 0.02).float()


def expected(plan, layout, flats, d, n_src):
  """The oracle's bf16 bits of sampler slot d from the trainers' fp32 flats."""
  out = np.zeros(layout[1][d][1], np.uint16)
  chunks = workloads.weight_sync_pull_chunks(plan, layout, d, 0, n_src)
  for s in range(n_src):
    mine = [(so, dp // 2 + do, size, ss, ds, cnt)
            for (t, dp, so, do, size, ss, ds, cnt) in chunks if t == s]
    ors.apply_element_chunks(flats[s], out, mine, cast_bf16=True)
  return out


def name(tag, i):
  return f"tsb_test_pull_{os.getpid()}_{tag}_{i}"


@pytest.mark.parametrize("n_src,n_dst,groups", [(2, 2, 5), (1, 2, 3), (2, 1, 16), (1, 1, 1)])
def test_pull_matches_oracle_over_generations(cuda, n_src, n_dst, groups):
  specs = workloads.weight_sync_specs(n_src, n_dst, small_params())
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, n_src, n_dst)
  srcs = [torch.empty(layout[0][s][1], dtype=torch.float32, device=cuda) for s in range(n_src)]
  senders = [ops.PullSender(name(f"g{n_src}{n_dst}", s), srcs[s], groups=groups)
             for s in range(n_src)]
  dsts = [torch.zeros(layout[1][d][1], dtype=torch.bfloat16, device=cuda) for d in range(n_dst)]
  recv = [ops.PullReceiver([snd.name for snd in senders],
                           workloads.weight_sync_pull_chunks(plan, layout, d, dsts[d].data_ptr(),
                                                             n_src), cuda)
          for d in range(n_dst)]
  assert all(snd.receivers == n_dst for snd in senders)
  try:
    for gen in range(3):
      flats = [trainer_flat(layout[0][s][1], 100 * gen + s) for s in range(n_src)]
      for s in range(n_src):
        srcs[s].copy_(flats[s])
        senders[s].stage()
      for r in recv:
        r.pull()
      torch.cuda.synchronize()
      for d in range(n_dst):
        want = expected(plan, layout, [f.numpy() for f in flats], d, n_src)
        got = dsts[d].view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got, want, err_msg=f"generation {gen}, sampler {d}")
  finally:
    for r in recv:
      r.close()
    for snd in senders:
      snd.close()


def test_pull_times_out_when_nothing_is_staged_and_sender_waits_for_receivers(cuda):
  src = torch.zeros(4096, dtype=torch.float32, device=cuda)
  snd = ops.PullSender(name("timeout", 0), src, groups=4)
  dst = torch.zeros(4096, dtype=torch.bfloat16, device=cuda)
  rcv = ops.PullReceiver([snd.name], [(0, dst, 0, 0, 4096, 4096, 4096, 1)], cuda)
  try:
    with pytest.raises(RuntimeError, match="not published within the timeout"):
      rcv.pull(timeout_ms=200)
    # the receiver attached but has not pulled generation 1: the sender may
    # stage it, but not overwrite it with generation 2
    snd.stage()
    snd.wait()
    with pytest.raises(RuntimeError, match="has not finished pulling generation 1"):
      snd.stage(timeout_ms=200)
  finally:
    rcv.close()
    snd.close()
  torch.cuda.synchronize()
  assert int(dst.view(torch.int16).abs().sum()) == 0


def test_pull_detached_receiver_does_not_hold_the_sender(cuda):
  src = torch.arange(1024, dtype=torch.float32, device=cuda)
  snd = ops.PullSender(name("detach", 0), src, groups=2)
  dst = torch.zeros(1024, dtype=torch.bfloat16, device=cuda)
  rcv = ops.PullReceiver([snd.name], [(0, dst, 0, 0, 1024, 1024, 1024, 1)], cuda)
  rcv.close()  # never pulled; its slot no longer counts
  try:
    for _ in range(3):
      snd.stage(timeout_ms=2000)
      snd.wait()
  finally:
    snd.close()


def test_pull_rejects_chunks_past_the_staging(cuda):
  src = torch.zeros(1000, dtype=torch.float32, device=cuda)
  snd = ops.PullSender(name("range", 0), src, groups=3)
  dst = torch.zeros(4096, dtype=torch.bfloat16, device=cuda)
  try:
    with pytest.raises(RuntimeError, match="reads past the 1000 elements"):
      ops.PullReceiver([snd.name], [(0, dst, 0, 0, 100, 100, 100, 11)], cuda)
    with pytest.raises(RuntimeError, match="reads past"):
      ops.PullReceiver([snd.name], [(0, dst, 950, 0, 51, 51, 51, 1)], cuda)
    with pytest.raises(RuntimeError, match="sender index 1 out of range"):
      ops.PullReceiver([snd.name], [(1, dst, 0, 0, 10, 10, 10, 1)], cuda)
    with pytest.raises(RuntimeError, match="pull mailbox"):
      ops.PullReceiver([name("missing", 0)], [(0, dst, 0, 0, 10, 10, 10, 1)], cuda)
    ok = ops.PullReceiver([snd.name], [(0, dst, 900, 0, 100, 100, 100, 1),
                                       (0, dst, 0, 100, 10, 99, 10, 10)], cuda)
    ok.close()
  finally:
    snd.close()


def test_pull_mailbox_names_are_exclusive(cuda):
  src = torch.zeros(64, dtype=torch.float32, device=cuda)
  snd = ops.PullSender(name("excl", 0), src, groups=1)
  try:
    with pytest.raises(RuntimeError, match="pull mailbox"):
      ops.PullSender(name("excl", 0), src, groups=1)
  finally:
    snd.close()
  again = ops.PullSender(name("excl", 0), src, groups=1)  # unlinked on close
  again.close()


_SENDER = textwrap.dedent("""
    import sys
    sys.path.insert(0, {root!r})
    import torch
    from tpu_sync_b200 import ops
    n, seed, mailbox = {n}, {seed}, {mailbox!r}
    dev = torch.device("cuda", {device})
    g = torch.Generator().manual_seed(seed)
    src = (torch.randn(n, generator=g) * 0.02).float().to(dev)
    snd = ops.PullSender(mailbox, src, groups=7)
    print("READY", flush=True)
    for line in sys.stdin:
      cmd = line.strip()
      if cmd == "GO":
        snd.stage()
        snd.wait()
        print("STAGED", flush=True)
      elif cmd == "EXIT":
        break
    snd.close()
    print("BYE", flush=True)
""")


def test_pull_from_a_sender_in_another_process(cuda):
  """The trainer in a child process (its staging mapped through CUDA IPC),
  the sampler here: two generations of the same values, exact."""
  specs = workloads.weight_sync_specs(1, 2, small_params())
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, 1, 2)
  n = layout[0][0][1]
  mailbox = name("xproc", 0)
  p = subprocess.Popen([sys.executable, "-c", _SENDER.format(root=str(ROOT), n=n, seed=77,
                                                             mailbox=mailbox, device=0)],
                       stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                       text=True)
  try:
    assert p.stdout.readline().strip() == "READY", p.stderr.read()[-3000:]
    dsts = [torch.zeros(layout[1][d][1], dtype=torch.bfloat16, device=cuda) for d in range(2)]
    recv = [ops.PullReceiver([mailbox],
                             workloads.weight_sync_pull_chunks(plan, layout, d,
                                                               dsts[d].data_ptr(), 1), cuda)
            for d in range(2)]
    flat = trainer_flat(n, 77).numpy()
    for gen in range(2):
      for d in range(2):
        dsts[d].zero_()
      torch.cuda.synchronize()
      p.stdin.write("GO\n")
      p.stdin.flush()
      for r in recv:
        r.pull(timeout_ms=60000)
      torch.cuda.synchronize()
      assert p.stdout.readline().strip() == "STAGED"
      for d in range(2):
        want = expected(plan, layout, [flat], d, 1)
        got = dsts[d].view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got, want, err_msg=f"generation {gen}, sampler {d}")
    for r in recv:
      r.close()
    p.stdin.write("EXIT\n")
    p.stdin.flush()
    out, err = p.communicate(timeout=60)
    assert "BYE" in out, err[-3000:]
  finally:
    if p.poll() is None:
      p.kill()
      p.wait()


def test_hybrid_pull_own_trainer_and_push_the_rest(cuda):
  """bench.py's hybrid weight sync (2 -> 2) on one GPU: sampler d pulls only
  from trainer d's staging, trainer t pushes its slices for the other
  sampler with the SM kernel (fp32 -> bf16) while it casts; exact against
  the oracle over two generations."""
  n = 2
  specs = workloads.weight_sync_specs(n, n, small_params())
  plan = rp.build_plan(specs)
  layout = workloads.weight_sync_layout(specs, n, n)
  srcs = [torch.empty(layout[0][s][1], dtype=torch.float32, device=cuda) for s in range(n)]
  dsts = [torch.zeros(layout[1][d][1], dtype=torch.bfloat16, device=cuda) for d in range(n)]
  senders = [ops.PullSender(name("hyb", s), srcs[s], groups=6) for s in range(n)]
  recv = [ops.PullReceiver([senders[d].name],
                           [(0,) + tuple(c[1:]) for c in workloads.weight_sync_pull_chunks(
                               plan, layout, d, dsts[d].data_ptr(), n, src_slots={d})], cuda)
          for d in range(n)]
  cross = [ops.ReshardProgram(workloads.weight_sync_chunks(
      plan, layout, t, srcs[t].data_ptr(), {d: dsts[d].data_ptr() for d in range(n)},
      dst_slots=set(range(n)) - {t}), torch.float32, torch.bfloat16, cuda) for t in range(n)]
  side = torch.cuda.Stream(cuda)
  try:
    for gen in range(2):
      flats = [trainer_flat(layout[0][s][1], 300 + 10 * gen + s) for s in range(n)]
      for d in range(n):
        dsts[d].zero_()
      for t in range(n):
        srcs[t].copy_(flats[t])
        side.wait_stream(torch.cuda.current_stream(cuda))
        cross[t].launch(side)
        senders[t].stage()
        torch.cuda.current_stream(cuda).wait_stream(side)
      for r in recv:
        r.pull()
      torch.cuda.synchronize()
      for d in range(n):
        want = expected(plan, layout, [f.numpy() for f in flats], d, n)
        got = dsts[d].view(torch.int16).cpu().numpy().view(np.uint16)
        np.testing.assert_array_equal(got, want, err_msg=f"generation {gen}, sampler {d}")
  finally:
    for r in recv:
      r.close()
    for snd in senders:
      snd.close()

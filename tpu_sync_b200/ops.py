"""Tensor-level wrappers of the manager-free kernels of the C ABI.

These take torch CUDA tensors, build the small device-side descriptor tables
the kernels read, and launch on the current stream.  They are what the
manager, the weight synchronizer and the hand-off executor are made of, and
what the parity tests and the benchmark call directly.
"""

from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import numpy as np
import torch

from tpu_sync_b200 import _native


def _stream(stream: Optional[torch.cuda.Stream], device) -> ctypes.c_void_p:
  s = stream if stream is not None else torch.cuda.current_stream(device)
  return ctypes.c_void_p(s.cuda_stream)


def _nbytes(t: torch.Tensor) -> int:
  return t.numel() * t.element_size()


def _to_device_bytes(arr: ctypes.Array, device) -> torch.Tensor:
  raw = np.frombuffer(bytes(arr), dtype=np.uint8).copy()
  return torch.from_numpy(raw).to(device)


class StorageTable:
  """Device table of (layer, shard) storages for the block kernels.

  stage_off of storage s = sum of the (16-byte rounded) slot bytes of the
  storages before it, so a staging block is [storage 0 | storage 1 | ...].
  `slot_scale` = 0.5 lays out fp8 payload slots (half the bf16 bytes).
  """

  def __init__(self, storages: Sequence[torch.Tensor], fp8: bool = False):
    if not storages:
      raise ValueError("need at least one storage")
    self.storages = list(storages)
    self.device = self.storages[0].device
    n = len(self.storages)
    arr = (_native.BlockStorage * n)()
    off = 0
    self.block_bytes = []
    self.stage_offs = []
    for i, t in enumerate(self.storages):
      if not t.is_cuda or not t.is_contiguous():
        raise ValueError("storages must be contiguous CUDA tensors")
      if t.device != self.device:
        raise ValueError("all storages must live on one device")
      bb = _nbytes(t) // t.shape[0]
      arr[i].dev_ptr = t.data_ptr()
      arr[i].block_bytes = bb
      arr[i].dev_bytes = _nbytes(t)
      arr[i].stage_off = off
      self.block_bytes.append(bb)
      self.stage_offs.append(off)
      slot = bb // 2 if fp8 else bb
      off += (slot + 15) // 16 * 16
    self.scale_off = off if fp8 else 0
    if fp8:
      off += (4 * n + 15) // 16 * 16
    self.pitch = (off + 15) // 16 * 16
    self.fp8 = fp8
    self.d_table = _to_device_bytes(arr, self.device)
    self.n = n

  def new_staging(self, n_blocks: int) -> torch.Tensor:
    return torch.empty((n_blocks, self.pitch), dtype=torch.uint8, device=self.device)


def _keep(tensors, stream: Optional[torch.cuda.Stream]) -> None:
  """Keeps temporaries alive for kernels queued on a non-current stream."""
  if stream is not None:
    for t in tensors:
      t.record_stream(stream)


def _ids(ids, device) -> torch.Tensor:
  if isinstance(ids, torch.Tensor):
    t = ids.to(device=device, dtype=torch.int64).contiguous()
  else:
    t = torch.tensor(list(ids), dtype=torch.int64, device=device)
  return t


def kv_extract(table: StorageTable, ids, staging: torch.Tensor,
               err_flag: Optional[torch.Tensor] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.Tensor:
  """staging[k] <- block ids[k] of every storage (block-major)."""
  d_ids = _ids(ids, table.device)
  fn = _native.lib().ts_kv_extract_fp8 if table.fp8 else _native.lib().ts_kv_extract
  args = [table.device.index, ctypes.c_void_p(table.d_table.data_ptr()), table.n,
          ctypes.c_void_p(d_ids.data_ptr()), d_ids.numel(),
          ctypes.c_void_p(staging.data_ptr()), table.pitch]
  if table.fp8:
    args.append(table.scale_off)
  args += [ctypes.c_void_p(err_flag.data_ptr() if err_flag is not None else 0),
           _stream(stream, table.device)]
  _native.check(fn(*args), "kv_extract: ")
  _keep([d_ids], stream)
  return staging


def kv_insert(table: StorageTable, ids, staging: torch.Tensor,
              err_flag: Optional[torch.Tensor] = None,
              stream: Optional[torch.cuda.Stream] = None) -> None:
  """block ids[k] of every storage <- staging[k]."""
  d_ids = _ids(ids, table.device)
  fn = _native.lib().ts_kv_insert_fp8 if table.fp8 else _native.lib().ts_kv_insert
  args = [table.device.index, ctypes.c_void_p(table.d_table.data_ptr()), table.n,
          ctypes.c_void_p(d_ids.data_ptr()), d_ids.numel(),
          ctypes.c_void_p(staging.data_ptr()), table.pitch]
  if table.fp8:
    args.append(table.scale_off)
  args += [ctypes.c_void_p(err_flag.data_ptr() if err_flag is not None else 0),
           _stream(stream, table.device)]
  _native.check(fn(*args), "kv_insert: ")
  _keep([d_ids], stream)


_TORCH_TO_TS = {torch.uint8: _native.DTYPE_U8, torch.bfloat16: _native.DTYPE_BF16,
                torch.float32: _native.DTYPE_F32, torch.float16: _native.DTYPE_F16}


def _extent_bytes(x) -> Optional[int]:
  """Bytes a chunk endpoint holds when it knows its size (a tensor or a
  PeerBuffer), else None (a raw address)."""
  if isinstance(x, torch.Tensor):
    return x.numel() * x.element_size()
  if isinstance(x, (int, np.integer)):
    return None
  if hasattr(x, "nbytes"):
    return int(x.nbytes)
  return None


def _check_chunks(chunks, src_es: int, dst_es: int) -> None:
  """Every chunk stays inside its source and destination where their sizes
  are known: (offset + (count - 1) * stride + size) elements."""
  for i, (sp, dp, so, do, size, ss, ds, cnt) in enumerate(chunks):
    if size <= 0 or cnt <= 0:
      continue
    for name, obj, off, stride, es in (("source", sp, so, ss, src_es),
                                       ("destination", dp, do, ds, dst_es)):
      n = _extent_bytes(obj)
      if n is None:
        continue
      end = (off + (cnt - 1) * stride + size) * es if cnt > 1 else (off + size * cnt) * es
      if off < 0 or end > n:
        raise ValueError(f"chunk {i} ends past its {name}: byte {end} of {n}")


class ReshardProgram:
  """A list of strided chunks compiled for one launch of ts_reshard_copy.

  chunks: iterables (src_tensor, dst_tensor_or_ptr, src_off, dst_off, size,
  src_stride, dst_stride, count) in elements.  All sources must be on
  `device`; destinations may be local or peer-GPU addresses.
  """

  def __init__(self, chunks, src_dtype: torch.dtype, dst_dtype: torch.dtype,
               device: torch.device):
    self.device = torch.device(device)
    self.src_dtype = _TORCH_TO_TS[src_dtype]
    self.dst_dtype = _TORCH_TO_TS[dst_dtype]
    chunks = list(chunks)
    _check_chunks(chunks, torch.empty((), dtype=src_dtype).element_size(),
                  torch.empty((), dtype=dst_dtype).element_size())
    n = len(chunks)
    arr = (_native.ReshardChunk * max(n, 1))()
    for i, (sp, dp, so, do, size, ss, ds, cnt) in enumerate(chunks):
      arr[i].src_ptr = sp.data_ptr() if hasattr(sp, "data_ptr") else int(sp)
      arr[i].dst_ptr = dp.data_ptr() if hasattr(dp, "data_ptr") else int(dp)
      arr[i].src_off, arr[i].dst_off, arr[i].size = int(so), int(do), int(size)
      arr[i].src_stride, arr[i].dst_stride, arr[i].count = int(ss), int(ds), int(cnt)
    prefix = np.zeros(n + 1, dtype=np.int64)
    _native.check(_native.lib().ts_reshard_work_items(
        arr, n, self.src_dtype, self.dst_dtype,
        prefix.ctypes.data_as(_native.c_i64_p)), "reshard plan: ")
    self.n_chunks = n
    self.n_items = int(prefix[-1])
    self.d_chunks = _to_device_bytes(arr, self.device)
    self.d_prefix = torch.from_numpy(prefix).to(self.device)

  def launch(self, stream: Optional[torch.cuda.Stream] = None) -> None:
    _native.check(_native.lib().ts_reshard_copy(
        self.device.index, ctypes.c_void_p(self.d_chunks.data_ptr()),
        ctypes.c_void_p(self.d_prefix.data_ptr()), self.n_chunks, self.n_items,
        self.src_dtype, self.dst_dtype, _stream(stream, self.device)), "reshard: ")


def _pages(storages, geom: dict, given: Optional[int], side: str) -> int:
  """Pages every storage holds: `given`, else the smallest storage's bytes
  (tensors and PeerBuffers know theirs) over the page size."""
  if given is not None:
    return int(given)
  page = int(geom["block_tokens"]) * int(geom["heads"]) * int(geom["head_bytes"])
  sizes = []
  for x in storages:
    if isinstance(x, torch.Tensor):
      sizes.append(x.numel() * x.element_size())
    elif hasattr(x, "nbytes"):
      sizes.append(int(x.nbytes))
    else:
      raise ValueError(f"{side} storages given as raw addresses need {side}_pages")
  return min(sizes) // page


class ReshardCopyEngineProgram:
  """The same chunks as ReshardProgram, pushed by the copy engines: the cast
  to the destination dtype goes to a local staging buffer and each staged
  chunk moves with one cudaMemcpy2DAsync, `groups` groups pipelining the
  cast against the copies (ts_reshard_ce_*)."""

  def __init__(self, chunks, src_dtype: torch.dtype, dst_dtype: torch.dtype,
               device: torch.device, groups: int = 16):
    self.device = torch.device(device)
    chunks = list(chunks)
    _check_chunks(chunks, torch.empty((), dtype=src_dtype).element_size(),
                  torch.empty((), dtype=dst_dtype).element_size())
    arr = (_native.ReshardChunk * max(len(chunks), 1))()
    for i, (sp, dp, so, do, size, ss, ds, cnt) in enumerate(chunks):
      arr[i].src_ptr = sp.data_ptr() if hasattr(sp, "data_ptr") else int(sp)
      arr[i].dst_ptr = dp.data_ptr() if hasattr(dp, "data_ptr") else int(dp)
      arr[i].src_off, arr[i].dst_off, arr[i].size = int(so), int(do), int(size)
      arr[i].src_stride, arr[i].dst_stride, arr[i].count = int(ss), int(ds), int(cnt)
    h = ctypes.c_void_p()
    _native.check(_native.lib().ts_reshard_ce_create(
        self.device.index, arr, len(chunks), _TORCH_TO_TS[src_dtype], _TORCH_TO_TS[dst_dtype],
        int(groups), ctypes.byref(h)), "reshard (copy engines): ")
    self._h = h
    g, b, c = ctypes.c_int64(), ctypes.c_uint64(), ctypes.c_int64()
    _native.check(_native.lib().ts_reshard_ce_info(h, ctypes.byref(g), ctypes.byref(b),
                                                   ctypes.byref(c)))
    self.groups, self.staging_bytes, self.copies = g.value, b.value, c.value

  def launch(self, stream: Optional[torch.cuda.Stream] = None) -> None:
    _native.check(_native.lib().ts_reshard_ce_launch(self._h, _stream(stream, self.device)),
                  "reshard (copy engines): ")

  def close(self) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_reshard_ce_destroy(self._h)
      self._h = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass


class PullSender:
  """Sender side of the staged-pull weight sync (ts_wpull_src_*): casts the
  fp32 `src` (a 1-D CUDA tensor, the shard as the receivers' chunks address
  it) into a bf16 staging of the same element layout in `groups` groups, and
  publishes each group in the /dev/shm mailbox `name` as soon as it is
  written.  `stage()` is one generation; it first waits until every attached
  receiver has pulled the previous one."""

  def __init__(self, name: str, src: torch.Tensor, groups: int = 16):
    if src.dtype != torch.float32 or not src.is_cuda or not src.is_contiguous():
      raise ValueError("PullSender needs a contiguous fp32 CUDA tensor")
    self.device = src.device
    self.name = name
    self._src = src  # kept alive: the cast kernels read it
    h = ctypes.c_void_p()
    _native.check(_native.lib().ts_wpull_src_create(
        self.device.index, name.encode(), ctypes.c_void_p(src.data_ptr()), src.numel(),
        int(groups), ctypes.byref(h)), "weight pull sender: ")
    self._h = h
    g, b = ctypes.c_int64(), ctypes.c_uint64()
    _native.check(_native.lib().ts_wpull_src_info(h, None, ctypes.byref(g), ctypes.byref(b), None))
    self.groups, self.staging_bytes = g.value, b.value

  def stage(self, stream: Optional[torch.cuda.Stream] = None, timeout_ms: int = 30000) -> None:
    _native.check(_native.lib().ts_wpull_src_stage(self._h, _stream(stream, self.device),
                                                   int(timeout_ms)), "weight pull sender: ")

  def wait(self, timeout_ms: int = 30000) -> None:
    _native.check(_native.lib().ts_wpull_src_wait(self._h, int(timeout_ms)),
                  "weight pull sender: ")

  @property
  def receivers(self) -> int:
    n = ctypes.c_int64()
    _native.check(_native.lib().ts_wpull_src_info(self._h, None, None, None, ctypes.byref(n)))
    return n.value

  def close(self) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_wpull_src_destroy(self._h)
      self._h = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass


class PullReceiver:
  """Receiver side of the staged-pull weight sync (ts_wpull_dst_*).

  names: the senders' mailboxes.  chunks: iterables (sender_index,
  dst_tensor_or_ptr, src_off, dst_off, size, src_stride, dst_stride, count)
  in bf16 elements; the source is the sender's staging (its fp32 shard's
  element layout).  `pull()` launches every chunk's copy on `stream` as soon
  as the groups it reads are published, and returns once all are queued."""

  def __init__(self, names: Sequence[str], chunks, device: torch.device):
    self.device = torch.device(device)
    chunks = list(chunks)
    _check_chunks([(None,) + tuple(c[1:]) for c in chunks], 2, 2)
    arr = (_native.ReshardChunk * max(len(chunks), 1))()
    self._keep = []
    for i, (t, dp, so, do, size, ss, ds, cnt) in enumerate(chunks):
      arr[i].src_ptr = int(t)
      arr[i].dst_ptr = dp.data_ptr() if hasattr(dp, "data_ptr") else int(dp)
      if hasattr(dp, "data_ptr"):
        self._keep.append(dp)
      arr[i].src_off, arr[i].dst_off, arr[i].size = int(so), int(do), int(size)
      arr[i].src_stride, arr[i].dst_stride, arr[i].count = int(ss), int(ds), int(cnt)
    cnames = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    h = ctypes.c_void_p()
    _native.check(_native.lib().ts_wpull_dst_create(
        self.device.index, cnames, len(names), arr, len(chunks), ctypes.byref(h)),
        "weight pull receiver: ")
    self._h = h
    lc, b = ctypes.c_int64(), ctypes.c_uint64()
    _native.check(_native.lib().ts_wpull_dst_info(h, None, ctypes.byref(lc), ctypes.byref(b)))
    self.launches, self.bytes = lc.value, b.value

  def pull(self, stream: Optional[torch.cuda.Stream] = None, timeout_ms: int = 30000) -> None:
    _native.check(_native.lib().ts_wpull_dst_pull(self._h, _stream(stream, self.device),
                                                  int(timeout_ms)), "weight pull receiver: ")

  def close(self) -> None:
    if getattr(self, "_h", None):
      _native.lib().ts_wpull_dst_destroy(self._h)
      self._h = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass


def kv_relayout(src_storages: Sequence, dst_storages: Sequence, src_geom: dict,
                dst_geom: dict, src_table: torch.Tensor, dst_table: torch.Tensor,
                seq_tokens: int, device=None,
                stream: Optional[torch.cuda.Stream] = None, src_pages: Optional[int] = None,
                dst_pages: Optional[int] = None,
                err: Optional[torch.Tensor] = None) -> torch.Tensor:
  """Copies every token of every sequence between two page geometries.

  src_storages / dst_storages: tensors, PeerBuffers or raw device addresses
  (destinations may be peer-GPU addresses; raw addresses need src_pages /
  dst_pages, the pages each storage holds).  Geometries are dicts with
  block_tokens, heads, head_bytes, head_major.  Tables are int32
  [n_seqs, blocks_per_seq].  Table entries outside a storage's pages are
  skipped and flagged: returns the device int32 flag (`err`, or a new one),
  non-zero after the kernel ran if any entry was out of range.
  """
  device = torch.device(device) if device is not None else src_table.device
  n = len(src_storages)
  if len(dst_storages) != n:
    raise ValueError("source and destination storage counts differ")
  sp = _pages(src_storages, src_geom, src_pages, "src")
  dp = _pages(dst_storages, dst_geom, dst_pages, "dst")
  if err is None:
    err = torch.zeros(1, dtype=torch.int32, device=device)
  ptr = lambda x: x.data_ptr() if hasattr(x, "data_ptr") else int(x)
  d_src = torch.tensor([ptr(x) for x in src_storages], dtype=torch.int64,
                       device=device)
  d_dst = torch.tensor([ptr(x) for x in dst_storages], dtype=torch.int64,
                       device=device)
  sg = _native.PageGeometry(int(src_geom["block_tokens"]), int(src_geom["heads"]),
                            int(src_geom["head_bytes"]), int(src_geom["head_major"]), 0)
  dg = _native.PageGeometry(int(dst_geom["block_tokens"]), int(dst_geom["heads"]),
                            int(dst_geom["head_bytes"]), int(dst_geom["head_major"]), 0)
  st = src_table.to(device=device, dtype=torch.int32).contiguous()
  dt = dst_table.to(device=device, dtype=torch.int32).contiguous()
  _native.check(_native.lib().ts_kv_relayout(
      device.index, ctypes.c_void_p(d_src.data_ptr()), ctypes.c_void_p(d_dst.data_ptr()),
      n, sg, dg, ctypes.c_void_p(st.data_ptr()), st.shape[1],
      ctypes.c_void_p(dt.data_ptr()), dt.shape[1], st.shape[0], int(seq_tokens), sp, dp,
      ctypes.c_void_p(err.data_ptr()), _stream(stream, device)), "kv_relayout: ")
  _keep([d_src, d_dst, st, dt, err], stream)
  return err

"""WeightSynchronizer: trainer -> sampler weight reshard on B200 GPUs.

Keeps the reference surface (tpu_sync/api/torch/weight_synchronizer.py:36-123:
``WeightSynchronizer(device_tensors[layers][shards], ...)``, ``d2h()``,
``h2d()``, ``get_host_buffer(layer, shard)``, ``push_weights(peers)``) and
replaces the resharded push (WeightSynchronizerBase::PushWeightsResharded,
tpu_sync/weight_sync/weight_synchronizer_base.cc:558-760: per-layer D2H, TCP
push of strided chunks into the peers' host buffers, H2D on the receiver)
with one kernel per source GPU that reads the trainer shard in HBM, converts
fp32 -> bf16 on the way when the sampler is bf16, and stores straight into the
sampler tensors -- on the same GPU or on a peer GPU over NVLink (peer pointers
within a process, CUDA IPC mappings across processes).

Destinations are described by a ``{(var_index, dst_shard): tensor}`` map; in a
multi-process job the sampler ranks export theirs with
``export_destinations`` and the trainer ranks map them with
``import_destinations``.
"""

from __future__ import annotations

import ctypes
import os
import pickle
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch

from tpu_sync_b200 import _native, ops
from tpu_sync_b200.reshard_plan import ReshardPlan


def enable_peer_access(device: int, peer: int) -> None:
  """Lets kernels on `device` load / store `peer`'s memory (idempotent)."""
  if device == peer:
    return
  _native.check(_native.lib().ts_enable_peer_access(int(device), int(peer)),
                "enable_peer_access: ")


class PushFuture:
  """Completion of one resharded push (device-side event on the source)."""

  def __init__(self, event: torch.cuda.Event, programs):
    self._event = event
    self._programs = programs  # keep device tables alive until completion

  def is_ready(self) -> bool:
    return self._event.query()

  def Await(self) -> None:
    self._event.synchronize()

  wait = Await

  def stream_wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
    (stream or torch.cuda.current_stream()).wait_event(self._event)


class WeightSynchronizer:
  """Zero-copy trainer -> sampler weight movement."""

  def __init__(
      self,
      device_tensors: List[List[torch.Tensor]],
      local_port: Optional[int] = None,
      parallelism: int = 1,
      listener_port: Optional[int] = None,
      bind_ip: Optional[str] = None,
      unsafe_skip_buffer_lock: bool = True,
      auto_h2d: bool = False,
      *,
      layer_names: Optional[Sequence[str]] = None,
  ):
    grid = [[t] if isinstance(t, torch.Tensor) else list(t) for t in device_tensors]
    if not grid or not grid[0]:
      raise ValueError("device_tensors must hold at least one tensor")
    n_sh = len(grid[0])
    for layer in grid:
      if len(layer) != n_sh:
        raise RuntimeError("Number of shards mismatch across layers")
      for t in layer:
        if not t.is_cuda or not t.is_contiguous():
          raise ValueError("device tensors must be contiguous CUDA tensors")
    self._grid = grid
    self.layer_names = list(layer_names) if layer_names else [str(i) for i in range(len(grid))]
    self._host: Dict[Tuple[int, int], torch.Tensor] = {}
    self.auto_h2d = auto_h2d
    self._wsync = None  # native ts_wsync of the resharded push, made on first use

  # -- reference properties --------------------------------------------------
  @property
  def num_layers(self) -> int:
    return len(self._grid)

  @property
  def num_shards(self) -> int:
    return len(self._grid[0])

  @property
  def slice_byte_size(self) -> int:
    t = self._grid[0][0]
    return t.numel() * t.element_size() // max(t.shape[0], 1) if t.dim() else t.element_size()

  @property
  def local_port(self) -> Optional[int]:
    return None

  @property
  def listener_port(self) -> Optional[int]:
    return None

  @property
  def is_listener_active(self) -> bool:
    return False

  # -- host staging (reference d2h / h2d / get_host_buffer) -----------------
  def _host_buf(self, l: int, s: int) -> torch.Tensor:
    key = (l, s)
    if key not in self._host:
      t = self._grid[l][s]
      self._host[key] = torch.empty(t.numel() * t.element_size(), dtype=torch.uint8,
                                    pin_memory=True)
    return self._host[key]

  def d2h(self) -> None:
    """Copies every (layer, shard) tensor into its pinned host buffer."""
    for l, layer in enumerate(self._grid):
      for s, t in enumerate(layer):
        self._host_buf(l, s).copy_(t.view(-1).view(torch.uint8), non_blocking=True)
    for layer in self._grid:
      for t in layer:
        torch.cuda.current_stream(t.device).synchronize()

  def h2d(self) -> None:
    """Copies every pinned host buffer back into its device tensor."""
    for l, layer in enumerate(self._grid):
      for s, t in enumerate(layer):
        t.view(-1).view(torch.uint8).copy_(self._host_buf(l, s), non_blocking=True)
    for layer in self._grid:
      for t in layer:
        torch.cuda.current_stream(t.device).synchronize()

  def get_host_buffer(self, layer_idx: int = 0, shard_idx: int = 0) -> torch.Tensor:
    """Zero-copy uint8 host view of one (layer, shard) staging buffer."""
    if not (0 <= layer_idx < self.num_layers and 0 <= shard_idx < self.num_shards):
      raise RuntimeError("layer or shard index out of range")
    return self._host_buf(layer_idx, shard_idx)

  def get_local_endpoint(self) -> str:
    """"ipc:<name>": this synchronizer's [layer][shard] buffers, published for
    peers' push_weights on the same node (CUDA IPC descriptors in /dev/shm).
    The buffers stay valid while this synchronizer lives; close() withdraws
    the endpoint."""
    if getattr(self, "_endpoint", None) is None:
      desc = export_destinations({(l, s): t for l, layer in enumerate(self._grid)
                                  for s, t in enumerate(layer)})
      local = {k: (t.data_ptr(), t.device.index) for k, t in
               ((k, self._grid[k[0]][k[1]]) for k in desc)}
      name = f"tsb_ws_{os.getpid()}_{id(self) & 0xffffffff:x}"
      with open(os.path.join("/dev/shm", name), "wb") as f:
        pickle.dump({"pid": os.getpid(), "desc": desc, "local": local}, f)
      self._endpoint = "ipc:" + name
    return self._endpoint

  def close(self) -> None:
    w = getattr(self, "_wsync", None)
    if w is not None:
      _native.lib().ts_wsync_destroy(w)  # waits for a push still running
      self._wsync = None
    ep = getattr(self, "_endpoint", None)
    if ep is not None:
      try:
        os.unlink(os.path.join("/dev/shm", ep[4:]))
      except FileNotFoundError:
        pass
      self._endpoint = None

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass

  def _push_to_endpoint(self, endpoint: str) -> None:
    """Byte copy of every (layer, shard) buffer into the peer's, one kernel
    per source GPU storing over NVLink."""
    try:
      with open(os.path.join("/dev/shm", endpoint[4:]), "rb") as f:
        info = pickle.load(f)
    except FileNotFoundError:
      raise RuntimeError(f"no weight synchronizer endpoint {endpoint}") from None
    desc = info["desc"]
    by_dev: Dict[int, List] = {}
    for l, layer in enumerate(self._grid):
      for s, t in enumerate(layer):
        if (l, s) not in desc:
          raise RuntimeError(f"peer {endpoint} has no buffer for layer {l} shard {s}")
        peer_dev, _, _, dtype, shape = desc[(l, s)]
        if dtype != t.dtype or tuple(shape) != tuple(t.shape):
          raise RuntimeError(f"peer {endpoint} layer {l} shard {s} is {dtype} {tuple(shape)}, "
                             f"this synchronizer's {t.dtype} {tuple(t.shape)}")
        dev = t.device.index
        if info["pid"] == os.getpid():  # the same process: plain peer pointers
          ptr = info["local"][(l, s)][0]
          enable_peer_access(dev, peer_dev)
        else:
          ptr = import_destinations({0: desc[(l, s)]}, kernel_device=dev)[0].data_ptr()
        n = t.numel() * t.element_size()
        by_dev.setdefault(dev, []).append((t.data_ptr(), ptr, 0, 0, n, 0, 0, 1))
    for dev, chunks in by_dev.items():
      device = torch.device("cuda", dev)
      prog = ops.ReshardProgram(chunks, torch.uint8, torch.uint8, device)
      prog.launch(torch.cuda.current_stream(device))
      torch.cuda.current_stream(device).synchronize()

  def push_weights(self, peers: Sequence[Any]) -> None:
    """Whole-buffer push to peer synchronizers with the same layout
    (PushWeights, weight_synchronizer_base.cc:541-556: D2H, then a TCP push
    of every host buffer), here straight between device buffers.

    ``peers``: "ipc:<name>" endpoints of synchronizers in other processes of
    this node (get_local_endpoint()), WeightSynchronizer objects, or
    [layers][shards] tensor grids, all with this synchronizer's shapes.
    Returns when every byte has landed.
    """
    if not peers:
      raise RuntimeError("Peer list cannot be empty for trainer weights sync")
    for p in peers:
      if isinstance(p, str):
        if not p.startswith("ipc:"):
          raise ValueError(f"peer {p!r}: only same-node 'ipc:' endpoints are supported "
                           "(get_local_endpoint()); there is no TCP transport")
        self._push_to_endpoint(p)
        continue
      grid = p._grid if isinstance(p, WeightSynchronizer) else p
      for l, layer in enumerate(self._grid):
        for s, t in enumerate(layer):
          grid[l][s].copy_(t, non_blocking=True)
    torch.cuda.synchronize()

  # -- resharded push -------------------------------------------------------
  def push_weights_resharded(self, plan: ReshardPlan, src_shards: Dict[int, int],
                             destinations: Dict[Tuple[int, int], torch.Tensor],
                             stream: Optional[torch.cuda.Stream] = None,
                             engine: str = "sm") -> PushFuture:
    """Executes every chunk of `plan` whose source shard lives here.

    engine: "sm" — one kernel per source GPU casts and stores into the
    destinations; "copy" — the kernel casts into local staging and the copy
    engines move the chunks (ops.ReshardCopyEngineProgram).

    src_shards: local shard index -> plan source shard index.
    destinations: (var index, plan dst shard) -> destination tensor (local or
      on a peer GPU of this process) or PeerBuffer (another process's memory,
      from import_destinations with this source's device).  Variable v reads layer
      ``plan.variables[v].layer_idx`` of this synchronizer.
    """
    programs = []
    last_event = None
    for local, src_shard in src_shards.items():
      by_kind: Dict[Tuple[torch.dtype, torch.dtype], List] = {}
      device = None
      for (vi, d), chunks in plan.for_source(src_shard).items():
        var = plan.variables[vi]
        src = self._grid[var.layer_idx][local]
        dst = destinations.get((vi, d))
        if dst is None:
          continue
        device = src.device
        if isinstance(dst, torch.Tensor) and dst.device != src.device:
          enable_peer_access(src.device.index, dst.device.index)
        kind = (src.dtype, dst.dtype)
        for (so, do, size, ss, ds, cnt) in chunks:
          by_kind.setdefault(kind, []).append((src, dst, so, do, size, ss, ds, cnt))
      if device is None:
        continue
      s = stream if stream is not None else torch.cuda.current_stream(device)
      for (sd, dd), chunk_list in by_kind.items():
        if engine == "copy":
          prog = ops.ReshardCopyEngineProgram(chunk_list, sd, dd, device)
        elif engine == "sm":
          prog = ops.ReshardProgram(chunk_list, sd, dd, device)
        else:
          raise ValueError(f"engine must be 'sm' or 'copy', got {engine!r}")
        prog.launch(s)
        programs.append(prog)
      ev = torch.cuda.Event()
      ev.record(s)
      last_event = ev
    if last_event is None:
      last_event = torch.cuda.Event()
      last_event.record()
    return PushFuture(last_event, programs)


  # -- controller-made byte schedules ------------------------------------------
  def _native_wsync(self):
    """The native synchronizer over this object's [layer][shard] buffers."""
    if self._wsync is None:
      L, S = self.num_layers, self.num_shards
      bufs = (_native.WsyncBuffer * (L * S))()
      for l, layer in enumerate(self._grid):
        for s, t in enumerate(layer):
          b = bufs[l * S + s]
          b.dev_ptr, b.nbytes, b.device = t.data_ptr(), t.numel() * t.element_size(), \
              t.device.index
      names = (ctypes.c_char_p * L)(*[n.encode() for n in self.layer_names])
      h = ctypes.c_void_p()
      _native.check(_native.lib().ts_wsync_create(bufs, L, S, names, ctypes.byref(h)),
                    "weight synchronizer: ")
      self._wsync = h
    return self._wsync

  def push_weights_resharded_entries(
      self, shard_push_schedules: Dict[int, Sequence[Dict[str, Any]]],
      destinations: Dict[Tuple[str, int, int], Any], src_data_name: Optional[str] = None,
      stream: Optional[torch.cuda.Stream] = None) -> "EntriesPushFuture":
    """PushWeightsResharded for a schedule made by the controller
    (StartTransferRequest.shard_push_schedules; weight_synchronizer_base.cc:558-760),
    executed by the native synchronizer (ts_wsync_register_plan / ts_wsync_push).

    shard_push_schedules: local shard index -> entries, each a dict with the
      ShardPushEntryProto fields dst_peer, dst_shard_idx, src_offset_bytes,
      dst_offset_bytes, size_bytes, src_stride_bytes, dst_stride_bytes,
      count and, optionally, layer_idx (absent: the layer whose name is
      `src_data_name`, the request's first source unit's data name).
    destinations: (dst_peer, layer_idx, dst_shard_idx) -> the tensor (or
      PeerBuffer) of that destination layer and shard; entry offsets are bytes
      into it.  The bytes move unchanged (the reference's push), every entry
      with `count` repeats as one strided task of one kernel per source GPU.

    The native checks keep the reference's order and words: ValueError for
    "Layer index out of bounds: <i>", "Push range out of bounds" (source
    range per contiguous payload or per repeat), "src_units list cannot be
    empty", and this build's destination checks ("No destination for ...",
    "Push destination range out of bounds"); LookupError for "Layer name not
    found in WeightSynchronizer: <name>".  Zero-byte entries and empty
    schedules push nothing.  A later call waits for this push before it
    replaces the plan.
    """
    entries, keep = [], []
    for i, lst in shard_push_schedules.items():
      for e in lst or ():
        peer = str(e["dst_peer"]).encode()
        keep.append(peer)
        layer = e.get("layer_idx")
        entries.append(_native.ShardPushEntry(
            src_shard_idx=int(i), has_layer_idx=int(layer is not None),
            layer_idx=int(layer) if layer is not None else 0, dst_peer=peer,
            dst_shard_idx=int(e.get("dst_shard_idx", 0)),
            src_offset_bytes=int(e.get("src_offset_bytes", 0)),
            dst_offset_bytes=int(e.get("dst_offset_bytes", 0)),
            size_bytes=int(e.get("size_bytes", 0)),
            src_stride_bytes=int(e.get("src_stride_bytes", 0)),
            dst_stride_bytes=int(e.get("dst_stride_bytes", 0)),
            count=int(e.get("count", 1))))
    dests = []
    for (peer, layer, shard), t in destinations.items():
      pb = str(peer).encode()
      keep.append(pb)
      if isinstance(t, torch.Tensor):
        nbytes, device = t.numel() * t.element_size(), t.device.index
      else:  # PeerBuffer: an IPC mapping already opened for the source device
        nbytes, device = int(t.nbytes), -1
      dests.append(_native.WsyncDest(peer=pb, layer_idx=int(layer), dst_shard_idx=int(shard),
                                     dst_ptr=t.data_ptr(), nbytes=nbytes, device=device))
    e_arr = (_native.ShardPushEntry * max(len(entries), 1))(*entries)
    d_arr = (_native.WsyncDest * max(len(dests), 1))(*dests)
    w = self._native_wsync()
    name = src_data_name.encode() if src_data_name is not None else None
    rc = _native.lib().ts_wsync_register_plan(w, e_arr, len(entries), name, d_arr, len(dests))
    if rc != _native.OK:
      msg = _native.last_error()
      if rc == _native.NOT_FOUND:
        raise LookupError(msg)
      if rc == _native.INVALID_ARGUMENT:
        raise ValueError(msg)
      raise RuntimeError(msg)
    s = stream if stream is not None else torch.cuda.current_stream(self._grid[0][0].device)
    _native.check(_native.lib().ts_wsync_push(w, ctypes.c_void_p(s.cuda_stream)),
                  "weight push: ")
    del keep
    return EntriesPushFuture(w)


class EntriesPushFuture:
  """Completion of a push of the native synchronizer (its latest push)."""

  def __init__(self, wsync):
    self._w = wsync

  def is_ready(self) -> bool:
    rc = _native.lib().ts_wsync_query(self._w)
    if rc not in (_native.OK, _native.PENDING):
      raise RuntimeError(_native.last_error())
    return rc == _native.OK

  def Await(self, timeout_ms: int = -1) -> None:
    _native.check(_native.lib().ts_wsync_wait(self._w, int(timeout_ms)), "weight push: ")

  wait = Await

  def stream_wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
    s = stream or torch.cuda.current_stream()
    _native.check(_native.lib().ts_wsync_stream_wait(self._w, ctypes.c_void_p(s.cuda_stream)),
                  "weight push: ")


class PeerBuffer:
  """Another process's device memory, mapped for kernels on `kernel_device`.

  Exposes what the reshard path reads from a destination: data_ptr(),
  device (the GPU that holds the memory), dtype and shape.
  """

  def __init__(self, ptr: int, device_index: int, dtype: torch.dtype, shape):
    self._ptr = ptr
    self.device = torch.device("cuda", device_index)
    self.dtype = dtype
    self.shape = tuple(shape)

  def data_ptr(self) -> int:
    return self._ptr

  @property
  def nbytes(self) -> int:
    n = 1
    for d in self.shape:
      n *= int(d)
    return n * torch.empty((), dtype=self.dtype).element_size()


# (kernel device, handle bytes) -> mapped base address; a handle may be opened
# once per device per process, and several tensors can share one allocation.
_IPC_BASES: Dict[Tuple[int, bytes], int] = {}


def export_destinations(dest: Dict[Any, torch.Tensor]) -> Dict:
  """Picklable CUDA-IPC descriptors of destination tensors (sampler side).

  Each descriptor is (device, 64-byte cudaIpcMemHandle of the allocation,
  byte offset, dtype, shape).  The tensors must stay alive until every
  importer has finished with them.
  """
  out = {}
  for k, t in dest.items():
    if not t.is_cuda or not t.is_contiguous():
      raise ValueError("destinations must be contiguous CUDA tensors")
    handle = ctypes.create_string_buffer(64)
    offset = ctypes.c_uint64()
    _native.check(_native.lib().ts_ipc_export(ctypes.c_void_p(t.data_ptr()), handle,
                                              ctypes.byref(offset)), "ipc export: ")
    out[k] = (t.device.index, handle.raw, int(offset.value), t.dtype, tuple(t.shape))
  return out


def import_destinations(desc: Dict, kernel_device: Optional[int] = None) -> Dict[Any, PeerBuffer]:
  """Maps exported destinations for kernels on `kernel_device` (trainer side).

  The IPC handle is opened with the kernel's device current (lazy peer
  access), which is what lets that device's kernels store into the peer's
  memory; a mapping opened under the peer's own device would not be visible
  to them.
  """
  dev = torch.cuda.current_device() if kernel_device is None else int(kernel_device)
  out = {}
  for k, (peer_dev, handle, offset, dtype, shape) in desc.items():
    key = (dev, handle)
    if key not in _IPC_BASES:
      base = ctypes.c_void_p()
      _native.check(_native.lib().ts_ipc_open(dev, handle, ctypes.byref(base)), "ipc open: ")
      _IPC_BASES[key] = base.value
    out[k] = PeerBuffer(_IPC_BASES[key] + offset, peer_dev, dtype, shape)
  return out


def close_imports(kernel_device: Optional[int] = None) -> None:
  """Unmaps every destination imported for `kernel_device` (all if None)."""
  for (dev, handle), base in list(_IPC_BASES.items()):
    if kernel_device is None or dev == kernel_device:
      _native.lib().ts_ipc_close(dev, ctypes.c_void_p(base))
      del _IPC_BASES[(dev, handle)]

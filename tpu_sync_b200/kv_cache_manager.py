"""KVCacheManager / RaidenFuture over the B200 C ABI.

Mirrors the reference's torch surface (tpu_sync/api/torch/kv_cache_manager.py:55-448
and the nanobind binding tpu_sync/frameworks/torch/tpu_raiden_torch_module.cc:179-496):
same class names, method names, argument meaning, block-unit offsets, the
``copy_sizes=[1]*n`` default, RuntimeError messages prefixed
"KVCacheManager D2h failed: " / "KVCacheManager H2d failed: " and futures
whose ``Await()`` raises "Async copy failed: ...".

Data enters as torch CUDA tensors: each (layer, shard) storage is a contiguous
CUDA tensor whose dim 0 indexes blocks.  The manager owns a pinned host tier
of ``host_blocks_to_allocate`` blocks (block-major: host block h holds block
h of every storage contiguously).

Transfer modes, chosen per direction: "staged" gathers blocks into an HBM
staging slot with the extract kernel and moves them with copy-engine DMAs on
`copy_streams` streams per direction (and the reverse for reload); "direct"
lets the extract / insert kernels read and write the mapped pinned host tier
over PCIe themselves (`max_ctas` caps their grid so most SMs stay free);
"direct_d2h" / "direct_h2d" use direct for one direction only.

The control-plane arguments of the reference constructor (ports, controller
address, worker id, staging slots for the TCP hand-off) are accepted for
signature compatibility and have no effect: there is no network path here.
"""

from __future__ import annotations

import ctypes
import os
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from tpu_sync_b200 import _native


def _stream(stream: Optional["torch.cuda.Stream"], device) -> ctypes.c_void_p:
  s = stream if stream is not None else torch.cuda.current_stream(device)
  return ctypes.c_void_p(s.cuda_stream)


def _numa_opt(numa_node) -> int:
  """ts_manager_opts.numa_node from the Python argument: None = the device's
  own node (the reference's detection), an int n >= 0 = node n (its
  assigned_numa_node_override), "none" = no placement."""
  if numa_node is None:
    return 0
  if isinstance(numa_node, str):
    if numa_node != "none":
      raise ValueError(f"numa_node must be None, a node number or 'none', got {numa_node!r}")
    return -1
  if int(numa_node) < 0:
    raise ValueError(f"numa_node must be >= 0, got {numa_node}")
  return int(numa_node) + 1


def _storage_grid(kv_caches) -> List[List[torch.Tensor]]:
  if isinstance(kv_caches, torch.Tensor):
    raise TypeError("kv_caches must be a list of tensors or a list of lists")
  grid = []
  for layer in kv_caches:
    if isinstance(layer, torch.Tensor):
      grid.append([layer])
    else:
      grid.append(list(layer))
  if not grid or not grid[0]:
    raise ValueError("kv_caches must hold at least one storage")
  nshards = len(grid[0])
  for layer in grid:
    if len(layer) != nshards:
      raise RuntimeError("Number of shards mismatch across layers")
    for t in layer:
      if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("every storage must be a CUDA tensor")
      if not t.is_contiguous():
        raise ValueError("every storage must be contiguous")
      if t.dim() == 0:
        raise ValueError("storages need a block dimension (dim 0)")
  return grid


class RaidenFuture:
  """Completion handle of one transfer (reference RaidenFuture)."""

  def __init__(self, handle: int, keepalive: Any = None):
    self._handle = ctypes.c_void_p(handle)
    self._keepalive = keepalive

  def _h(self):
    if not self._handle:
      raise RuntimeError("future already released")
    return self._handle

  def Await(self, timeout_s: Optional[float] = None) -> None:
    timeout_ms = -1 if timeout_s is None else int(timeout_s * 1000)
    rc = _native.lib().ts_event_wait(self._h(), timeout_ms)
    if rc != _native.OK:
      raise RuntimeError("Async copy failed: " + _native.last_error())

  wait = Await

  def IsReady(self) -> bool:
    return _native.lib().ts_event_query(self._h()) != _native.PENDING

  is_ready = IsReady

  def ok(self) -> bool:
    rc = _native.lib().ts_event_query(self._h())
    return rc in (_native.OK, _native.PENDING)

  def error_message(self) -> str:
    rc = _native.lib().ts_event_query(self._h())
    if rc in (_native.OK, _native.PENDING):
      return ""
    buf = ctypes.create_string_buffer(1024)
    _native.lib().ts_event_error(self._h(), buf, 1024)
    return buf.value.decode()

  def stream_wait(self, stream: Optional[torch.cuda.Stream] = None) -> None:
    """Makes `stream` (default: current) wait for the transfer on the device."""
    s = stream if stream is not None else torch.cuda.current_stream()
    _native.check(_native.lib().ts_event_stream_wait(self._h(), ctypes.c_void_p(s.cuda_stream)))

  def elapsed_ms(self) -> float:
    """Device time from the transfer's first queued operation to its end."""
    self.Await()
    ms = ctypes.c_float()
    _native.check(_native.lib().ts_event_elapsed_ms(self._h(), ctypes.byref(ms)))
    return float(ms.value)

  def release(self) -> None:
    if self._handle:
      _native.lib().ts_event_release(self._handle)
      self._handle = ctypes.c_void_p(0)
      self._keepalive = None

  def __del__(self):
    try:
      self.release()
    except Exception:  # interpreter shutdown
      pass


class KVCacheManager:
  """Paged KV block offload / reload between HBM and a pinned host tier."""

  def __init__(
      self,
      kv_caches: List[Any],
      local_control_port: int = 0,
      max_blocks: Optional[int] = None,
      num_slots: Optional[int] = None,
      timeout_s: float = 120.0,
      unsafe_skip_buffer_lock: bool = True,
      host_blocks_to_allocate: Optional[int] = None,
      parallelism: int = 4,
      node_id: int = 0,
      listener_port: Optional[int] = None,
      raiden_worker_port: int = 0,
      raiden_controller_address: Optional[str] = None,
      worker_id: Optional[str] = None,
      *,
      shm_name: str = "",
      model_uid: str = "",
      fp8: bool = False,
      chunk_blocks: int = 0,
      mode: str = "staged",
      copy_streams: int = 2,
      max_ctas: int = 0,
      reload_staged_every: int = 0,
      sched: Sequence[str] = (),
      numa_node: Any = None,
  ):
    if host_blocks_to_allocate is None:
      if max_blocks is None or num_slots is None:
        raise ValueError(
            "Must specify either (max_blocks, num_slots) or"
            " host_blocks_to_allocate.")
      host_blocks_to_allocate = int(max_blocks) * int(num_slots)
    grid = _storage_grid(kv_caches)
    self._grid = grid
    self._node_id = node_id
    self._timeout_s = timeout_s
    self.num_layers = len(grid)
    self.num_shards = len(grid[0])
    descs = (_native.StorageDesc * (self.num_layers * self.num_shards))()
    i = 0
    for layer in grid:
      for t in layer:
        descs[i].dev_ptr = t.data_ptr()
        descs[i].nbytes = t.numel() * t.element_size()
        descs[i].dim0 = t.shape[0]
        descs[i].device = t.device.index
        i += 1
    if not shm_name and os.environ.get("RAIDEN_SHM_KEY"):
      # CreateHostMemoryAllocator / SharedMemoryHostMemoryAllocator
      # (tpu_sync/core/utils.h:48-75, core/host_memory_allocator.cc:255-280):
      # the host tier lives in /dev/shm as RAIDEN_SHM_KEY [+ "_" +
      # RAIDEN_SHM_SERVER_NAME] + "_dev_<device>", validated against
      # RAIDEN_SHM_MODEL_UID (default "default_model") on a warm restart.
      shm_name = os.environ["RAIDEN_SHM_KEY"]
      server = os.environ.get("RAIDEN_SHM_SERVER_NAME", "")
      if server:
        shm_name += "_" + server
      shm_name += f"_dev_{grid[0][0].device.index}"
      if not model_uid:
        model_uid = os.environ.get("RAIDEN_SHM_MODEL_UID", "default_model")
    modes = {"staged": 0, "direct_d2h": 1, "direct_h2d": 2, "direct": 3}
    if mode not in modes:
      raise ValueError(f"mode must be one of {sorted(modes)}")
    flags = {"offload_priority": _native.SCHED_OFFLOAD_PRIORITY,
             "reload_per_piece": _native.SCHED_RELOAD_PER_PIECE,
             "reload_overlap": _native.SCHED_RELOAD_OVERLAP,
             "bulk_copy": _native.SCHED_BULK_COPY,
             "wide_loads": _native.SCHED_WIDE_LOADS}
    if isinstance(sched, str):
      sched = (sched,)
    unknown = [f for f in sched if f not in flags]
    if unknown:
      raise ValueError(f"sched flags must be among {sorted(flags)}, got {unknown}")
    opts = _native.ManagerOpts(
        host_blocks=int(host_blocks_to_allocate), chunk_blocks=int(chunk_blocks),
        shm_name=shm_name.encode(), model_uid=model_uid.encode(), fp8=int(fp8),
        mode=modes[mode], copy_streams=int(copy_streams),
        max_ctas=int(max_ctas), reload_staged_every=int(reload_staged_every),
        sched=sum(flags[f] for f in set(sched)), numa_node=_numa_opt(numa_node))
    handle = ctypes.c_void_p()
    rc = _native.lib().ts_mgr_create(descs, self.num_layers, self.num_shards,
                                     ctypes.byref(opts), ctypes.byref(handle))
    if rc != _native.OK:
      raise RuntimeError(_native.last_error())
    self._mgr = handle
    self.device = grid[0][0].device
    hb, pitch, major, bpb = (ctypes.c_int64(), ctypes.c_uint64(), ctypes.c_int64(),
                             ctypes.c_uint64())
    _native.check(_native.lib().ts_mgr_info(self._mgr, ctypes.byref(hb),
                                            ctypes.byref(pitch), ctypes.byref(major),
                                            ctypes.byref(bpb)))
    self.host_blocks = hb.value
    self.host_block_pitch = pitch.value
    self.major_dim = major.value
    self.bytes_per_block = bpb.value
    self.slice_byte_size = bpb.value
    self.fp8 = fp8

  # -- reference properties ------------------------------------------------
  @property
  def node_id(self) -> int:
    return self._node_id

  @property
  def assigned_numa_node(self) -> Optional[int]:
    """The NUMA node assigned to this manager (RaidenManagerBase::
    assigned_numa_node, raiden_manager_base.h:102): the device's own unless
    `numa_node` overrode it; None when unknown."""
    node, _ = self._numa()
    return None if node < 0 else node

  @property
  def host_tier_numa_placed(self) -> bool:
    """Whether the host tier's pages were placed on the assigned node
    (False on single-node hosts, or when the kernel refused the policy)."""
    return self._numa()[1]

  def _numa(self):
    node, placed = ctypes.c_int(), ctypes.c_int()
    _native.check(_native.lib().ts_mgr_numa_node(self._mgr, ctypes.byref(node),
                                                  ctypes.byref(placed)))
    return node.value, bool(placed.value)

  @property
  def local_port(self) -> Optional[int]:
    return None

  @property
  def local_control_port(self) -> int:
    return 0

  @property
  def raiden_worker_port(self) -> int:
    return 0

  @property
  def transfer_address(self) -> str:
    """The block hand-off endpoint of this manager ("ipc:<name>")."""
    return self.get_local_endpoints()[0]["endpoint"]

  @property
  def listener_address(self) -> str:
    return ""

  @property
  def listener_port(self) -> Optional[int]:
    return None

  @property
  def is_listener_active(self) -> bool:
    return False

  def close(self) -> None:
    for attr, fn in (("_xfer_reader", "ts_xfer_reader_destroy"),
                     ("_xfer_ep", "ts_xfer_endpoint_destroy")):
      h = getattr(self, attr, None)
      if h:
        getattr(_native.lib(), fn)(h)
        setattr(self, attr, None)
    if getattr(self, "_mgr", None):
      _native.lib().ts_mgr_destroy(self._mgr)
      self._mgr = None

  # -- block hand-off between managers (pull protocol) ----------------------
  # The reference's notify_for_read / start_read / complete_read
  # (api/torch/kv_cache_manager.py:172-175, :334-396;
  # core/kv_cache_manager_with_transfer.cc:624-665, :1478-1760) over a
  # /dev/shm mailbox, CUDA IPC and an NVLink copy kernel instead of TCP; the
  # endpoint descriptors of get_local_endpoints() are what a peer passes to
  # start_read().

  def _endpoint(self):
    if getattr(self, "_xfer_ep", None) is None:
      name = f"tsb_xfer_{os.getpid()}_{self._node_id}_{id(self) & 0xffffffff:x}"
      h = ctypes.c_void_p()
      max_blocks = int(min(self.major_dim, 1 << 16))
      _native.check(_native.lib().ts_xfer_endpoint_create(
          self._mgr, name.encode(), 64, max_blocks, int(self._timeout_s * 1000),
          ctypes.byref(h)), "transfer endpoint: ")
      self._xfer_ep = h
    return self._xfer_ep

  def _reader(self):
    if getattr(self, "_xfer_reader", None) is None:
      h = ctypes.c_void_p()
      _native.check(_native.lib().ts_xfer_reader_create(
          self._mgr, int(self._timeout_s * 1000), ctypes.byref(h)), "transfer reader: ")
      self._xfer_reader = h
    return self._xfer_reader

  def get_local_endpoints(self) -> List[Dict[str, Any]]:
    """[{"endpoint": "ipc:<mailbox>", "shards": [...]}] for peers' start_read."""
    buf = ctypes.create_string_buffer(256)
    _native.check(_native.lib().ts_xfer_endpoint_name(self._endpoint(), buf, 256))
    return [{"endpoint": "ipc:" + buf.value.decode(), "shards": list(range(self.num_shards))}]

  def register_read(self, req_id: str, uuid: int, block_ids: List[int],
                    stream: Optional[torch.cuda.Stream] = None) -> bool:
    """Producer: the blocks may be read once the work queued so far on
    `stream` (default: the current stream) is done.  True if a transfer is
    needed, False for an empty list."""
    ids = _native.i64_array(block_ids)
    reg = ctypes.c_int()
    _native.check(_native.lib().ts_xfer_register_read(
        self._endpoint(), req_id.encode(), int(uuid), _native.i64_ptr(ids), ids.size,
        _stream(stream, self.device), ctypes.byref(reg)), "register_read: ")
    return bool(reg.value)

  READ_STATES = {0: "none", 2: "registered", 3: "ready", 4: "reading", 5: "consumed",
                 6: "failed"}

  def read_state(self, uuid: int) -> str:
    """Producer: where read `uuid` stands ("ready" = its blocks are written
    and a consumer may pull them)."""
    st = ctypes.c_int()
    _native.check(_native.lib().ts_xfer_read_state(self._endpoint(), int(uuid),
                                                   ctypes.byref(st)))
    return self.READ_STATES.get(st.value, str(st.value))

  # -- reference entry points with no counterpart on one node -----------------
  @classmethod
  def create_host_only_for_testing(cls, *, num_layers: int, num_shards: int = 1,
                                   slice_byte_size: int, node_id: int,
                                   local_port: Optional[int] = None, host_blocks: int,
                                   parallelism: int = 4) -> "KVCacheManager":
    """The reference's CPU-only manager over host memory
    (tpu_sync/api/torch/kv_cache_manager.py:137-160).  Blocks live in HBM
    here and nothing runs on a CPU path, so there is none: CPU tests use the
    oracle's byte model of the manager."""
    raise NotImplementedError(
        "create_host_only_for_testing: this build has no host-only manager (blocks live "
        "in HBM); construct KVCacheManager over device tensors")

  def register_active_plan(self, uuid: int, request, is_sender: bool) -> None:
    """Registers a serialized StartTransferRequest for a strided TCP push in
    the reference (tpu_sync/api/torch/kv_cache_manager.py:196-204).  The TCP
    transport is not part of this build: on one node a planned hand-off runs
    as a PoolReshardProgram or push_weights_resharded_entries over NVLink."""
    raise NotImplementedError(
        "register_active_plan: strided TCP push plans are not supported; use "
        "pool_reshard.PoolReshardProgram or WeightSynchronizer.push_weights_resharded_entries")

  def unregister_active_plan(self, uuid: int) -> None:
    """See register_active_plan (tpu_sync/api/torch/kv_cache_manager.py:206-208)."""
    raise NotImplementedError("unregister_active_plan: strided TCP push plans are not supported")

  def push_registered_plan(self, uuid: int, peer: str, src_block_ids: Sequence[int],
                           dst_block_ids: Sequence[int], layer_idx: int = -1,
                           parallelism: int = 1) -> None:
    """See register_active_plan (tpu_sync/api/torch/kv_cache_manager.py:210-227)."""
    raise NotImplementedError(
        "push_registered_plan: strided TCP push plans are not supported; use "
        "pool_reshard.PoolReshardProgram or WeightSynchronizer.push_weights_resharded_entries")

  def register_recv(self, uuid: int, req_id: str, expected_block_count: int) -> None:
    """Receivers need no staging here: a pool reshard program stores
    straight into this manager's HBM (PoolReshardProgram), so there is
    nothing to arm."""
    if expected_block_count < 0:
      raise ValueError("expected_block_count must be >= 0")

  def start_read(self, req_id: str, uuid: int, remote_endpoint, remote_block_ids: List[int],
                 local_block_ids: List[int], parallelism: int = 1,
                 stream: Optional[torch.cuda.Stream] = None) -> int:
    """Consumer: pulls remote_block_ids of the producer at `remote_endpoint`
    (its endpoint string, or its get_local_endpoints() list) into
    local_block_ids, queued on `stream` behind the producer's registration.
    Completion is reported by poll_stats()."""
    if isinstance(remote_endpoint, (list, tuple)):
      if not remote_endpoint:
        return 0
      remote_endpoint = remote_endpoint[0]["endpoint"]
    r = _native.i64_array(remote_block_ids)
    l = _native.i64_array(local_block_ids)
    if r.size != l.size:
      raise ValueError("remote_block_ids and local_block_ids must have the same length")
    _native.check(_native.lib().ts_xfer_start_read(
        self._reader(), req_id.encode(), int(uuid), str(remote_endpoint).encode(),
        _native.i64_ptr(r), _native.i64_ptr(l), r.size, _stream(stream, self.device)),
        "start_read: ")
    return 0

  def _poll_list(self, fn, handle, *lead) -> List[str]:
    n, need = ctypes.c_int64(), ctypes.c_int64()
    cap_b, cap_n = 4096, 64
    while True:
      buf = ctypes.create_string_buffer(cap_b)
      offs = np.zeros(cap_n + 1, np.int64)
      rc = fn(handle, *lead, buf, cap_b, offs.ctypes.data_as(_native.c_i64_p), cap_n + 1,
              ctypes.byref(n), ctypes.byref(need))
      if rc == _native.OK:
        raw = buf.raw
        return [raw[offs[i]:offs[i + 1]].decode() for i in range(n.value)]
      if rc != _native.RESOURCE_EXHAUSTED:
        _native.check(rc, "poll_stats: ")
      cap_b, cap_n = max(cap_b, need.value), max(cap_n, n.value)

  def poll_stats(self) -> Tuple[List[str], List[str], List[str]]:
    """(done_sending, done_recving, failed_recving) request ids."""
    lib = _native.lib()
    sends = (self._poll_list(lib.ts_xfer_poll_sends, self._xfer_ep)
             if getattr(self, "_xfer_ep", None) else [])
    done, failed = [], []
    if getattr(self, "_xfer_reader", None):
      done = self._poll_list(lib.ts_xfer_poll_reads, self._xfer_reader, 0)
      failed = self._poll_list(lib.ts_xfer_poll_reads, self._xfer_reader, 1)
    return sends, done, failed

  def __del__(self):
    try:
      self.close()
    except Exception:
      pass

  # -- transfers -----------------------------------------------------------
  def _transfer(self, fn, what, src_offsets, dst_offsets, copy_sizes, layer_idx,
                shard_idx, stream):
    if copy_sizes is None:
      copy_sizes = [1] * len(src_offsets)
    src = _native.i64_array(src_offsets)
    dst = _native.i64_array(dst_offsets)
    sizes = _native.i64_array(copy_sizes)
    if stream is None:
      stream = torch.cuda.current_stream(self.device)
    ev = ctypes.c_void_p()
    rc = fn(self._mgr, _native.i64_ptr(src), _native.i64_ptr(dst),
            _native.i64_ptr(sizes), src.size, dst.size, sizes.size,
            -1 if layer_idx is None else int(layer_idx),
            -1 if shard_idx is None else int(shard_idx),
            ctypes.c_void_p(stream.cuda_stream), ctypes.byref(ev))
    if rc != _native.OK:
      raise RuntimeError(f"KVCacheManager {what} failed: " + _native.last_error())
    return RaidenFuture(ev.value, keepalive=self)

  def d2h(self, src_offsets: List[int], dst_offsets: List[int],
          copy_sizes: Optional[List[int]] = None, *, layer_idx: Optional[int] = None,
          shard_idx: Optional[int] = None,
          stream: Optional[torch.cuda.Stream] = None) -> RaidenFuture:
    """Device-to-host copy of blocks (block units); returns a future."""
    return self._transfer(_native.lib().ts_d2h, "D2h", src_offsets, dst_offsets,
                          copy_sizes, layer_idx, shard_idx, stream)

  def h2d(self, src_offsets: List[int], dst_offsets: List[int],
          copy_sizes: Optional[List[int]] = None, *, layer_idx: Optional[int] = None,
          shard_idx: Optional[int] = None,
          stream: Optional[torch.cuda.Stream] = None) -> RaidenFuture:
    """Host-to-device copy of blocks (block units); returns a future."""
    return self._transfer(_native.lib().ts_h2d, "H2d", src_offsets, dst_offsets,
                          copy_sizes, layer_idx, shard_idx, stream)

  # nanobind-style spellings of the reference binding
  def D2h(self, src_offsets_major_dim=(), dst_offsets_major_dim=(),
          copy_sizes_major_dim=()):
    return self._transfer(_native.lib().ts_d2h, "D2h", list(src_offsets_major_dim),
                          list(dst_offsets_major_dim), list(copy_sizes_major_dim),
                          None, None, None)

  def H2d(self, src_offsets_major_dim=(), dst_offsets_major_dim=(),
          copy_sizes_major_dim=()):
    return self._transfer(_native.lib().ts_h2d, "H2d", list(src_offsets_major_dim),
                          list(dst_offsets_major_dim), list(copy_sizes_major_dim),
                          None, None, None)

  # -- kernel timing -------------------------------------------------------
  def set_profiling(self, on: bool = True) -> None:
    """Times every extract / insert kernel launch with CUDA events."""
    _native.check(_native.lib().ts_mgr_set_profiling(self._mgr, int(bool(on))))

  def kernel_stats(self, which: str = "extract") -> Dict[str, float]:
    """Launches, summed device ms and algorithmic bytes since the last call."""
    n, ms, b = ctypes.c_int64(), ctypes.c_double(), ctypes.c_uint64()
    _native.check(_native.lib().ts_mgr_kernel_stats(
        self._mgr, 0 if which == "extract" else 1, ctypes.byref(n), ctypes.byref(ms),
        ctypes.byref(b)))
    return {"launches": n.value, "ms": ms.value, "bytes": b.value}

  # -- host tier access ----------------------------------------------------
  def _host_block(self, layer_idx: int, block_id: int, shard_idx: int = 0):
    ptr, nbytes = ctypes.c_uint64(), ctypes.c_uint64()
    rc = _native.lib().ts_mgr_host_block_ptr(self._mgr, int(layer_idx), int(shard_idx),
                                             int(block_id), ctypes.byref(ptr),
                                             ctypes.byref(nbytes))
    return rc, ptr.value, nbytes.value

  def read_block_bytes(self, layer_idx: int, block_id: int, shard_idx: int = 0) -> bytes:
    """Returns one host block of one storage as bytes."""
    rc, ptr, nbytes = self._host_block(layer_idx, block_id, shard_idx)
    if rc != _native.OK:
      raise RuntimeError("KVCacheManager read_block_bytes failed: " + _native.last_error())
    return ctypes.string_at(ptr, nbytes)

  def write_block_bytes(self, layer_idx: int, block_id: int, payload: bytes,
                        shard_idx: int = 0) -> None:
    """Overwrites one host block of one storage with bytes."""
    rc, ptr, nbytes = self._host_block(layer_idx, block_id, shard_idx)
    if rc != _native.OK:
      raise RuntimeError("KVCacheManager write_block_bytes failed: " + _native.last_error())
    if len(payload) > nbytes:
      raise RuntimeError("KVCacheManager write_block_bytes failed: payload exceeds block size")
    ctypes.memmove(ptr, payload, len(payload))

  def host_tier_view(self) -> np.ndarray:
    """Zero-copy uint8 view [host_blocks, host_block_pitch] of the host tier."""
    rc, ptr, _ = self._host_block(0, 0, 0)
    _native.check(rc)
    buf = (ctypes.c_uint8 * (self.host_blocks * self.host_block_pitch)).from_address(ptr)
    return np.frombuffer(buf, dtype=np.uint8).reshape(self.host_blocks, self.host_block_pitch)

  def block_bytes(self, layer_idx: int) -> int:
    t = self._grid[layer_idx][0]
    return t.numel() * t.element_size() // self.major_dim

  # -- pools (RegisterPools / CopyPoolBlocks) -------------------------------
  def register_pools(self, pools: Sequence[Any]) -> Dict[str, Any]:
    """Registers explicit block pools over the wrapped storages.

    ``pools``: PoolSpec objects or equivalent mappings, in the caller's
    canonical order (pool indices are positions in it).  Returns the admission
    summary (tpu_sync/api/torch/kv_cache_manager.py:239-283).
    """
    from tpu_sync_b200 import pool_layout
    coerced = tuple(pool_layout.coerce_pool_spec(p) for p in pools)
    if not coerced:
      raise ValueError("pool table must be non-empty")
    for i, p in enumerate(coerced):
      try:
        p.validate()
      except ValueError as exc:
        raise ValueError(f"invalid pool {i}: {exc}") from exc
      if p.storage_index >= self.num_layers:
        raise ValueError(f"pool {i} ({p.tag}) storage_index {p.storage_index} out of range: "
                         f"manager wraps {self.num_layers} storages")
    arr, keep = pool_layout.pools_c(coerced)
    rc = _native.lib().ts_mgr_register_pools(self._mgr, arr, len(coerced))
    del keep
    if rc != _native.OK:
      raise RuntimeError("KVCacheManager register_pools failed: " + _native.last_error())
    self._pools = coerced
    tags: Dict[str, int] = {}
    for p in coerced:
      tags[p.tag] = tags.get(p.tag, 0) + 1
    self._admission_summary = {"admitted": True, "pools": len(coerced),
                               "storages": len({p.storage_index for p in coerced}), "tags": tags}
    return dict(self._admission_summary)

  def admission_summary(self) -> Dict[str, Any]:
    summary = getattr(self, "_admission_summary", None)
    return dict(summary) if summary else {"admitted": False}

  def has_explicit_pools(self) -> bool:
    n, ex = ctypes.c_int64(), ctypes.c_int()
    _native.check(_native.lib().ts_mgr_num_pools(self._mgr, ctypes.byref(n), ctypes.byref(ex)))
    return bool(ex.value)

  def num_pools(self) -> int:
    """Pools (implicit: one per storage with positive block bytes; or explicit)."""
    n = ctypes.c_int64()
    _native.check(_native.lib().ts_mgr_num_pools(self._mgr, ctypes.byref(n), None))
    return n.value

  def pool_spec(self, pool_idx: int) -> Dict[str, Any]:
    """One pool's descriptor as a dict (implicit pools: tag "opaque", region "block")."""
    if getattr(self, "_pools", None) is not None:
      if not 0 <= pool_idx < len(self._pools):
        raise IndexError(f"pool index out of range: {pool_idx}")
      return self._pools[pool_idx].to_dict()
    si, stride, nb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    rc = _native.lib().ts_mgr_pool_geometry(self._mgr, int(pool_idx), ctypes.byref(si),
                                            ctypes.byref(stride), ctypes.byref(nb))
    if rc != _native.OK:
      raise IndexError(f"pool index out of range: {pool_idx}")
    bb = stride.value
    return {"tag": "opaque", "storage_index": si.value, "base_offset_bytes": 0,
            "block_stride_bytes": bb, "num_blocks": nb.value,
            "regions": [{"name": "block", "offset_bytes": 0, "stride_bytes": bb,
                         "unit_bytes": bb, "num_units": 1, "units_per_stride": 1}],
            "dtype_tag": ""}

  def pool_ids_with_tag(self, tag: str) -> List[int]:
    return [i for i in range(self.num_pools()) if self.pool_spec(i)["tag"] == tag]

  def get_block_ref(self, pool_idx: int, block_id: int, shard_idx: int = 0) -> Dict[str, Any]:
    """Host-side reference to one pool block (pointer into the host tier)."""
    ptr = ctypes.c_uint64()
    rc = _native.lib().ts_mgr_pool_block_ref(self._mgr, int(pool_idx), int(shard_idx),
                                             int(block_id), ctypes.byref(ptr))
    if rc != _native.OK:
      raise RuntimeError("KVCacheManager get_pool_block_ref failed: " + _native.last_error())
    spec = self.pool_spec(pool_idx)
    return {"ptr": ptr.value, "block_stride_bytes": spec["block_stride_bytes"],
            "tag": spec["tag"], "dtype_tag": spec.get("dtype_tag", ""), "pool_idx": pool_idx,
            "shard_idx": shard_idx, "block_id": block_id, "regions": spec["regions"]}

  def _pool_copy(self, fn, what, pool_idx, block_ids, shard_idx, stream):
    ids = _native.i64_array(list(block_ids))
    if stream is None:
      stream = torch.cuda.current_stream(self.device)
    ev = ctypes.c_void_p()
    rc = fn(self._mgr, int(pool_idx), _native.i64_ptr(ids), ids.size,
            -1 if shard_idx is None else int(shard_idx), ctypes.c_void_p(stream.cuda_stream),
            ctypes.byref(ev))
    if rc != _native.OK:
      raise RuntimeError(f"KVCacheManager {what} failed: " + _native.last_error())
    return RaidenFuture(ev.value, keepalive=self)

  def d2h_pool_blocks(self, pool_idx: int, block_ids: Sequence[int],
                      shard_idx: Optional[int] = None, *,
                      stream: Optional[torch.cuda.Stream] = None) -> RaidenFuture:
    """Partial D2H of the declared-live bytes of pool blocks into the host mirror."""
    return self._pool_copy(_native.lib().ts_d2h_pool_blocks, "d2h_pool_blocks", pool_idx,
                           block_ids, shard_idx, stream)

  def h2d_pool_blocks(self, pool_idx: int, block_ids: Sequence[int],
                      shard_idx: Optional[int] = None, *,
                      stream: Optional[torch.cuda.Stream] = None) -> RaidenFuture:
    """Partial H2D of the declared-live bytes of pool blocks from the host mirror."""
    return self._pool_copy(_native.lib().ts_h2d_pool_blocks, "h2d_pool_blocks", pool_idx,
                           block_ids, shard_idx, stream)

  def read_storage_bytes(self, layer_idx: int, offset: int, size: int,
                         shard_idx: int = 0) -> bytes:
    """Bytes [offset, offset + size) of one storage's host mirror (byte offsets
    as on the device, across host blocks)."""
    bb = self.block_bytes(layer_idx)
    out = bytearray()
    x, end = int(offset), int(offset) + int(size)
    while x < end:
      blk, inb = divmod(x, bb)
      take = min(bb - inb, end - x)
      out += self.read_block_bytes(layer_idx, blk, shard_idx)[inb:inb + take]
      x += take
    return bytes(out)

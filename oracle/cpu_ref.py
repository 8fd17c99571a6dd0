"""ctypes wrapper of oracle/liboracle_ref.so -- TEST / BASELINE INFRASTRUCTURE.

The timed CPU baseline: the reference's host copy loops restated in C
(oracle/cpu_ref.c), run on the host cores.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from oracle import build_oracle

_lib = None


def lib():
  global _lib
  if _lib is None:
    path = build_oracle.build()
    l = ctypes.CDLL(str(path))
    P = ctypes.POINTER
    l.oref_copy_runs.argtypes = [P(ctypes.c_void_p), P(ctypes.c_void_p), P(ctypes.c_uint64),
                                 ctypes.c_int, P(ctypes.c_int64), P(ctypes.c_int64),
                                 P(ctypes.c_int64), ctypes.c_int64, ctypes.c_int]
    l.oref_copy_runs.restype = ctypes.c_int
    l.oref_reshard_f32_bf16.argtypes = [ctypes.c_void_p, ctypes.c_void_p, P(ctypes.c_int64),
                                        ctypes.c_int64, ctypes.c_int]
    l.oref_reshard_f32_bf16.restype = ctypes.c_int
    _lib = l
  return _lib


def host_threads() -> int:
  try:
    return len(os.sched_getaffinity(0))
  except AttributeError:
    return os.cpu_count() or 1


def copy_runs(dst_bufs, src_bufs, block_bytes, src_ids, dst_ids, sizes, threads):
  """dst_bufs/src_bufs: lists of numpy uint8 arrays (one per storage)."""
  n = len(dst_bufs)
  D = (ctypes.c_void_p * n)(*[b.ctypes.data for b in dst_bufs])
  S = (ctypes.c_void_p * n)(*[b.ctypes.data for b in src_bufs])
  BB = (ctypes.c_uint64 * n)(*block_bytes)
  s = np.ascontiguousarray(src_ids, np.int64)
  d = np.ascontiguousarray(dst_ids, np.int64)
  z = np.ascontiguousarray(sizes, np.int64)
  P = ctypes.POINTER(ctypes.c_int64)
  lib().oref_copy_runs(D, S, BB, n, s.ctypes.data_as(P), d.ctypes.data_as(P),
                       z.ctypes.data_as(P), s.size, int(threads))


def reshard_f32_bf16(src: np.ndarray, dst_bits: np.ndarray, chunks, threads: int):
  c = np.ascontiguousarray(np.asarray(chunks, np.int64).reshape(-1, 6))
  lib().oref_reshard_f32_bf16(src.ctypes.data, dst_bits.ctypes.data,
                              c.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                              c.shape[0], int(threads))

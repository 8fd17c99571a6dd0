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
    l.oref_e4m3.argtypes = [ctypes.c_float]
    l.oref_e4m3.restype = ctypes.c_uint8
    l.oref_extract_fp8.argtypes = [P(ctypes.c_void_p), P(ctypes.c_uint64), P(ctypes.c_uint64),
                                   ctypes.c_int, P(ctypes.c_int64), ctypes.c_int64,
                                   ctypes.c_void_p, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int]
    l.oref_extract_fp8.restype = ctypes.c_int
    l.oref_relayout.argtypes = [P(ctypes.c_void_p), P(ctypes.c_void_p), ctypes.c_int, ctypes.c_int,
                                ctypes.c_uint64, ctypes.c_int64, ctypes.c_int64,
                                P(ctypes.c_int32), P(ctypes.c_int32), ctypes.c_int64,
                                ctypes.c_int64, ctypes.c_int]
    l.oref_relayout.restype = ctypes.c_int
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


def extract_fp8(storages, ids, staging, pitch, stage_offs, scale_off, threads):
  """storages: numpy uint16 [blocks, elems] per storage (bf16 bits);
  staging: numpy uint8 [n, pitch] (fp8 payloads + fp32 scales)."""
  n = len(storages)
  S = (ctypes.c_void_p * n)(*[a.ctypes.data for a in storages])
  E = (ctypes.c_uint64 * n)(*[a.shape[1] for a in storages])
  O = (ctypes.c_uint64 * n)(*[int(x) for x in stage_offs])
  i = np.ascontiguousarray(ids, np.int64)
  lib().oref_extract_fp8(S, E, O, n, i.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), i.size,
                         staging.ctypes.data, int(pitch), int(scale_off), int(threads))


def relayout(src_pages, dst_pages, heads, head_bytes, st_tok, dt_tok, src_table, dst_table,
             tokens, threads):
  """src_pages / dst_pages: numpy uint8 arrays, one per storage."""
  n = len(src_pages)
  S = (ctypes.c_void_p * n)(*[a.ctypes.data for a in src_pages])
  D = (ctypes.c_void_p * n)(*[a.ctypes.data for a in dst_pages])
  st = np.ascontiguousarray(src_table, np.int32)
  dt = np.ascontiguousarray(dst_table, np.int32)
  P32 = ctypes.POINTER(ctypes.c_int32)
  lib().oref_relayout(S, D, n, int(heads), int(head_bytes), int(st_tok), int(dt_tok),
                      st.ctypes.data_as(P32), dt.ctypes.data_as(P32), st.shape[0], int(tokens),
                      int(threads))

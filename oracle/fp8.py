"""CPU oracle for the fused bf16 <-> fp8 e4m3 KV cast -- TEST INFRASTRUCTURE ONLY.

The reference has no fp8 cast (the only e4m3 mentions are dtype tables in
tpu_sync/benchmarks/perf_core.py:36-37), so parity for this row is "unpinned
by the reference": the contract is the arithmetic written below, restated
from the OCP 8-bit floating point definition of E4M3 (1 sign, 4 exponent
bits with bias 7, 3 mantissa bits, no infinities, S.1111.111 = NaN, largest
finite 448, smallest subnormal 2^-9):

  per (block, layer, K/V) unit of bf16 values x:
    amax  = max |x| over the non-NaN values (0 if none)
    scale = amax / 448 in fp32 round-to-nearest-even, or 1 if amax == 0
    q     = e4m3_rn_satfinite(fp32(x) / scale)     (fp32 RN division)
    x'    = bf16_rn(fp32(q) * scale)               (fp32 RN product)

e4m3_rn_satfinite rounds to nearest-even and clamps magnitudes above 448 to
448 (NaN stays NaN).  The encoder here works on exact float64 arithmetic of
fp32 inputs and is cross-checked against ml_dtypes / torch in the tests.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
  return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits_rne(x: np.ndarray) -> np.ndarray:
  """fp32 -> bf16 round-to-nearest-even (NaN -> quiet NaN 0x7fc0 | sign)."""
  b = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
  rounding = 0x7FFF + ((b >> 16) & 1)
  out = ((b + rounding) >> 16).astype(np.uint16)
  nan = np.isnan(np.asarray(x, dtype=np.float32))
  if nan.any():
    out = np.where(nan, ((b >> 16) & 0x8000).astype(np.uint16) | np.uint16(0x7FC0), out)
  return out


def e4m3_encode(v: np.ndarray) -> np.ndarray:
  """fp32 values -> e4m3fn bytes, round-to-nearest-even, saturating to 448."""
  v = np.asarray(v, dtype=np.float32)
  a = np.abs(v).astype(np.float64)
  sign = np.signbit(v).astype(np.uint8) << 7
  out = np.zeros(v.shape, dtype=np.uint8)
  nan = np.isnan(v)
  a = np.where(nan, 0.0, a)
  a = np.minimum(a, E4M3_MAX)  # satfinite (also maps inf to 448)
  # quantum of the binade: normal binades [2^e, 2^(e+1)) for e >= -6 have
  # 8 steps of 2^(e-3); below 2^-6 the subnormal quantum is 2^-9.
  with np.errstate(divide="ignore"):
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
  e = np.maximum(e, -6.0)
  q = np.exp2(e - 3.0)
  r = np.rint(a / q) * q  # a/q is exact (power-of-two quantum); rint = RNE
  r = np.minimum(r, E4M3_MAX)
  # encode r
  is_zero = r == 0
  with np.errstate(divide="ignore"):
    er = np.floor(np.log2(np.where(is_zero, 1.0, r)))
  normal = (er >= -6) & ~is_zero
  exp_field = np.where(normal, er + 7, 0).astype(np.int64)
  mant = np.where(normal, r / np.exp2(er) - 1.0, r / 2.0 ** -9)
  mant_field = np.where(normal, np.rint(mant * 8), np.rint(mant)).astype(np.int64)
  bits = (exp_field << 3) | mant_field
  out = (bits.astype(np.uint8) | sign)
  out = np.where(nan, np.uint8(0x7F) | sign, out)
  return out.astype(np.uint8)


def e4m3_decode(b: np.ndarray) -> np.ndarray:
  """e4m3fn bytes -> fp32 values (exact)."""
  b = np.asarray(b, dtype=np.uint8).astype(np.int64)
  s = np.where(b & 0x80, -1.0, 1.0)
  e = (b >> 3) & 0xF
  m = b & 0x7
  val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
  val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
  return (s * val).astype(np.float32)


def unit_scale(x_f32: np.ndarray) -> np.float32:
  finite = x_f32[~np.isnan(x_f32)]
  amax = np.float32(np.max(np.abs(finite))) if finite.size else np.float32(0)
  if amax == 0:
    return np.float32(1.0)
  return np.float32(amax) / np.float32(E4M3_MAX)  # fp32 RN division


def quantize_unit(bits_bf16: np.ndarray):
  """One unit of bf16 bit patterns -> (e4m3 bytes, fp32 scale)."""
  x = bf16_bits_to_f32(bits_bf16.reshape(-1))
  scale = unit_scale(x)
  with np.errstate(invalid="ignore", divide="ignore"):
    y = (x / scale).astype(np.float32)
  return e4m3_encode(y), scale


def dequantize_unit(q: np.ndarray, scale: np.float32) -> np.ndarray:
  """e4m3 bytes + scale -> bf16 bit patterns."""
  with np.errstate(invalid="ignore", over="ignore"):
    y = (e4m3_decode(q) * np.float32(scale)).astype(np.float32)
  return f32_to_bf16_bits_rne(y)


def extract_fp8(storages_bf16_bits, ids):
  """Per block id k and storage s: (payload[k][s], scale[k][s]).

  storages_bf16_bits: uint16 arrays [num_blocks, elems_per_block].
  Returns payload uint8 [n, S, elems] and scales float32 [n, S].
  """
  n, S = len(ids), len(storages_bf16_bits)
  elems = storages_bf16_bits[0].reshape(storages_bf16_bits[0].shape[0], -1).shape[1]
  payload = np.zeros((n, S, elems), np.uint8)
  scales = np.zeros((n, S), np.float32)
  for s, st in enumerate(storages_bf16_bits):
    flat = st.reshape(st.shape[0], -1)
    for k, i in enumerate(ids):
      payload[k, s], scales[k, s] = quantize_unit(flat[int(i)])
  return payload, scales


def insert_fp8(payload, scales, ids, storages_bf16_bits) -> None:
  for s, st in enumerate(storages_bf16_bits):
    flat = st.reshape(st.shape[0], -1)
    for k, i in enumerate(ids):
      flat[int(i)] = dequantize_unit(payload[k, s], scales[k, s])

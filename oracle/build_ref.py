"""Compiles reference sources into test oracle binaries.

    python oracle/build_ref.py     # -> oracle/_ref/{lru_ref, pool_ref, meta_ref, plan_ref, bm_ref,
                                   #                 store_trace_ref}

* lru_ref: oracle/ref_lru_driver.cc over the header-only LRUCache
  (tpu_sync/kv_cache/lru_cache.h);
* pool_ref: oracle/ref_pool_driver.cc linked with tpu_sync/kv_cache/pool_layout.cc;
* meta_ref: oracle/ref_meta_driver.cc linked with tpu_sync/kv_cache/kv_cache_metadata.cc
  and kv_cache_metadata_shm.cc;
* plan_ref: oracle/ref_pool_reshard_driver.cc linked with tpu_sync/kv_cache/pool_layout.cc
  and reshard/{declaration_types, work_unit_directory, request_block_registry,
  pool_reshard_planner}.cc;
* bm_ref: oracle/ref_bm_driver.cc linked with tpu_sync/kv_cache/logical_block_manager.cc;
* store_trace_ref: oracle/ref_store_trace_driver.cc over lru_cache.h, linked with
  tpu_sync/kv_cache/logical_block_manager.cc (the C1 access trace through the
  reference's index and allocator).

g++ compiles them where they lie in the reference checkout (REFERENCE_ROOT,
else BASELINE.json's reference_path); oracle/shim stands in for the few absl types they
use (flat_hash_map, Status, StatusOr, StrCat, StrJoin, Span, string_view, LOG, Mutex,
HashOf, thread annotations) and for the proto message classes those sources name.  Nothing is copied from the reference;
the binaries go to oracle/_ref/ only.  Test infrastructure: tests/ use them to
pin the product's LRU, pool geometry, metadata table and pool reshard planner
(tests/golden/make_*_golden.py record the binaries' answers as fixtures).
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "lru_ref"


def reference_root() -> Path:
  """The reference checkout: $REFERENCE_ROOT, else BASELINE.json's reference_path."""
  env = os.environ.get("REFERENCE_ROOT")
  if env:
    return Path(env)
  try:
    import json
    return Path(json.loads((HERE.parent / "BASELINE.json").read_text())["reference_path"])
  except (OSError, KeyError, ValueError):
    return HERE / "_no_reference_checkout"


def build(force: bool = False) -> Path | None:
  """Builds the oracle if the reference checkout is present; returns its path."""
  ref = reference_root()
  header = ref / "tpu_sync" / "kv_cache" / "lru_cache.h"
  src = HERE / "ref_lru_driver.cc"
  if OUT.exists() and not force and OUT.stat().st_mtime >= src.stat().st_mtime:
    return OUT
  if not header.exists():
    return OUT if OUT.exists() else None
  OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O1", f"-I{HERE / 'shim'}", f"-I{ref}", str(src),
                  "-o", str(OUT)], check=True)
  return OUT


POOL_OUT = HERE / "_ref" / "pool_ref"


def build_pool(force: bool = False) -> Path | None:
  """Builds pool_ref if the reference checkout is present; returns its path."""
  ref = reference_root()
  cc = ref / "tpu_sync" / "kv_cache" / "pool_layout.cc"
  src = HERE / "ref_pool_driver.cc"
  if POOL_OUT.exists() and not force and POOL_OUT.stat().st_mtime >= src.stat().st_mtime:
    return POOL_OUT
  if not cc.exists():
    return POOL_OUT if POOL_OUT.exists() else None
  POOL_OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O1", f"-I{HERE / 'shim'}", f"-I{ref}", str(src), str(cc),
                  "-o", str(POOL_OUT)], check=True)
  return POOL_OUT


META_OUT = HERE / "_ref" / "meta_ref"


def build_meta(force: bool = False) -> Path | None:
  """Builds meta_ref if the reference checkout is present; returns its path."""
  ref = reference_root()
  kv = ref / "tpu_sync" / "kv_cache"
  ccs = [kv / "kv_cache_metadata.cc", kv / "kv_cache_metadata_shm.cc"]
  src = HERE / "ref_meta_driver.cc"
  if META_OUT.exists() and not force and META_OUT.stat().st_mtime >= src.stat().st_mtime:
    return META_OUT
  if not all(c.exists() for c in ccs):
    return META_OUT if META_OUT.exists() else None
  META_OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O1", f"-I{HERE / 'shim'}", f"-I{ref}", str(src),
                  *map(str, ccs), "-o", str(META_OUT)], check=True)
  return META_OUT


PLAN_OUT = HERE / "_ref" / "plan_ref"


def build_plan(force: bool = False) -> Path | None:
  """Builds plan_ref if the reference checkout is present; returns its path."""
  ref = reference_root()
  kv = ref / "tpu_sync" / "kv_cache"
  ccs = [kv / "pool_layout.cc"] + [kv / "reshard" / f"{n}.cc" for n in (
      "declaration_types", "work_unit_directory", "request_block_registry",
      "pool_reshard_planner")]
  src = HERE / "ref_pool_reshard_driver.cc"
  if PLAN_OUT.exists() and not force and PLAN_OUT.stat().st_mtime >= src.stat().st_mtime:
    return PLAN_OUT
  if not all(c.exists() for c in ccs):
    return PLAN_OUT if PLAN_OUT.exists() else None
  PLAN_OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O1", f"-I{HERE / 'shim'}", f"-I{ref}", str(src),
                  *map(str, ccs), "-o", str(PLAN_OUT)], check=True)
  return PLAN_OUT


BM_OUT = HERE / "_ref" / "bm_ref"


def build_bm(force: bool = False) -> Path | None:
  """Builds bm_ref if the reference checkout is present; returns its path."""
  ref = reference_root()
  cc = ref / "tpu_sync" / "kv_cache" / "logical_block_manager.cc"
  src = HERE / "ref_bm_driver.cc"
  if BM_OUT.exists() and not force and BM_OUT.stat().st_mtime >= src.stat().st_mtime:
    return BM_OUT
  if not cc.exists():
    return BM_OUT if BM_OUT.exists() else None
  BM_OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O1", f"-I{HERE / 'shim'}", f"-I{ref}", str(src), str(cc),
                  "-o", str(BM_OUT)], check=True)
  return BM_OUT


STORE_OUT = HERE / "_ref" / "store_trace_ref"


def build_store_trace(force: bool = False) -> Path | None:
  """Builds store_trace_ref if the reference checkout is present; returns its path."""
  ref = reference_root()
  cc = ref / "tpu_sync" / "kv_cache" / "logical_block_manager.cc"
  header = ref / "tpu_sync" / "kv_cache" / "lru_cache.h"
  src = HERE / "ref_store_trace_driver.cc"
  if STORE_OUT.exists() and not force and STORE_OUT.stat().st_mtime >= src.stat().st_mtime:
    return STORE_OUT
  if not (cc.exists() and header.exists()):
    return STORE_OUT if STORE_OUT.exists() else None
  STORE_OUT.parent.mkdir(parents=True, exist_ok=True)
  cxx = shutil.which("g++") or "c++"
  subprocess.run([cxx, "-std=c++17", "-O2", f"-I{HERE / 'shim'}", f"-I{ref}", str(src), str(cc),
                  "-o", str(STORE_OUT)], check=True)
  return STORE_OUT


if __name__ == "__main__":
  print(build(force=True))
  print(build_pool(force=True))
  print(build_meta(force=True))
  print(build_plan(force=True))
  print(build_bm(force=True))
  print(build_store_trace(force=True))

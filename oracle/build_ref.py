"""Compiles the reference's header-only LRUCache into a test oracle binary.

    python oracle/build_ref.py     # -> oracle/_ref/lru_ref

g++ builds oracle/ref_lru_driver.cc against tpu_sync/kv_cache/lru_cache.h
where it lies in the reference checkout (REFERENCE_ROOT, default
/root/reference), with oracle/shim standing in for absl's flat_hash_map.
Nothing is copied from the reference; the binary goes to oracle/_ref/ only.
Test infrastructure: tests/ use the binary to pin the product's LRU.
"""

from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "lru_ref"


def reference_root() -> Path:
  return Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))


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


if __name__ == "__main__":
  print(build(force=True))

"""Builds the native library ``tpu_sync_b200/_lib/libtpusync_b200.so``.

Every CUDA source under ``csrc/`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with nvcc and linked into one
shared library whose exported symbols are the C ABI declared in
``include/tpusync_b200.h``.  The CUDA runtime is linked statically, so the
library does not depend on which libcudart the host process (torch) loaded.

Run ``python -m tpu_sync_b200.build`` or call :func:`build`.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_DIR = PKG_DIR / "_lib"
OBJ_DIR = REPO_DIR / "_build" / "native"
LIB_NAME = "libtpusync_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xcompiler",
    "-Wall",
]


def _nvcc() -> str:
  cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
  if not Path(cand).exists():
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build")
  return cand


def _needs_build(src: Path, obj: Path, headers: list[Path]) -> bool:
  if not obj.exists():
    return True
  t = obj.stat().st_mtime
  return src.stat().st_mtime > t or any(h.stat().st_mtime > t for h in headers)


def build(verbose: bool = False, force: bool = False) -> Path:
  """Compiles (incrementally) and links the library; returns its path."""
  nvcc = _nvcc()
  OBJ_DIR.mkdir(parents=True, exist_ok=True)
  LIB_DIR.mkdir(parents=True, exist_ok=True)
  sources = sorted(CSRC.glob("*.cu"))
  headers = sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
  objs = []
  jobs = []
  for src in sources:
    obj = OBJ_DIR / (src.stem + ".o")
    objs.append(obj)
    if force or _needs_build(src, obj, headers):
      cmd = [nvcc, *ARCH_FLAGS, *CFLAGS, f"-I{INCLUDE}", f"-I{CSRC}",
             "-DTS_BUILDING_LIB", "-c", str(src), "-o", str(obj)]
      jobs.append(cmd)

  def run(cmd):
    if verbose:
      print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
      raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r

  with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
    list(ex.map(run, jobs))
  lib = LIB_DIR / LIB_NAME
  if force or jobs or not lib.exists():
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(lib),
           *[str(o) for o in objs], "-lpthread", "-lrt"]
    run(cmd)
  return lib


if __name__ == "__main__":
  path = build(verbose="-v" in sys.argv, force="-f" in sys.argv)
  print(path)

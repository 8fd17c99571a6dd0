"""Builds oracle/liboracle_ref.so from oracle/cpu_ref.c (gcc).

Test / baseline infrastructure: the library is loaded only by tests/ and by
bench.py's CPU arms (oracle/cpu_ref.py).
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "cpu_ref.c"
LIB = HERE / "liboracle_ref.so"


def build(force: bool = False) -> Path:
  if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
    return LIB
  cc = shutil.which("gcc") or "cc"
  subprocess.run([cc, "-O3", "-march=x86-64-v2", "-fPIC", "-shared", "-pthread",
                  str(SRC), "-o", str(LIB)], check=True)
  return LIB


if __name__ == "__main__":
  print(build(force=True))

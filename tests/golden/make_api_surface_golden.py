"""Generates tests/golden/api_surface.json: the reference's Python surface.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_api_surface_golden.py

Reads (as text, with Python's ast parser; nothing is imported or run) the
classes a caller of the reference's torch API uses --
tpu_sync/api/torch/{kv_cache_manager, kv_cache_store, weight_synchronizer,
pool_layout}.py -- and records, per public method or property: its kind,
its parameter names in order (positional-or-keyword, then keyword-only) and
the defaults that are literals.  tests/test_cpu_api_surface.py checks the
package's classes against it.

The output is committed; tests never read the reference.
"""

from __future__ import annotations

import ast
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "api_surface.json"
sys.path.insert(0, str(ROOT))

FILES = {
    "tpu_sync/api/torch/kv_cache_manager.py": ["KVCacheManager"],
    "tpu_sync/api/torch/kv_cache_store.py": ["RaidenId", "RaidenBlockId", "KVCacheStore"],
    "tpu_sync/api/torch/weight_synchronizer.py": ["WeightSynchronizer"],
    "tpu_sync/api/torch/pool_layout.py": ["RegionSpec", "PoolSpec"],
}


def _literal(node):
  try:
    return {"value": ast.literal_eval(node)}
  except ValueError:
    return None


def _method(fn: ast.FunctionDef):
  decos = {d.id if isinstance(d, ast.Name) else getattr(d, "attr", "") for d in fn.decorator_list}
  kind = ("property" if "property" in decos else "classmethod" if "classmethod" in decos
          else "staticmethod" if "staticmethod" in decos else "method")
  a = fn.args
  positional = [x.arg for x in a.posonlyargs + a.args]
  if kind in ("method", "classmethod") and positional:
    positional = positional[1:]  # self / cls
  pos_defaults = dict(zip([x.arg for x in (a.posonlyargs + a.args)][-len(a.defaults):]
                          if a.defaults else [], a.defaults))
  kw_defaults = {x.arg: d for x, d in zip(a.kwonlyargs, a.kw_defaults) if d is not None}
  defaults = {}
  for name, node in list(pos_defaults.items()) + list(kw_defaults.items()):
    lit = _literal(node)
    if lit is not None:
      defaults[name] = lit["value"]
  return {"kind": kind, "positional": positional, "keyword_only": [x.arg for x in a.kwonlyargs],
          "defaults": defaults, "line": fn.lineno}


def main():
  from oracle.build_ref import reference_root
  ref = reference_root()
  out = {}
  for rel, classes in FILES.items():
    tree = ast.parse((ref / rel).read_text())
    for node in tree.body:
      if isinstance(node, ast.ClassDef) and node.name in classes:
        methods = {}
        for fn in node.body:
          if isinstance(fn, (ast.FunctionDef, ast.AsyncFunctionDef)) and (
              not fn.name.startswith("_") or fn.name == "__init__"):
            methods[fn.name] = _method(fn)
        out[node.name] = {"file": rel, "line": node.lineno, "methods": methods}
  OUT.write_text(json.dumps(out, indent=1, sort_keys=True) + "\n")
  print(f"{sum(len(c['methods']) for c in out.values())} methods of {len(out)} classes -> {OUT}")


if __name__ == "__main__":
  main()

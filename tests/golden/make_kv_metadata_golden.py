"""Generates tests/golden/kv_metadata.json: KV metadata table fixtures.

Run in a container that has the reference checkout (read-only) at
REFERENCE_ROOT (else BASELINE.json's reference_path):

    python tests/golden/make_kv_metadata_golden.py

Every script (oracle/ref_meta.py: the reference unit test's cases and seeded
random scripts) is executed by the REFERENCE's own
tpu_sync/kv_cache/kv_cache_metadata.cc, compiled by oracle/build_ref.py into
oracle/_ref/meta_ref; its answers (statuses, entries, table bytes) are
recorded.  The header's bytes [84, 128) are padding that the reference fills
from an uninitialised stack object, so they are zeroed in the record and
ignored by the tests.  The output is committed; tests never read the
reference.
"""

from __future__ import annotations

import json
import random
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "kv_metadata.json"
sys.path.insert(0, str(ROOT))

from oracle import ref_meta  # noqa: E402


def mask_padding(out):
  res = []
  for line in out:
    if line.startswith("bytes "):
      b = bytearray.fromhex(line[6:])
      b[84:128] = bytes(44)
      line = "bytes " + b.hex()
    res.append(line)
  return res


def main():
  cases = []
  for name, script in ref_meta.kat_scripts().items():
    cases.append({"name": name, "script": script, "out": mask_padding(ref_meta.run(script))})
  rng = random.Random(20261201)
  for i in range(40):
    script = ref_meta.random_script(rng)
    cases.append({"name": f"random_{i}", "script": script,
                  "out": mask_padding(ref_meta.run(script))})
  OUT.write_text(json.dumps({"padding_ignored": [84, 128], "cases": cases}, indent=0) + "\n")
  print(f"wrote {len(cases)} cases to {OUT}")


if __name__ == "__main__":
  main()

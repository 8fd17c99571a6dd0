"""Runs the reference's KVCacheMetadata through oracle/_ref/meta_ref.

Test infrastructure only (tests/ and the golden-fixture script use it): the
reference's tpu_sync/kv_cache/kv_cache_metadata.cc and
kv_cache_metadata_shm.cc, compiled by oracle/build_ref.py, execute a command
script (oracle/ref_meta_driver.cc lists the commands) and their answers come
back as lines.
"""

from __future__ import annotations

import subprocess
from typing import List, Optional

from oracle import build_ref


def binary() -> Optional[str]:
  p = build_ref.build_meta()
  return str(p) if p is not None and p.exists() else None


def hx(b: bytes) -> str:
  return b.hex() if b else "-"


def run(lines: List[str]) -> List[str]:
  exe = binary()
  if exe is None:
    raise FileNotFoundError("meta_ref is not built (the reference checkout is absent)")
  r = subprocess.run([exe], input=("\n".join(lines) + "\n").encode(), capture_output=True,
                     timeout=60, check=True)
  # messages quote recorded model uids byte for byte
  return r.stdout.decode("latin-1").splitlines()


def parse_entries(out: List[str], start: int):
  """Entries printed by one 'entries' command starting at out[start];
  returns ([(block_id, hash, seq)], index after 'end')."""
  res = []
  i = start
  while out[i] != "end":
    _, bid, h, seq = out[i].split(" ")
    res.append((int(bid), b"" if h == "-" else bytes.fromhex(h), int(seq)))
    i += 1
  return res, i + 1


# -- command scripts shared by the golden generator and the live tests -------

def kat_scripts():
  """The reference unit test's cases (tpu_sync/kv_cache/kv_cache_metadata_test.cc),
  restated as driver scripts: name -> lines."""
  req = lambda n: 128 + 128 * n  # noqa: E731
  h = lambda s: s.encode().hex()  # noqa: E731
  return {
      # FormatCreatesEmptyTable (:52-58)
      "format_creates_empty_table": [f"region {req(4)}", "format 4 -", "entries", "dump"],
      # FormatRejectsInvalidRegions (:60-73)
      "format_rejects_invalid_regions": [
          f"region {req(4)}", "format 0 -", "format 4 - null", "format 8 - 0 128",
          f"format 2 - 1 {req(4) - 1}"],
      # SetAndClearRoundTrip (:75-88)
      "set_and_clear_round_trip": [
          f"region {req(4)}", "format 4 -", f"set 1 {h('hash_b')} 2", f"set 3 {h('hash_d')} 1",
          "entries", "clear 1", "entries", "dump"],
      # SetOverwritesPreviousBinding (:90-98)
      "set_overwrites_previous_binding": [
          f"region {req(2)}", "format 2 -", f"set 0 {h('old_hash')} 1", f"set 0 {h('new')} 2",
          "entries", "dump"],
      # SetValidatesArguments (:100-120)
      "set_validates_arguments": [
          f"region {req(2)}", "format 2 -", "set -1 68 0", "set 2 68 0", "set 0 - 0",
          f"set 0 {'78' * 113} 0", "clear 2", f"set 0 {'79' * 112} 0", "entries", "dump"],
      # HashesAreOpaqueBytes (:122-130)
      "hashes_are_opaque_bytes": [
          f"region {req(1)}", "format 1 -", "set 0 00ff0072616964656e01 7", "entries", "dump"],
      # AttachRecoversEntriesFromSurvivingRegion (:132-148)
      "attach_recovers_entries": [
          f"region {req(4)}", "format 4 -", f"set 0 {h('hash_a')} 3", f"set 2 {h('hash_c')} 4",
          "attach 4 -", "entries"],
      # AttachRejectsUnformattedOrMismatchedRegions (:150-166)
      "attach_rejects_unformatted_or_mismatched": [
          f"region {req(8)}", "attach 4 -", "format 4 -", "attach 8 -", "attach 4 -"],
      # AttachValidatesModelUid (:168-186)
      "attach_validates_model_uid": [
          f"region {req(4)}", f"format 4 {h('model_a')}", f"attach 4 {h('model_a')}",
          f"attach 4 {h('model_b')}", "attach 4 -", f"format 4 {'78' * 64}"],
      # FormatWipesSurvivingEntries (:188-197)
      "format_wipes_surviving_entries": [
          f"region {req(2)}", "format 2 -", f"set 0 {h('stale')} 1", "format 2 -", "entries",
          "dump"],
      # UncommittedEntryIsInvisible (:199-217): seq 9, hash_len 4, "torn", valid 0
      "uncommitted_entry_is_invisible": [
          f"region {req(2)}", "format 2 -", "poke 128 09000000000000000400",
          f"poke 144 {h('torn')}", "attach 2 -", "entries"],
  }


def random_script(rng):
  """A seeded random command script: valid and invalid sets / clears,
  re-attaches under matching and mismatching geometry, corrupted headers and
  re-formats; ends with the table's bytes."""
  nb = rng.randint(1, 8)
  size = 128 + 128 * nb + rng.choice([0, 0, 64, 192])
  uid_len = rng.choice([0, 1, 7, 20, 63])
  uid = bytes(rng.randint(0x21, 0x7e) for _ in range(uid_len))
  lines = [f"region {size}", f"format {nb} {hx(uid)}"]
  for _ in range(rng.randint(10, 40)):
    r = rng.random()
    if r < 0.45:
      bid = rng.choice([rng.randrange(nb)] * 6 + [-1, nb, nb + 3])
      hl = rng.choice([1, 5, 16, 32, 64, 111, 112] * 3 + [0, 113, 200])
      h = bytes(rng.randrange(256) for _ in range(hl))
      lines.append(f"set {bid} {hx(h)} {rng.randrange(1 << 64)}")
    elif r < 0.6:
      lines.append(f"clear {rng.choice([rng.randrange(nb)] * 4 + [-1, nb])}")
    elif r < 0.72:
      lines.append("entries")
    elif r < 0.84:
      k = rng.random()
      if k < 0.5:
        lines.append(f"attach {nb} {hx(uid)}")
      elif k < 0.7:
        lines.append(f"attach {nb + 1} {hx(uid)}")
      else:
        lines.append(f"attach {nb} {hx(uid + b'x')}")
    elif r < 0.92:
      field = rng.choice([(0, 8), (8, 4), (16, 4), (12, 4), (20, 1)])
      # the uid byte stays printable: mismatch messages quote it
      lo, hi = (0x21, 0x7e) if field[0] == 20 else (0, 255)
      junk = bytes(rng.randint(lo, hi) for _ in range(field[1]))
      lines += [f"poke {field[0]} {junk.hex()}", f"attach {nb} {hx(uid)}",
                f"format {nb} {hx(uid)}"]
    else:
      lines.append(f"format {nb} {hx(uid)}")
  lines += ["entries", "dump"]
  return lines

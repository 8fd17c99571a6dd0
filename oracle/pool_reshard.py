"""CPU oracle for the pool reshard planner -- TEST INFRASTRUCTURE ONLY.

Only tests/ import this module, as the checker; the product never calls it.

Pure-Python restatement of the data-plane part of BuildPoolReshardPlan
(tpu_sync/kv_cache/reshard/pool_reshard_planner.cc:132-859) and of how the
reference applies a plan's entries (the sender resolves each entry's source
range in its pool block and the receiver the destination range in its pool
block, tpu_sync/kv_cache/kv_cache_manager_base.cc:2400-2510; every pool of
the entry's group gets the bytes).

Parity pinning: the known answers of the reference's planner tests
(tpu_sync/kv_cache/reshard/reshard_service_test.cc:288-487) and 300 seeded
requests answered by the reference's own planning flow -- its
pool_layout.cc, work_unit_directory.cc, request_block_registry.cc and
pool_reshard_planner.cc compiled here (oracle/build_ref.py -> plan_ref),
recorded in tests/golden/pool_reshard_plans.json -- are checked in
tests/test_cpu_pool_reshard.py.  The registration checks the reference makes
before planning (unit and byte-span registration) come first here too.

Pools are dicts as in oracle/pool_layout.py; a declaration is
(unit, {"tag", "block_ids", "spans": [span dicts], "declared_bytes",
"dst_space_version"}); a span dict has the PoolByteSpan fields.
"""

from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

from oracle import pool_layout as opl

MAX_LIVE = 1 << 20


class PlanError(Exception):
  pass


def _q(s):
  return f"'{s}'"


def _sig(p):
  return (p["tag"], p["storage_index"], p["base_offset_bytes"], p["block_stride_bytes"],
          p["num_blocks"], p.get("dtype_tag", ""),
          tuple((r["name"], r["offset_bytes"], r["stride_bytes"], r["unit_bytes"],
                 r["num_units"], r["units_per_stride"]) for r in p["regions"]))


MAX_SPAN_COUNT = 1 << 20


def check_unit_registrations(src_pools, dst_pools, ranks, unit_parallelism):
  """WorkUnitDirectory::Validate (kv_cache/reshard/work_unit_directory.cc:66-86)
  for every source unit in order, then the destination.  A unit without an
  explicit transfer_parallelism declares the number of source units, without
  a rank its index."""
  nu = len(src_pools)
  for u in range(nu):
    if not src_pools[u]:
      raise PlanError("pool_manifest must not be empty")
    par = unit_parallelism[u] if unit_parallelism else nu
    rank = ranks[u] if ranks else u
    if par <= 0:
      raise PlanError("transfer_parallelism must be positive")
    if rank < 0:
      raise PlanError("transfer_rank must be non-negative")
    if rank >= par:
      raise PlanError("transfer_rank must be less than transfer_parallelism")
  if not dst_pools:
    raise PlanError("pool_manifest must not be empty")


def check_span_registrations(src_pools, decls, name):
  """RequestBlockRegistry::Register (kv_cache/reshard/request_block_registry.cc:142-245)
  for every source unit in order: its declarations, in the order given,
  against the live bytes of its manifest's pools per tag."""
  for uu, _ in decls:
    if uu < 0 or uu >= len(src_pools):
      raise PlanError(f"Work unit is not registered: src unit {uu}")
  for u in range(len(src_pools)):
    mine = [d for uu, d in decls if uu == u]
    if not mine:
      continue
    live_by_tag = {}
    for p in src_pools[u]:
      try:
        live = sum(x[2] for x in opl.live_segments(p))
      except opl.PoolError as e:
        raise PlanError(e.message) from None
      if live_by_tag.setdefault(p["tag"], live) != live:
        raise PlanError(f"pools tagged {p['tag']} disagree on live bytes for {name(u)}; "
                        "byte-span registration requires one geometry per tag")
    seen = set()
    for d in mine:
      tag = d["tag"]
      if not tag:
        raise PlanError("pool span registration tag must not be empty")
      if tag in seen:
        raise PlanError(f"duplicate pool span registration tag: {tag}")
      seen.add(tag)
      if tag not in live_by_tag:
        raise PlanError(f"pool span registration {tag} does not match any registered pool for "
                        f"{name(u)}")
      live = live_by_tag[tag]
      ids = list(d["block_ids"])
      if any(b < 0 for b in ids):
        raise PlanError(f"pool span registration {tag} block_ids must be non-negative")
      if len(set(ids)) != len(ids):
        raise PlanError(f"pool span registration {tag} block_ids must not contain duplicates")
      total = 0
      for sp in d["spans"]:
        if sp["size_bytes"] <= 0:
          raise PlanError(f"byte span size_bytes must be positive ({tag})")
        if sp["count"] <= 0:
          raise PlanError(f"byte span count must be positive ({tag})")
        if sp["count"] > MAX_SPAN_COUNT:
          raise PlanError(f"byte span count {sp['count']} exceeds the expansion bound ({tag})")
        if min(sp["src_offset_bytes"], sp["dst_offset_bytes"], sp["src_stride_bytes"],
               sp["dst_stride_bytes"], sp["dst_block_index"]) < 0:
          raise PlanError(f"byte span fields must be non-negative ({tag})")
        o = sp["src_block_ordinal"]
        if o < 0 or o >= len(ids):
          raise PlanError(f"byte span ordinal {o} is outside the registration's {len(ids)} "
                          f"block ids ({tag})")
        end = sp["src_offset_bytes"] + (sp["count"] - 1) * sp["src_stride_bytes"] + sp["size_bytes"]
        if end > live:
          raise PlanError(f"byte span exceeds its source block live bytes ({tag}): end={end}, "
                          f"live={live}")
        total += sp["size_bytes"] * sp["count"]
      if d["declared_bytes"] != total:
        raise PlanError(f"pool span registration {tag} declared_bytes {d['declared_bytes']} "
                        f"disagrees with the span sum {total}")


def build_plan(src_pools, dst_pools, tags, dst_ids, decls, dst_block_counts=None,
               dst_skip_bytes=None, parallelism=None, ranks=None, unit_parallelism=None,
               unit_names=None):
  """Returns {"schedules": {unit: [entry tuples]}, "groups": [...], "src_units": [...]}.

  entry tuple = (src_block, dst_block, src_off, dst_off, size, group).
  Raises PlanError(message) with the reference's messages: the registration
  checks first (check_unit_registrations, check_span_registrations), then
  the planner's.
  """
  nu = len(src_pools)
  name = (lambda u: unit_names[u]) if unit_names else (lambda u: f"src unit {u}")
  check_unit_registrations(src_pools, dst_pools, ranks, unit_parallelism)
  check_span_registrations(src_pools, decls, name)
  if not dst_ids:
    raise PlanError("dst_device_block_ids must not be empty")
  if any(b < 0 for b in dst_ids):
    raise PlanError("dst_device_block_ids must be non-negative")
  for u in range(nu):
    if not src_pools[u]:
      raise PlanError(f"Missing explicit pool manifest for {name(u)}")
  ident = [(p["tag"], p.get("dtype_tag", "")) for p in dst_pools]
  for u in range(nu):
    if [(p["tag"], p.get("dtype_tag", "")) for p in src_pools[u]] != ident:
      raise PlanError("Canonical pool manifest mismatch between source and destination for "
                      + name(u))
  for u in range(1, nu):
    if [_sig(p) for p in src_pools[u]] != [_sig(p) for p in src_pools[0]]:
      raise PlanError(f"Source pool geometry differs across ranks at {name(u)}")
  if not tags:
    raise PlanError("transfer_pool_tags must name at least one pool tag")
  if len(set(tags)) != len(tags):
    raise PlanError("transfer_pool_tags must not repeat tags; got [" +
                    ", ".join(_q(t) for t in tags) + "]")
  counts = list(dst_block_counts or [])
  if counts:
    if len(counts) != len(tags):
      raise PlanError(f"dst_block_counts must align 1:1 with transfer_pool_tags: {len(counts)} "
                      f"counts for {len(tags)} tags")
    if any(c <= 0 for c in counts) or sum(counts) != len(dst_ids):
      raise PlanError("dst_block_counts must be positive and sum to the destination block count: "
                      f"counts=[{', '.join(map(str, counts))}], blocks={len(dst_ids)}")
  elif len(tags) == 1:
    counts = [len(dst_ids)]
  else:
    raise PlanError("Multi-tag transfers must split dst_device_block_ids with dst_block_counts")
  tag_dst, cur = [], 0
  for c in counts:
    tag_dst.append(list(dst_ids[cur:cur + c]))
    cur += c
  skips = [0] * len(tags)
  if dst_skip_bytes:
    if len(dst_skip_bytes) != len(tags):
      raise PlanError(f"dst_skip_bytes must align 1:1 with transfer_pool_tags: "
                      f"{len(dst_skip_bytes)} skips for {len(tags)} tags")
    for i, s in enumerate(dst_skip_bytes):
      if s < 0:
        raise PlanError(f"dst_skip_bytes must be non-negative; tag {_q(tags[i])} requested {s}")
      skips[i] = s
  avail = {p["tag"] for p in dst_pools}
  for t in tags:
    if t not in avail:
      raise PlanError(f"transfer_pool_tags do not match any registered pool: [{_q(t)}]")
  par = {(unit_parallelism[u] if unit_parallelism else nu) for u in range(nu)}
  rank_of = {(ranks[u] if ranks else u): u for u in range(nu)}
  if len(par) != 1 or min(par) <= 0:
    raise PlanError("All source ranks must declare one consistent positive transfer_parallelism")
  topo = par.pop()
  if len(rank_of) != nu:
    raise PlanError("Source transfer_rank values must be unique")
  if sorted(rank_of) != list(range(nu)):
    raise PlanError("Source transfer_rank values must be contiguous from zero")
  req_par = parallelism if parallelism else topo
  if req_par > topo:
    raise PlanError(f"parallelism exceeds source admission: requested={req_par}, admitted={topo}")

  pre = []
  for g, tag in enumerate(tags):
    ids = tag_dst[g]
    if len(set(ids)) != len(ids):
      raise PlanError(f"dst_device_block_ids for tag {_q(tag)} must not contain duplicates")
    sel = [i for i, p in enumerate(dst_pools) if p["tag"] == tag]
    sl, dl, smaps, dmaps = set(), set(), [], []
    for pi in sel:
      try:
        ss = opl.live_segments(src_pools[0][pi])
        ds = opl.live_segments(dst_pools[pi])
      except opl.PoolError as e:
        raise PlanError(e.message) from None
      s_live, d_live = sum(x[2] for x in ss), sum(x[2] for x in ds)
      if s_live <= 0 or d_live <= 0:
        raise PlanError(f"Pool {pi} has no declared live bytes")
      sl.add(s_live)
      dl.add(d_live)
      if ss not in smaps:
        smaps.append(ss)
      if ds not in dmaps:
        dmaps.append(ds)
    if len(sl) != 1 or len(dl) != 1:
      raise PlanError(f"Pools tagged {tag} must share one geometry per side; "
                      f"src=[{', '.join(map(str, sorted(sl)))}] dst=[{', '.join(map(str, sorted(dl)))}]")
    if len(smaps) != 1 or len(dmaps) != 1:
      raise PlanError(f"Pools tagged {tag} must share one live-region map per side")
    s_live, d_live = sl.pop(), dl.pop()
    if skips[g] % d_live:
      raise PlanError("dst_skip_bytes must be a whole multiple of the destination page live bytes "
                      f"for tag {_q(tag)}: skip={skips[g]}, page_live_bytes={d_live}")
    pre.append((sel, s_live, d_live, smaps[0], dmaps[0]))

  schedules: Dict[int, List[tuple]] = {}
  groups, union_sel, emitted = [], [], 0
  for g, tag in enumerate(tags):
    ids = tag_dst[g]
    sel, s_live, d_live, sseg, dseg = pre[g]
    skip = skips[g]
    declared = []
    for u in range(nu):
      for du, d in decls:
        if du == u and d["tag"] == tag and d["spans"]:
          declared.append((u, dict(d, spans=[dict(s) for s in d["spans"]])))
    if not declared:
      raise PlanError(f"No byte-span declarations are registered for tag {tag}")
    clipped = global_end = 0
    for u, d in declared:
      if d.get("dst_space_version", 0) == 0:
        if skip > 0:
          raise PlanError("dst_skip_bytes requires destination-page-agnostic (dst_space_version=1) "
                          f"declarations for tag {_q(tag)} (declared by {name(u)})")
        continue
      split = []
      for sp in d["spans"]:
        if sp.get("count", 1) > 1 or sp.get("src_stride_bytes", 0) or sp.get("dst_stride_bytes", 0):
          raise PlanError("Global-space byte spans must be plain contiguous ranges (declared by "
                          f"{name(u)})")
        if sp["dst_block_index"] != 0:
          raise PlanError("Global-space byte spans must leave dst_block_index zero (declared by "
                          f"{name(u)})")
        global_end = max(global_end, sp["dst_offset_bytes"] + sp["size_bytes"])
        adv = 0
        if sp["dst_offset_bytes"] + sp["size_bytes"] <= skip:
          clipped += sp["size_bytes"]
          continue
        if sp["dst_offset_bytes"] < skip:
          adv = skip - sp["dst_offset_bytes"]
          clipped += adv
        left = sp["size_bytes"] - adv
        goff = sp["dst_offset_bytes"] + adv - skip
        soff = sp["src_offset_bytes"] + adv
        while left > 0:
          page, inp = divmod(goff, d_live)
          take = min(left, d_live - inp)
          split.append({"src_block_ordinal": sp["src_block_ordinal"], "src_offset_bytes": soff,
                        "dst_block_index": page, "dst_offset_bytes": inp, "size_bytes": take,
                        "src_stride_bytes": 0, "dst_stride_bytes": 0, "count": 1})
          goff += take
          soff += take
          left -= take
      d["spans"] = split
      d["dst_space_version"] = 0
    if skip > 0 and skip >= global_end:
      raise PlanError(f"dst_skip_bytes removes the entire tag {_q(tag)}: skip={skip}, "
                      f"declared_extent={global_end}; a full local hit must not reach the planner")
    for pi in sel:
      for u, d in declared:
        if any(b >= src_pools[u][pi]["num_blocks"] for b in d["block_ids"]):
          raise PlanError(f"Source block id is out of range for pool {pi} at {name(u)}")
      if any(b >= dst_pools[pi]["num_blocks"] for b in ids):
        raise PlanError(f"Destination block id is out of range for pool {pi}")
    cov = [[] for _ in ids]
    repeats = declared_total = covered_total = 0
    for u, d in declared:
      declared_total += d["declared_bytes"]
      for sp in d["spans"]:
        cnt = sp.get("count", 1)
        ss, ds = sp.get("src_stride_bytes", 0), sp.get("dst_stride_bytes", 0)
        if sp["dst_block_index"] >= len(ids):
          raise PlanError(f"Byte span destination index {sp['dst_block_index']} exceeds the "
                          f"transfer's {len(ids)} destination blocks for tag {_q(tag)} "
                          f"(declared by {name(u)})")
        src_end = sp["src_offset_bytes"] + (cnt - 1) * ss + sp["size_bytes"]
        if src_end > s_live:
          raise PlanError(f"Byte span exceeds its source block live bytes: end={src_end}, "
                          f"live={s_live} (declared by {name(u)})")
        dst_end = sp["dst_offset_bytes"] + (cnt - 1) * ds + sp["size_bytes"]
        if dst_end > d_live:
          raise PlanError(f"Byte span exceeds its destination block live bytes: end={dst_end}, "
                          f"live={d_live} (declared by {name(u)})")
        repeats += cnt
        if repeats > MAX_LIVE:
          raise PlanError("Byte span plan exceeds the repeat expansion bound")
        for r in range(cnt):
          st = sp["dst_offset_bytes"] + r * ds
          cov[sp["dst_block_index"]].append((st, st + sp["size_bytes"]))
          covered_total += sp["size_bytes"]
    extents = []
    for i in range(len(ids)):
      iv = sorted(cov[i])
      if not iv:
        raise PlanError(f"Destination block index {i} has no declared coverage for tag {_q(tag)}")
      until = 0
      for s, e in iv:
        if s != until:
          kind = "overlap" if s < until else "gap"
          raise PlanError(f"Declared byte spans have a destination coverage {kind} at byte "
                          f"{min(s, until)} of destination block index {i}")
        until = e
      if i != len(ids) - 1 and until != d_live:
        raise PlanError(f"Destination block index {i} is covered to {until} of {d_live} live "
                        "bytes; only the final block may be partial")
      extents.append(until)
    if declared_total != covered_total + clipped:
      m = f"Declared byte totals disagree with coverage: declared={declared_total}, covered={covered_total}"
      if clipped:
        m += f", clipped={clipped}"
      raise PlanError(m)
    ordered = [(u, d, sp) for u, d in declared for sp in d["spans"]]
    ordered.sort(key=lambda x: (x[2]["dst_block_index"], x[2]["dst_offset_bytes"]))
    pairs: Dict[int, set] = {}
    for u, d, sp in ordered:
      if not 0 <= sp["src_block_ordinal"] < len(d["block_ids"]):
        raise PlanError(f"Byte span source ordinal {sp['src_block_ordinal']} is out of range "
                        f"(declared by {name(u)})")
      sb = d["block_ids"][sp["src_block_ordinal"]]
      db = ids[sp["dst_block_index"]]
      for r in range(sp.get("count", 1)):
        try:
          chunks = opl.translate_live_copy(
              sseg, dseg, sp["src_offset_bytes"] + r * sp.get("src_stride_bytes", 0),
              sp["dst_offset_bytes"] + r * sp.get("dst_stride_bytes", 0), sp["size_bytes"])
        except opl.PoolError as e:
          raise PlanError(e.message) from None
        emitted += len(chunks)
        if emitted > MAX_LIVE:
          raise PlanError("Byte-span plan exceeds the live-region expansion bound")
        for sph, dph, n in chunks:
          schedules.setdefault(u, []).append((sb, db, sph, dph, n, g))
      pairs.setdefault(u, set()).add((sb, db))
    pushes = sum(min(req_par, len(p)) for p in pairs.values())
    if pushes <= 0:
      raise PlanError(f"Pool reshard plan contains no source pushes for tag {_q(tag)}")
    groups.append({"pool_indices": tuple(sel), "dst_device_block_ids": tuple(ids),
                   "expected_pushes": pushes, "dst_expected_extent_bytes": tuple(extents),
                   "order_rank": 0 if g == 0 else 1})
    union_sel += sel
  if len(set(union_sel)) != len(union_sel):
    raise PlanError("Requested tags select overlapping pool indices; tags must partition their pools")
  src_units = [rank_of[r] for r in sorted(rank_of) if rank_of[r] in schedules]
  return {"schedules": schedules, "groups": groups, "src_units": src_units,
          "transfer_pool_indices": union_sel}


def apply_plan(plan, unit, src_pools, dst_pools, src_storages, dst_storages):
  """Applies one source unit's entries (numpy uint8 storages, by storage index)."""
  for sb, db, so, do, n, g in plan["schedules"].get(unit, []):
    for pi in plan["groups"][g]["pool_indices"]:
      sp, dp = src_pools[pi], dst_pools[pi]
      s0 = sp["base_offset_bytes"] + sb * sp["block_stride_bytes"] + so
      d0 = dp["base_offset_bytes"] + db * dp["block_stride_bytes"] + do
      dst_storages[dp["storage_index"]][d0:d0 + n] = src_storages[sp["storage_index"]][s0:s0 + n]

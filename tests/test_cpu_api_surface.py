"""The package's classes carry the reference's Python surface.

tests/golden/api_surface.json records, from the reference's
tpu_sync/api/torch/{kv_cache_manager, kv_cache_store, weight_synchronizer,
pool_layout}.py (read as text by tests/golden/make_api_surface_golden.py),
every public method and property of the classes a caller uses, with its
parameter order and literal defaults.  Each must exist here as the same kind
(method, classmethod, property), take the reference's positional parameters
in the reference's order (extra trailing parameters are allowed), accept its
keyword-only parameters and default to the same literal values, so code
written against the reference calls this package unchanged.  A few entry
points the reference serves over its TCP transport or on a host-only
manager exist here only to raise NotImplementedError with the on-node
alternative; they are listed in NOT_ON_ONE_NODE and checked to do so.
"""

import dataclasses
import inspect
import json
from pathlib import Path

import pytest

from tpu_sync_b200 import (KVCacheManager, KVCacheStore, PoolSpec, RaidenBlockId, RegionSpec,
                           WeightSynchronizer)
from tpu_sync_b200.kv_cache_store import BlockStatus, RaidenId

OURS = {"KVCacheManager": KVCacheManager, "KVCacheStore": KVCacheStore, "RaidenId": RaidenId,
        "RaidenBlockId": RaidenBlockId, "WeightSynchronizer": WeightSynchronizer,
        "RegionSpec": RegionSpec, "PoolSpec": PoolSpec}
NOT_ON_ONE_NODE = {("KVCacheManager", "create_host_only_for_testing"),
                   ("KVCacheManager", "register_active_plan"),
                   ("KVCacheManager", "unregister_active_plan"),
                   ("KVCacheManager", "push_registered_plan")}

SURFACE = json.loads((Path(__file__).resolve().parent / "golden" / "api_surface.json").read_text())
CASES = [(c, m) for c, spec in sorted(SURFACE.items()) for m in sorted(spec["methods"])]


@pytest.mark.parametrize("cls_name,name", CASES)
def test_reference_member(cls_name, name):
  spec = SURFACE[cls_name]["methods"][name]
  cls = OURS[cls_name]
  fields = getattr(cls, "__dataclass_fields__", {})
  if name in fields:
    assert spec["kind"] == "property", (cls_name, name)  # a dataclass field reads the same
    return
  attr = inspect.getattr_static(cls, name, None)
  assert attr is not None, f"{cls_name}.{name} is missing"
  if spec["kind"] == "property":
    assert isinstance(attr, property), f"{cls_name}.{name} should be a property"
    return
  if spec["kind"] == "classmethod":
    assert isinstance(attr, classmethod), f"{cls_name}.{name} should be a classmethod"
  fn = attr.__func__ if isinstance(attr, (classmethod, staticmethod)) else attr
  sig = inspect.signature(fn)
  params = list(sig.parameters.values())
  if spec["kind"] in ("method", "classmethod") and params and params[0].name in ("self", "cls"):
    params = params[1:]
  positional = [p.name for p in params
                if p.kind in (p.POSITIONAL_ONLY, p.POSITIONAL_OR_KEYWORD)]
  assert positional[:len(spec["positional"])] == spec["positional"], (cls_name, name, positional)
  names = {p.name for p in params}
  for k in spec["keyword_only"]:
    assert k in names, (cls_name, name, k)
  for k, want in spec["defaults"].items():
    got = sig.parameters[k].default
    assert got is not inspect.Parameter.empty and got == want, (cls_name, name, k, got, want)


@pytest.mark.parametrize("cls_name,name", sorted(NOT_ON_ONE_NODE))
def test_transport_only_entry_points_say_so(cls_name, name):
  fn = getattr(OURS[cls_name], name)
  with pytest.raises(NotImplementedError):
    if name == "create_host_only_for_testing":
      fn(num_layers=1, slice_byte_size=1, node_id=0, host_blocks=1)
    else:
      fn(object.__new__(OURS[cls_name]), *([1] * (len(SURFACE[cls_name]["methods"][name]
                                                             ["positional"]))))


def test_block_id_positional_order_and_accessors():
  rid = RaidenId("job", "0", "kv", 2)
  b = RaidenBlockId(rid, 7, BlockStatus.HOST, 3)  # the reference's positional order
  assert (b.host_block_id, b.status, b.device_block_id) == (7, BlockStatus.HOST, 3)
  assert (b.job_name, b.job_replica_id, b.data_name, b.data_replica_idx) == ("job", "0", "kv", 2)
  assert RaidenBlockId(None).raiden_id == RaidenId()
  assert dataclasses.replace(b, status=BlockStatus.HBM).status == BlockStatus.HBM

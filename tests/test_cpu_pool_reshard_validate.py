"""Received pool reshard plans: the executor's validation on the CPU.

Ports the reference's executor tests
(tpu_sync/core/kv_cache_manager_with_transfer_pool_reshard_test.cc:185-619)
as known answers for ts_pool_reshard_validate: each case builds the same
plan (ValidPlan / AddEntry, :92-133, :391-406) and expects acceptance or the
same error fragment.  The transport identity checks of that file (req_id,
uuid, use_block_chunks) and the device-attachment gate are control plane and
have no counterpart here.
"""

import copy

import pytest

from tpu_sync_b200.pool_layout import PoolSpec, RegionSpec
from tpu_sync_b200.pool_reshard import plan_from_received, validate_pool_reshard_plan

INT64_MAX = (1 << 63) - 1


def dense_pool(tag, block_stride=128, dtype_tag="bf16"):  # :72-90
  return PoolSpec(tag, 0, 0, block_stride, 4,
                  (RegionSpec("block", 0, block_stride, block_stride, 1, 1),), dtype_tag)


def implicit_pool():
  """The implicit pool of the test manager (1 storage, 128-byte slices, 4 host blocks)."""
  return PoolSpec("opaque", 0, 0, 128, 4, (RegionSpec("block", 0, 128, 128, 1, 1),), "")


def entry(dst_block=0, dst_off=0, size=16, group=0, **kw):
  e = dict(dst_peer="127.0.0.1:1", dst_shard_idx=0, src_block_id=0, dst_block_id=dst_block,
           src_offset_bytes=0, dst_offset_bytes=dst_off, size_bytes=size, src_stride_bytes=0,
           dst_stride_bytes=0, count=1, pool_group=group)
  e.update(kw)
  return e


def valid_plan(dtype_tags=("bf16",), pools=(0,)):  # ValidPlan, :92-125
  return {"transfer_pool_indices": list(pools), "pool_dtype_tags": list(dtype_tags),
          "parallelism": 1,
          "pool_groups": [{"pool_indices": list(pools), "dst_device_block_ids": [0],
                           "expected_pushes": 1, "dst_expected_extent_bytes": [16],
                           "order_rank": 0}],
          "shard_push_schedules": {0: [entry()]}}


def check(plan, pools, ids, is_sender, fragment=None):
  if fragment is None:
    validate_pool_reshard_plan(plan, pools, ids, is_sender)
  else:
    with pytest.raises(ValueError, match=fragment):
      validate_pool_reshard_plan(plan, pools, ids, is_sender)


def test_accepts_canonical_plan_on_explicit_pools():  # :185-198
  check(valid_plan(), [dense_pool("fa")], [0], False)
  check(valid_plan(), [dense_pool("fa")], [0], True)


def test_accepts_implicit_pools():  # :200-211
  check(valid_plan(dtype_tags=("",)), [implicit_pool()], [0], False)


def test_has_no_tag_policy():  # :213-225
  check(valid_plan(), [dense_pool("gdn.conv")], [0], False)


def test_rejects_missing_pool_fields():  # :245-277 (pool fields)
  p = valid_plan()
  p["transfer_pool_indices"] = []
  check(p, [dense_pool("fa")], [0], False, "transfer_pool_indices")
  p = valid_plan()
  p["pool_groups"] = []
  check(p, [dense_pool("fa")], [0], False, "must declare pool_groups")


def test_rejects_out_of_range_duplicate_and_dtype_mismatch():  # :279-304
  pools = [dense_pool("fa")]
  check(valid_plan(pools=(1,)), pools, [0], False, "out of range")
  check(valid_plan(pools=(0, 0)), pools, [0], False, "duplicate transfer pool index")
  check(valid_plan(dtype_tags=("fp8",)), pools, [0], False, "dtype tag mismatch")
  check(valid_plan(dtype_tags=("bf16", "bf16")), pools, [0], False, "one dtype tag per pool")


def test_checks_every_pool_span_and_destination_zero_cover():  # :306-334
  pools = [dense_pool("fa", 128), dense_pool("fa", 64)]
  p = valid_plan(("bf16", "bf16"), (0, 1))
  p["shard_push_schedules"][0][0].update(dst_offset_bytes=48, size_bytes=32)
  check(p, pools, [0], False, "destination span exceeds declared pool 1")
  p = valid_plan(("bf16", "bf16"), (0, 1))
  p["shard_push_schedules"][0][0].update(dst_offset_bytes=16)
  check(p, pools, [0], False, "no transfer entry starting at offset 0")
  p = valid_plan(("bf16", "bf16"), (0, 1))
  p["shard_push_schedules"][0] = []
  check(p, pools, [0], False, "no entries")


def test_rejects_overflowing_sender_span():  # :336-350
  p = valid_plan()
  p["shard_push_schedules"][0][0].update(src_offset_bytes=96, src_stride_bytes=INT64_MAX,
                                         dst_stride_bytes=1, size_bytes=16, count=2)
  check(p, [dense_pool("fa")], [0], True, "source span exceeds declared pool 0")


def test_rejects_sender_span_between_packed_token_regions():  # :352-389
  pool = PoolSpec("fa", 0, 0, 128, 4, (RegionSpec("head_group_0", 0, 8, 4, 4, 2),
                                        RegionSpec("head_group_1", 64, 8, 4, 4, 2)), "bf16")
  p = valid_plan()
  check(p, [pool], [0], True)
  p["shard_push_schedules"][0][0].update(src_offset_bytes=32, size_bytes=16)
  check(p, [pool], [0], True, "source span exceeds declared pool 0 live regions")


def test_receiver_coverage_cases():  # :408-544
  pools = [dense_pool("fa")]
  p = valid_plan()
  p["pool_groups"][0]["dst_expected_extent_bytes"] = [48]
  p["shard_push_schedules"][0].append(entry(0, 32, 16))
  check(p, pools, [0], False, "coverage gap")
  check(p, pools, [0], True)

  p = valid_plan()
  p["pool_groups"][0]["dst_expected_extent_bytes"] = [24]
  p["shard_push_schedules"][0].append(entry(0, 8, 16))
  check(p, pools, [0], False, "coverage overlap")

  p = valid_plan()
  p["pool_groups"][0]["dst_expected_extent_bytes"] = [24]
  check(p, pools, [0], False, "does not cover the exact live bytes")

  p = valid_plan()
  p["pool_groups"][0]["dst_device_block_ids"] = [0, 1]
  p["pool_groups"][0]["dst_expected_extent_bytes"] = [16, 16]
  p["shard_push_schedules"][0].append(entry(1, 0, 16))
  check(p, pools, [0, 1], False, "except the final one")

  p = valid_plan()
  p["pool_groups"][0]["dst_expected_extent_bytes"] = []
  check(p, pools, [0], False, "require dst_expected_extent_bytes")

  p = valid_plan()
  p["parallelism"] = 0
  check(p, pools, [0], False, "positive parallelism")

  p = valid_plan()
  p["pool_groups"][0]["expected_pushes"] = 2
  check(p, pools, [0], False, "do not match the received schedules")


def test_rejects_write_beyond_declared_live_tail():  # :500-544
  pool = PoolSpec("fa", 0, 0, 128, 4, (RegionSpec("run_0", 0, 32, 32, 1, 1),
                                        RegionSpec("run_1", 64, 32, 32, 1, 1)), "bf16")
  p = valid_plan()
  p["pool_groups"][0]["dst_expected_extent_bytes"] = [40]
  p["shard_push_schedules"][0] = [entry(0, 0, 32), entry(0, 64, 16)]
  check(p, [pool], [0], False, "declared live tail")
  p["shard_push_schedules"][0][1]["size_bytes"] = 8
  check(p, [pool], [0], False)


def test_group_scopes_destination_blocks():  # :546-584
  pools = [dense_pool("fa", 128), dense_pool("gdn", 64)]
  p = valid_plan(("bf16", "bf16"), (0, 1))
  p["pool_groups"] = [
      {"pool_indices": [0], "dst_device_block_ids": [2], "expected_pushes": 1,
       "dst_expected_extent_bytes": [16], "order_rank": 0},
      {"pool_indices": [1], "dst_device_block_ids": [3], "expected_pushes": 1,
       "dst_expected_extent_bytes": [8], "order_rank": 1}]
  p["shard_push_schedules"][0] = [entry(2, 0, 16, 0), entry(3, 0, 8, 1)]
  check(p, pools, [2, 3], False)
  p["shard_push_schedules"][0].append(entry(2, 0, 8, 1))
  check(p, pools, [2, 3], False, "outside its group")


def test_rejects_block_ids_outside_declared_pool():  # :586-619
  pools = [dense_pool("fa")]
  p = valid_plan()
  p["pool_groups"][0]["dst_device_block_ids"] = [9]
  check(p, pools, [9], False, "out of range for pool")
  p = valid_plan()
  check(p, pools, [8], False, "must concatenate to the plan's local block ids")
  check(p, pools, [0, 0], False, "must cover the plan's local block ids")
  check(p, pools, [], False, "must not be empty")


def test_plan_from_received_checks_both_ends():
  pools = [dense_pool("fa")]
  plan = plan_from_received(valid_plan(), pools, pools, [0], [0])
  assert plan.schedules[0][0].size_bytes == 16
  bad = copy.deepcopy(valid_plan())
  bad["shard_push_schedules"][0][0].update(src_offset_bytes=120)
  with pytest.raises(ValueError, match="^sender: source span exceeds declared pool 0"):
    plan_from_received(bad, pools, pools, [0], [0])
  with pytest.raises(ValueError, match="^receiver: .*must concatenate"):
    plan_from_received(valid_plan(), pools, pools, [0], [1])

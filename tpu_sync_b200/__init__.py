"""B200-native data-movement hot path of tpu_sync.

KV block extract/insert between paged HBM storages and a block-major
staging layout, the pinned host tier offload/reload built on it (with the
tier-2 prefix cache and its crash-persistent metadata), the prefill -> decode
KV hand-offs (relayout, pool reshard plans, the managers' pull protocol), and
the weight-sync reshard executor.  Compute runs in hand-written sm_100a
kernels behind the C ABI of ``include/tpusync_b200.h``; this package is the
Python surface over it, with the reference's class names.
"""

from tpu_sync_b200 import _native
from tpu_sync_b200.kv_cache_manager import KVCacheManager, RaidenFuture
from tpu_sync_b200.kv_cache_store import BlockStatus, KVCacheStore, RaidenBlockId, RaidenId
from tpu_sync_b200.kv_metadata import KVCacheMetadata, KVCacheMetadataShmRegion
from tpu_sync_b200.pool_layout import PoolSpec, RegionSpec
from tpu_sync_b200.weight_synchronizer import WeightSynchronizer

__all__ = ["BlockStatus", "KVCacheManager", "KVCacheMetadata", "KVCacheMetadataShmRegion",
           "KVCacheStore", "PoolSpec", "RaidenBlockId", "RaidenFuture", "RaidenId",
           "RegionSpec", "WeightSynchronizer", "_native"]

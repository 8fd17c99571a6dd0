"""B200-native data-movement hot path of tpu_sync.

KV block extract/insert between paged HBM storages and a block-major
staging layout, the pinned host tier offload/reload built on it, the
prefill -> decode KV relayout, and the weight-sync reshard executor.
Compute runs in hand-written sm_100a kernels behind the C ABI of
``include/tpusync_b200.h``; this package is the Python surface over it.
"""

from tpu_sync_b200 import _native
from tpu_sync_b200.kv_cache_manager import KVCacheManager, RaidenFuture

__all__ = ["KVCacheManager", "RaidenFuture", "_native"]

// Stand-in for absl's flat_hash_map used ONLY to compile the reference's
// header-only LRUCache (tpu_sync/kv_cache/lru_cache.h) as a test oracle.
// The LRU order lives in its std::list members; the map is only an index,
// so an unordered_map with the same interface is behaviour-equivalent here.
#pragma once
#include <unordered_map>
namespace absl {
template <typename K, typename V>
using flat_hash_map = std::unordered_map<K, V>;
}  // namespace absl

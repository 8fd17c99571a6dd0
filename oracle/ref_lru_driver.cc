// Test driver around the REFERENCE LRUCache (tpu_sync/kv_cache/lru_cache.h),
// compiled from the reference checkout by oracle/build_ref.py into
// oracle/_ref/lru_ref.  Reads one operation per line on stdin and prints one
// result line, so tests can replay the same trace on the product's LRU.
//
//   put K H D S    -> evicted key or "-"        (Put with RaidenBlockId-like value)
//   pin K | unpin K | erase K | contains K      -> 1 / 0
//   peek K | peekany K                          -> "H D S" or "-"
//   pins K                                     -> pin count
//   avail | size                               -> number
//   evictable N                                -> keys (space separated) or "-"
#include <iostream>
#include <sstream>
#include <string>
#include <tuple>

#include "tpu_sync/kv_cache/lru_cache.h"

struct Val {
  int h = -1, d = -1, s = 0;
};

int main(int argc, char** argv) {
  size_t cap = argc > 1 ? std::stoul(argv[1]) : 8;
  tpu_raiden::kv_cache::LRUCache<std::string, Val> lru(cap);
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    std::string op, k;
    in >> op;
    if (op == "put") {
      Val v;
      in >> k >> v.h >> v.d >> v.s;
      auto ev = lru.Put(k, v);
      std::cout << (ev ? ev->first : std::string("-")) << "\n";
    } else if (op == "pin") {
      in >> k;
      std::cout << lru.Pin(k) << "\n";
    } else if (op == "unpin") {
      in >> k;
      std::cout << lru.Unpin(k) << "\n";
    } else if (op == "erase") {
      in >> k;
      std::cout << lru.Erase(k) << "\n";
    } else if (op == "contains") {
      in >> k;
      std::cout << lru.Contains(k) << "\n";
    } else if (op == "peek" || op == "peekany") {
      in >> k;
      const Val* v = op == "peek" ? lru.Peek(k) : lru.PeekIncludingCandidates(k);
      if (v) std::cout << v->h << " " << v->d << " " << v->s << "\n";
      else std::cout << "-\n";
    } else if (op == "pins") {
      in >> k;
      std::cout << lru.GetPinCount(k) << "\n";
    } else if (op == "avail") {
      std::cout << lru.available_space() << "\n";
    } else if (op == "size") {
      std::cout << lru.size() << "\n";
    } else if (op == "evictable") {
      size_t n;
      in >> n;
      auto keys = lru.GetEvictableKeys(n);
      if (keys.empty()) std::cout << "-";
      for (size_t i = 0; i < keys.size(); ++i) std::cout << (i ? " " : "") << keys[i];
      std::cout << "\n";
    } else {
      std::cout << "?\n";
    }
  }
  return 0;
}

// Minimal stand-in for absl::HashOf used ONLY to compile reference sources
// as test oracles (oracle/build_ref.py).  Combines std::hash values.
#pragma once
#include <cstddef>
#include <functional>

namespace absl {

template <typename... Ts>
size_t HashOf(const Ts&... values) {
  size_t h = 0;
  ((h = h * 1000003u ^ std::hash<Ts>()(values)), ...);
  return h;
}

}  // namespace absl

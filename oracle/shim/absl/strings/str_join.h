// Minimal stand-in for absl::StrJoin used ONLY to compile reference sources
// as test oracles (oracle/build_ref.py): elements streamed with a separator.
#pragma once
#include <sstream>
#include <string>

namespace absl {

template <typename Range, typename Sep>
std::string StrJoin(const Range& range, const Sep& sep) {
  std::ostringstream os;
  bool first = true;
  for (const auto& v : range) {
    if (!first) os << sep;
    os << v;
    first = false;
  }
  return os.str();
}

}  // namespace absl

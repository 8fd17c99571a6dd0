// Minimal stand-in for absl::string_view used ONLY to compile reference
// sources as test oracles (oracle/build_ref.py).
#pragma once
#include <string_view>

namespace absl {
using string_view = std::string_view;
}  // namespace absl

// Minimal stand-in for absl::StrCat used ONLY to compile the reference's
// pool_layout.cc as a test oracle (oracle/build_ref.py): decimal integers,
// strings and C strings concatenated.
#pragma once
#include <sstream>
#include <string>

namespace absl {

template <typename... Args>
std::string StrCat(const Args&... args) {
  std::ostringstream os;
  (os << ... << args);
  return os.str();
}

}  // namespace absl

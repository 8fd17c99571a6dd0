// Minimal stand-in for absl::StrCat / StrAppend used ONLY to compile
// reference sources as test oracles (oracle/build_ref.py): decimal integers,
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

template <typename... Args>
void StrAppend(std::string* out, const Args&... args) {
  out->append(StrCat(args...));
}

}  // namespace absl

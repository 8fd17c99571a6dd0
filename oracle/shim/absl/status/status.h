// Minimal stand-in for absl::Status used ONLY to compile the reference's
// reference sources as test oracles (oracle/build_ref.py).  Carries a code and
// a message; codes are absl::StatusCode's numeric values.
#pragma once
#include <string>
#include <utility>

namespace absl {

enum class StatusCode : int {
  kOk = 0, kInvalidArgument = 3, kNotFound = 5, kFailedPrecondition = 9,
  kResourceExhausted = 8, kOutOfRange = 11, kInternal = 13,
};

class Status {
 public:
  Status() = default;
  Status(StatusCode c, std::string m) : code_(c), msg_(std::move(m)) {}
  bool ok() const { return code_ == StatusCode::kOk; }
  StatusCode code() const { return code_; }
  const std::string& message() const { return msg_; }
  std::string ToString() const { return msg_; }

 private:
  StatusCode code_ = StatusCode::kOk;
  std::string msg_;
};

inline Status OkStatus() { return Status(); }
inline Status InvalidArgumentError(std::string m) { return Status(StatusCode::kInvalidArgument, std::move(m)); }
inline Status OutOfRangeError(std::string m) { return Status(StatusCode::kOutOfRange, std::move(m)); }
inline Status InternalError(std::string m) { return Status(StatusCode::kInternal, std::move(m)); }
inline Status ResourceExhaustedError(std::string m) { return Status(StatusCode::kResourceExhausted, std::move(m)); }
inline Status FailedPreconditionError(std::string m) { return Status(StatusCode::kFailedPrecondition, std::move(m)); }

}  // namespace absl

// Minimal stand-in for absl::StatusOr used ONLY to compile the reference's
// pool_layout.cc as a test oracle (oracle/build_ref.py).
#pragma once
#include <optional>
#include <utility>

#include "absl/status/status.h"

namespace absl {

template <typename T>
class StatusOr {
 public:
  StatusOr(Status s) : status_(std::move(s)) {}  // NOLINT: implicit like absl
  StatusOr(T v) : value_(std::move(v)) {}         // NOLINT
  template <typename U>
  StatusOr(U&& v) : value_(T(std::forward<U>(v))) {}  // NOLINT
  bool ok() const { return value_.has_value(); }
  const Status& status() const { return status_; }
  T& operator*() { return *value_; }
  const T& operator*() const { return *value_; }
  T* operator->() { return &*value_; }
  const T* operator->() const { return &*value_; }
  T& value() { return *value_; }

 private:
  Status status_;
  std::optional<T> value_;
};

}  // namespace absl

// Minimal stand-in for absl::Span used ONLY to compile the reference's
// pool_layout.cc as a test oracle (oracle/build_ref.py): a read-only view of
// a vector or an initializer list.
#pragma once
#include <cstddef>
#include <initializer_list>
#include <type_traits>
#include <vector>

namespace absl {

template <typename T>
class Span {
 public:
  using V = std::remove_const_t<T>;
  Span() = default;
  Span(const std::vector<V>& v) : p_(v.data()), n_(v.size()) {}         // NOLINT
  Span(std::initializer_list<V> l) : p_(l.begin()), n_(l.size()) {}      // NOLINT
  Span(const V* p, size_t n) : p_(p), n_(n) {}
  const V* begin() const { return p_; }
  const V* end() const { return p_ + n_; }
  size_t size() const { return n_; }
  const V& operator[](size_t i) const { return p_[i]; }

 private:
  const V* p_ = nullptr;
  size_t n_ = 0;
};

template <typename T>
Span<T> MakeSpan(std::vector<T>& v) { return Span<T>(v); }

}  // namespace absl

// Minimal stand-in for absl::Span used ONLY to compile reference sources as
// test oracles (oracle/build_ref.py): a view of a vector, an initializer
// list or a pointer range; mutable when T is not const.
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
  Span(std::vector<V>& v) : p_(v.data()), n_(v.size()) {}               // NOLINT
  template <typename U = T, typename = std::enable_if_t<std::is_const_v<U>>>
  Span(const std::vector<V>& v) : p_(v.data()), n_(v.size()) {}         // NOLINT
  template <typename U = T, typename = std::enable_if_t<std::is_const_v<U>>>
  Span(std::initializer_list<V> l) : p_(l.begin()), n_(l.size()) {}      // NOLINT
  Span(T* p, size_t n) : p_(p), n_(n) {}
  T* data() const { return p_; }
  T* begin() const { return p_; }
  T* end() const { return p_ + n_; }
  size_t size() const { return n_; }
  bool empty() const { return n_ == 0; }
  T& operator[](size_t i) const { return p_[i]; }
  Span subspan(size_t pos, size_t len = size_t(-1)) const {
    const size_t p = pos < n_ ? pos : n_;
    const size_t l = len < n_ - p ? len : n_ - p;
    return Span(p_ + p, l);
  }

 private:
  T* p_ = nullptr;
  size_t n_ = 0;
};

template <typename T>
Span<T> MakeSpan(std::vector<T>& v) { return Span<T>(v); }
template <typename T>
Span<T> MakeSpan(T* p, size_t n) { return Span<T>(p, n); }

}  // namespace absl

// Minimal stand-in for absl::Mutex / absl::MutexLock used ONLY to compile
// reference sources as test oracles (oracle/build_ref.py), over std::mutex.
#pragma once
#include <mutex>

#include "absl/base/thread_annotations.h"

namespace absl {

class Mutex {
 public:
  void Lock() { m_.lock(); }
  void Unlock() { m_.unlock(); }
  void AssertHeld() const {}

 private:
  std::mutex m_;
};

class MutexLock {
 public:
  explicit MutexLock(Mutex* m) : m_(m) { m_->Lock(); }
  explicit MutexLock(Mutex& m) : m_(&m) { m_->Lock(); }
  ~MutexLock() { m_->Unlock(); }
  MutexLock(const MutexLock&) = delete;
  MutexLock& operator=(const MutexLock&) = delete;

 private:
  Mutex* m_;
};

}  // namespace absl

// Stand-in for absl's thread-safety annotation macros used ONLY to compile
// reference sources as test oracles (oracle/build_ref.py): all expand to nothing.
#pragma once
#define ABSL_GUARDED_BY(x)
#define ABSL_PT_GUARDED_BY(x)
#define ABSL_LOCK_RETURNED(x)
#define ABSL_EXCLUSIVE_LOCKS_REQUIRED(...)
#define ABSL_SHARED_LOCKS_REQUIRED(...)
#define ABSL_LOCKS_EXCLUDED(...)
#define ABSL_NO_THREAD_SAFETY_ANALYSIS

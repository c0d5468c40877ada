// Kill switches of the C3 path, unchanged from the reference (include/C3/C3Config.h:34-87):
// a compile-time macro CT_C3_DISABLE_* or the environment variable C3_DISABLE_*=1 turns a
// feature off; the environment is read once and cached.
#pragma once

#include <cstdlib>

namespace ct {
namespace c3 {
namespace detail {
inline bool envFlag(const char* name) {
  const char* v = std::getenv(name);
  return v != nullptr && v[0] == '1';
}
}  // namespace detail

inline bool singleKernelInjectionEnabled() {
#ifdef CT_C3_DISABLE_SINGLE_KERNEL
  return false;
#else
  static const bool enabled = !detail::envFlag("C3_DISABLE_SINGLE_KERNEL");
  return enabled;
#endif
}

inline bool regionFusionEnabled() {
#ifdef CT_C3_DISABLE_REGION_FUSION
  return false;
#else
  static const bool enabled = !detail::envFlag("C3_DISABLE_REGION_FUSION");
  return enabled;
#endif
}

inline bool backwardFusionEnabled() {
#ifdef CT_C3_DISABLE_BACKWARD
  return false;
#else
  static const bool enabled = !detail::envFlag("C3_DISABLE_BACKWARD");
  return enabled;
#endif
}

inline bool hotPathTrackingEnabled() {
#ifdef CT_C3_DISABLE_HOTPATH
  return false;
#else
  static const bool enabled = !detail::envFlag("C3_DISABLE_HOTPATH");
  return enabled;
#endif
}

}  // namespace c3
}  // namespace ct

// Minimal stand-in for <glog/logging.h> so the reference's operator sources
// compile unmodified for the GPU oracle (glog is not installed).  Every log
// statement becomes a discarded stream.
#pragma once
#include <ostream>

namespace cuopx_ref_shim {
struct NullStream {
  template <typename T>
  NullStream& operator<<(const T&) { return *this; }
  NullStream& operator<<(std::ostream& (*)(std::ostream&)) { return *this; }
};
}  // namespace cuopx_ref_shim

#define LOG(severity) ::cuopx_ref_shim::NullStream()
#define VLOG(level) ::cuopx_ref_shim::NullStream()
#define LOG_IF(severity, cond) ::cuopx_ref_shim::NullStream()
#define CHECK(cond) ::cuopx_ref_shim::NullStream()
#define DLOG(severity) ::cuopx_ref_shim::NullStream()

namespace google {
inline void InitGoogleLogging(const char*) {}
inline void ShutdownGoogleLogging() {}
}  // namespace google

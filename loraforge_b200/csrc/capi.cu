// C ABI bookkeeping: version and the per-thread last-error message.
#include "common.cuh"

namespace lfb {
std::string& last_error() {
  thread_local std::string message;
  return message;
}
}  // namespace lfb

extern "C" int lf_version(void) { return 100; }  // 0.1.0

extern "C" const char* lf_last_error_string(void) { return lfb::last_error().c_str(); }

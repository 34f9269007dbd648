// Host-side plumbing of the C ABI: thread-local error text and the version probe.
#include "hl_common.cuh"

namespace hl {

namespace {
thread_local char g_error[512] = {0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_error[0] = 0; }

}  // namespace hl

extern "C" const char* hl_last_error_string(void) { return hl::g_error; }

extern "C" int hl_version(void) { return 1; }

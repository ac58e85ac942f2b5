// Thread-local error message behind tw_last_error().
#include "common.cuh"

namespace tw {

namespace {
thread_local char g_error[512] = {0};
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

}  // namespace tw

extern "C" const char* tw_last_error(void) { return tw::g_error; }
extern "C" int tw_abi_version(void) { return 100; }

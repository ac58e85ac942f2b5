// Thread-local error message behind tw_last_error(), and the FFN kernels' wait limit.
#include <atomic>

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

namespace {
constexpr uint32_t kDefaultWaitLimit = 1u << 24;  // the kernels' own cap (tc_common.cuh)
std::atomic<uint32_t> g_wait_limit{kDefaultWaitLimit};
}  // namespace

uint32_t ffn_wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

}  // namespace tw

extern "C" const char* tw_last_error(void) { return tw::g_error; }

extern "C" int tw_set_wait_limit(uint32_t polls) {
  tw::g_wait_limit.store(polls == 0 ? tw::kDefaultWaitLimit : polls, std::memory_order_relaxed);
  return TW_OK;
}
extern "C" int tw_abi_version(void) { return 103; }

// Library-wide entry points: the thread-local error message and the ABI version.
#include <atomic>

#include "common.cuh"

namespace vb {
namespace {
thread_local char g_error[1024] = "";
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_error[0] = '\0'; }

namespace {
std::atomic<unsigned long long> g_launches{0};
}
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace vb

extern "C" const char* vb_last_error(void) { return vb::g_error; }

extern "C" int vb_abi_version(void) { return 1; }

extern "C" unsigned long long vb_launch_count(void) {
  return vb::g_launches.load(std::memory_order_relaxed);
}

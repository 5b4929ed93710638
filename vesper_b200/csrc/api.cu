// Library-wide entry points: the thread-local error message and the ABI version.
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
}  // namespace vb

extern "C" const char* vb_last_error(void) { return vb::g_error; }

extern "C" int vb_abi_version(void) { return 1; }

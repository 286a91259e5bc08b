// Per-thread error message behind pa_last_error(), and the ABI revision.
#include "capi_util.h"

namespace pa {
namespace {
thread_local std::string g_last_error;
}

void set_error(const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

void clear_error() { g_last_error.clear(); }

}  // namespace pa

extern "C" const char* pa_last_error(void) { return pa::g_last_error.c_str(); }

extern "C" int pa_abi_version(void) { return 8; }

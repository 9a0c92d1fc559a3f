// Library-wide C ABI helpers: error text and ABI revision.
#include "common.cuh"

namespace tread {

static thread_local char g_last_error[512] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

}  // namespace tread

extern "C" const char* tread_last_error(void) { return tread::g_last_error; }

extern "C" int tread_abi_version(void) { return 5; }

// Library-level C ABI: version and per-thread error text.
#include "common.cuh"

#include <string.h>

namespace mrb {

static thread_local char g_last_error[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_last_error[0] = 0; }

}  // namespace mrb

extern "C" int mrb_abi_version(void) { return 3; }

extern "C" const char* mrb_last_error(void) { return mrb::g_last_error; }

// Error reporting and version of the C-ABI (include/pgf.h).
#include "common.cuh"

#include <string.h>

namespace pgf {

static thread_local char g_err[1024] = {0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

}  // namespace pgf

extern "C" const char* pgf_last_error(void) { return pgf::g_err; }

extern "C" int pgf_version(void) { return 100; /* 0.1.0 */ }

// capi.cu -- error reporting and version of the C ABI (include/mfd_b200.h).
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace mfd {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

}  // namespace mfd

extern "C" const char* mfd_last_error(void) { return mfd::g_error; }

extern "C" int mfd_abi_version(void) { return 1; }

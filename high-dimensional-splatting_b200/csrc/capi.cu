// capi.cu -- C ABI support: thread-local error text and the ABI version.
#include <cstring>

#include "hds_common.cuh"

namespace hds {

namespace {
thread_local char g_error[512];
}

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_error, sizeof(g_error), fmt, ap);
    va_end(ap);
}

void clear_error() { g_error[0] = '\0'; }

}  // namespace hds

extern "C" const char* hds_last_error(void) { return hds::g_error; }

extern "C" int hds_abi_version(void) { return HDS_ABI_VERSION; }

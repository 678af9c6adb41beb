// capi.cu -- C ABI support: thread-local error text and the ABI version.
#include <atomic>
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

namespace {
std::atomic<unsigned long long> g_launches{0};
}

void note_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

}  // namespace hds

extern "C" const char* hds_last_error(void) { return hds::g_error; }

extern "C" int hds_abi_version(void) { return HDS_ABI_VERSION; }

extern "C" unsigned long long hds_launch_count(void) { return hds::g_launches.load(std::memory_order_relaxed); }

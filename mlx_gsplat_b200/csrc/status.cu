// Error reporting of the C ABI: one message buffer per host thread.
#include "common.cuh"

#include <atomic>

namespace gs {
static thread_local char g_msg[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void note_launches(int n) { g_launches.fetch_add((unsigned long long)n, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return code;
}
}  // namespace gs

extern "C" const char* gs_last_error(void) { return gs::g_msg; }
extern "C" int gs_abi_version(void) { return 3; }
extern "C" unsigned long long gs_kernel_launches(void) { return gs::g_launches.load(std::memory_order_relaxed); }

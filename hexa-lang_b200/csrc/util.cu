// util.cu — error reporting and device queries shared by the library.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include "forge_internal.h"

namespace {
thread_local char g_last_error[512] = "";
int g_sm_count[64] = {0};
}  // namespace

int forge_fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    fprintf(stderr, "[forge_b200] %s\n", g_last_error);
    return code;
}

int forge_check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return forge_fail(-1, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return 0;
}

int forge_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!g_sm_count[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        g_sm_count[dev] = n;
    }
    return g_sm_count[dev];
}

extern "C" FORGE_API const char* forge_b200_last_error(void) { return g_last_error; }
extern "C" FORGE_API uint32_t forge_api_version_v2(void) { return 0x00020000u; }

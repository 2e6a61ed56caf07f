// C-ABI plumbing: the per-thread error message and version query.
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

namespace f2s {

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess)
        return fail(F2S_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(err));
    return F2S_OK;
}

int sm_count() {
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace f2s

extern "C" const char* f2s_last_error(void) { return g_last_error; }

extern "C" int f2s_version(void) { return 100; }

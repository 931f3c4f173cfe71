// Error reporting and device queries of the C ABI (include/t2c_sm100.h).
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace t2c {

static thread_local char g_last_error[1024] = "";

int set_error(int code, const char *fmt, ...) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, args);
    va_end(args);
    return code;
}

int check_launch(const char *what) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        return set_error(T2C_ECUDA, "%s: %s", what, cudaGetErrorString(err));
    }
    return T2C_OK;
}

int sm_count() {
    static thread_local int cached_device = -1;
    static thread_local int cached_count = 0;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 148;
    if (device != cached_device) {
        int count = 0;
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || count <= 0) {
            count = 148;
        }
        cached_device = device;
        cached_count = count;
    }
    return cached_count;
}

}  // namespace t2c

extern "C" const char *t2c_last_error(void) { return t2c::g_last_error; }

extern "C" int t2c_abi_version(void) { return 1; }

extern "C" int t2c_device_sm_count(void) { return t2c::sm_count(); }

// Error reporting and device queries of the C ABI (include/t2c_sm100.h).
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace t2c {

cudaError_t status_qlinear(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_decode(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_surface(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_qgemm(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_comm(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_asr(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_qbatch(unsigned int *bits, int clear, cudaStream_t s);
cudaError_t status_attn_tc(unsigned int *bits, int clear, cudaStream_t s);

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

extern "C" int t2c_device_status(unsigned int *bits, int clear, void *stream) {
    if (bits == nullptr) return t2c::set_error(T2C_EINVAL, "t2c_device_status: bits is NULL");
    cudaStream_t s = t2c::as_stream(stream);
    unsigned int value = 0;
    cudaError_t err = t2c::status_qlinear(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_decode(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_surface(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_qgemm(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_comm(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_asr(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_qbatch(&value, clear, s);
    if (err == cudaSuccess) err = t2c::status_attn_tc(&value, clear, s);
    if (err != cudaSuccess) return t2c::set_error(T2C_ECUDA, "t2c_device_status: %s", cudaGetErrorString(err));
    *bits = value;
    return T2C_OK;
}

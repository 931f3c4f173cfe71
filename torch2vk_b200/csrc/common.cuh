// Shared helpers for the sm_100a kernels of libt2c_sm100.so: status/error
// reporting for the C ABI, fp16 bit helpers, and the few PTX instructions the
// kernels use directly.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/t2c_sm100.h"

namespace t2c {

// Records a message for t2c_last_error() and returns `code`.
int set_error(int code, const char *fmt, ...);
int check_launch(const char *what);

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

int sm_count();

// Bytes per packed row of K values for a GGUF weight type, or -1.
inline int64_t row_bytes(int wtype, int64_t K) {
    switch (wtype) {
        case T2C_Q4_K: return (K % 256) ? -1 : K / 256 * 144;
        case T2C_Q6_K: return (K % 256) ? -1 : K / 256 * 210;
        case T2C_Q8_0: return (K % 32) ? -1 : K / 32 * 34;
        case T2C_F16: return K * 2;
        default: return -1;
    }
}

__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

// d = dot(a bytes as u8, b bytes as s8) + c
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// d = dot(a bytes as s8, b bytes as s8) + c
__device__ __forceinline__ int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_nc_u32(const void *p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ldg_nc_u16(const void *p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// Explicit-width stores.  Packing fp16 bit patterns byte by byte
// (static_cast<uint8_t>(bits & 0xff) of a __half_as_ushort result) was
// observed to store 0 for the low byte with nvcc 12.9 / sm_100a, so fp16
// fields are always written with one 16- or 32-bit store.
__device__ __forceinline__ void st_u16(void *p, uint32_t v) {
    asm volatile("st.u16 [%0], %1;" ::"l"(p), "h"(static_cast<unsigned short>(v)) : "memory");
}
__device__ __forceinline__ void st_u32(void *p, uint32_t v) {
    asm volatile("st.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ------------------------------------------------------------ mbarrier / TMA
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// try_wait (potentially blocking: the thread may be suspended until the phase
// completes or a system-dependent time limit passes).  Measured without a
// suspend-time hint: handoffs between warp roles were 2-5 % faster than with a
// 64 us hint (GEMM chunks, the decode and prefill steps).
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// System-scope release store / acquire load of a u32 (flags shared with peer GPUs).
__device__ __forceinline__ void ar_store_release(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ar_load_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait on an mbarrier phase: false after `limit_ns` without completion.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - start > limit_ns) return false;
    }
}
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`
// (no multicast).  dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load (no multicast) of a box at element coordinates (x, y) of the
// tensor map `tmap` (a __grid_constant__ kernel parameter) into shared memory.
// x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Device-side status word of this translation unit: kernels OR in 1 << T2C_E*
// (e.g. T2C_ETIMEOUT after a bounded wait ran out).  Every .cu file with such
// kernels exposes a reader (status_<file>) that t2c_device_status() combines.
static __device__ unsigned int g_device_status = 0;
__device__ __forceinline__ void report_device_error(unsigned int code) { atomicOr(&g_device_status, 1u << code); }

static inline cudaError_t read_tu_status(unsigned int *bits, int clear, cudaStream_t s) {
    unsigned int value = 0;
    cudaError_t err = cudaMemcpyFromSymbolAsync(&value, g_device_status, sizeof(value), 0, cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess && clear) {
        static const unsigned int zero = 0;
        err = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    }
    if (err == cudaSuccess) *bits |= value;
    return err;
}

// Programmatic dependent launch.  pdl_wait(): block until the preceding
// kernel in the stream has completed and its memory is visible (a no-op when
// launched without the attribute).  pdl_trigger(): allow the next kernel to
// launch now; it still waits in its own pdl_wait() for this kernel to finish,
// so only work that needs nothing from this kernel (weight prefetch) runs
// early.  Every kernel here triggers right after its wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace t2c

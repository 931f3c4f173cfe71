// One-shot all-reduce of small fp16 tensors over NVLink peer memory, for the
// tensor-parallel decode step (the two per-layer reductions of the row-split
// o_proj / down_proj partial sums; a few KB at batch 1).
//
// Every rank owns one buffer, mapped into every other rank by CUDA IPC:
//   [flags: kMaxCtas x kMaxRanks u32][region 0: n_max fp16][region 1: n_max fp16]
// CTA c of the launch reduces its own slice of x and uses flag row c.
// A call with epoch e (a per-rank device counter pair [epoch, arrivals],
// advanced by the kernel itself, so the same launch replays inside a CUDA
// graph) uses region e % 2:
//   1. copy the local partial into the own region e % 2;
//   2. store e into flags[rank] of every peer (release, system scope);
//   3. wait until the own flags[p] >= e for every peer p (acquire; bounded);
//   4. sum region e % 2 of all ranks (fp32) into the local tensor.
// Peers finish reading region e % 2 before they signal epoch e + 1, and a rank
// reuses that region only at epoch e + 2, after it has seen every e + 1 signal,
// so two regions suffice.  Plain peer loads and stores only (no multicast).
// A wait that runs out reports T2C_ETIMEOUT in t2c_device_status and leaves the
// local tensor unreduced.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "common.cuh"

namespace t2c {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 32;
constexpr int kFlagBytes = kMaxCtas * kMaxRanks * 4;
constexpr int kArThreads = 512;

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct PeerBufs {
    uint8_t *base[kMaxRanks];
};

__global__ void __launch_bounds__(kArThreads) allreduce_f16_kernel(__half *x, int64_t n, PeerBufs bufs, int rank,
                                                                   int tp, uint32_t *counter, int64_t n_max) {
    __shared__ uint32_t epoch_s;
    __shared__ int ok_s;
    pdl_wait();
    pdl_trigger();
    if (threadIdx.x == 0) {
        epoch_s = counter[0] + 1;  // counter[0] moves on only after every CTA of this launch has read it
        ok_s = 1;
    }
    __syncthreads();
    const uint32_t epoch = epoch_s;
    const int64_t region = kFlagBytes / 2 + static_cast<int64_t>(epoch & 1u) * n_max;  // in halves
    __half *mine = reinterpret_cast<__half *>(bufs.base[rank]) + region;
    // this CTA's slice, in units of 8 halves
    const int64_t units = n / 8, per = (units + gridDim.x - 1) / gridDim.x;
    const int64_t u0 = blockIdx.x * per, u1 = min(units, u0 + per);
    // 1. local partial into the own region
    for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x)
        *reinterpret_cast<uint4 *>(mine + 8 * u) = *reinterpret_cast<const uint4 *>(x + 8 * u);
    __syncthreads();
    // 2. signal every peer, 3. wait for every peer
    if (threadIdx.x < tp) {
        const int p = threadIdx.x;
        // a system-scope release: the CTA's copies are ordered before it by the barrier above
        st_release_sys(reinterpret_cast<uint32_t *>(bufs.base[p]) + blockIdx.x * kMaxRanks + rank, epoch);
        const uint32_t *flag = reinterpret_cast<const uint32_t *>(bufs.base[rank]) + blockIdx.x * kMaxRanks + p;
        if (ld_acquire_sys(flag) < epoch) {
            const uint64_t start = global_timer_ns();
            while (ld_acquire_sys(flag) < epoch) {
                if (global_timer_ns() - start > 1000000000ull) {
                    ok_s = 0;
                    report_device_error(T2C_ETIMEOUT);
                    break;
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // counter[1] counts the CTAs of this launch past their read of counter[0]; the last one advances it
        __threadfence();
        if (atomicAdd(&counter[1], 1u) == gridDim.x - 1) {
            counter[1] = 0u;
            counter[0] = epoch;
        }
    }
    if (!ok_s) return;
    // 4. sum the tp regions (volatile loads: never a stale L1 line of a peer's region)
    for (int64_t u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
        const int64_t i = 8 * u;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < tp; ++p) {
            const uint4 v = __ldcv(reinterpret_cast<const uint4 *>(reinterpret_cast<const __half *>(bufs.base[p]) + region + i));
            const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(h[e]);
                acc[2 * e] += f.x;
                acc[2 * e + 1] += f.y;
            }
        }
        uint4 o;
        __half2 *h = reinterpret_cast<__half2 *>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2half2_rn(acc[2 * e], acc[2 * e + 1]);
        *reinterpret_cast<uint4 *>(x + i) = o;
    }
}

}  // namespace

cudaError_t status_comm(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c

using namespace t2c;

extern "C" int64_t t2c_allreduce_buffer_bytes(int64_t n_max) { return kFlagBytes + 2 * n_max * 2; }

// IPC handle of the allocation holding `ptr` and the byte offset of `ptr` in it.
extern "C" int t2c_ipc_get_handle(const void *ptr, void *handle64, int64_t *offset) {
    if (!ptr || !handle64 || !offset) return set_error(T2C_EINVAL, "ipc_get_handle: NULL pointer");
    static PFN_cuMemGetAddressRange range = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuMemGetAddressRange>(fn);
    }();
    if (range == nullptr) return set_error(T2C_ECUDA, "ipc_get_handle: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
        return set_error(T2C_ECUDA, "ipc_get_handle: cuMemGetAddressRange failed");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
    if (e != cudaSuccess) return set_error(T2C_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    static_assert(sizeof(h) == 64, "IPC handle size");
    memcpy(handle64, &h, 64);
    *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
    return T2C_OK;
}

extern "C" int t2c_ipc_open_handle(const void *handle64, void **ptr) {
    if (!handle64 || !ptr) return set_error(T2C_EINVAL, "ipc_open_handle: NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle64, 64);
    const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return set_error(T2C_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
    return T2C_OK;
}

extern "C" int t2c_ipc_close_handle(void *ptr) {
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return set_error(T2C_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
    return T2C_OK;
}

extern "C" int t2c_allreduce_sum_f16(void *x, int64_t n, void *const *bufs, int rank, int tp, uint32_t *counter,
                                     int64_t n_max, void *stream) {
    if (!x || !bufs || !counter || tp < 1 || tp > kMaxRanks || rank < 0 || rank >= tp)
        return set_error(T2C_EINVAL, "allreduce: bad argument");
    if (n <= 0 || n > n_max || n % 8)
        return set_error(T2C_EINVAL, "allreduce: n=%lld must be a multiple of 8 in 1..%lld", (long long)n, (long long)n_max);
    if (reinterpret_cast<uintptr_t>(x) % 16 || n_max % 8) return set_error(T2C_EINVAL, "allreduce: x must be 16-byte aligned");
    PeerBufs pb = {};
    for (int p = 0; p < tp; ++p) {
        if (!bufs[p] || reinterpret_cast<uintptr_t>(bufs[p]) % 256) return set_error(T2C_EINVAL, "allreduce: bad peer buffer");
        pb.base[p] = static_cast<uint8_t *>(bufs[p]);
    }
    cudaLaunchConfig_t cfg = {};
    int64_t ctas = (n / 8 + kArThreads - 1) / kArThreads;
    if (ctas > kMaxCtas) ctas = kMaxCtas;
    cfg.gridDim = dim3(static_cast<unsigned>(ctas));
    cfg.blockDim = dim3(kArThreads);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, allreduce_f16_kernel, static_cast<__half *>(x), n, pb, rank, tp,
                                             counter, n_max);
    if (e != cudaSuccess) return set_error(T2C_ECUDA, "allreduce launch: %s", cudaGetErrorString(e));
    return T2C_OK;
}

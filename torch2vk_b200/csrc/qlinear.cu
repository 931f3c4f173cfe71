// Quantized linear for decode-sized batches (M <= 8 per launch chunk):
// y[m, n] = sum_k x[m, k] * deq(W)[n, k] over GGUF Q4_K / Q6_K / Q8_0 rows.
//
// Arithmetic (M <= 4) follows the reference matvec shaders
// (src/models/quantized_qwen3/shaders/linear_nobias_q4_k_matvec_f32.py:107-197,
//  linear_nobias_q6_k_matvec_f32.py:116-193, linear_nobias_q8_0_matvec_f32.py:84-119):
// the fp16 x (with a fused RMSNorm: the normalized values rounded to fp16
// once, as the reference's fp16 activation tensor) times the decoded weight,
// accumulated in fp32.  The products run on fp16 tensor cores (mma.sync
// m16n8k16, fp32 accumulators) with every weight code entering as an exactly
// representable fp16 value (Q4_K nibbles as subnormals q * 2^-24, Q6_K levels
// L - 32 and Q8_0 codes as small integers) and the block scales applied in
// fp32; only the summation order differs from the reference's fp32 loop.
//
// B200 design (HBM-bound):
//  * qmv_m1_kernel (Q4_K, M = 1): per-warp rings of 16-row x 288-byte 2-D TMA
//    boxes (bounded mbarrier waits, weights requested before
//    griddepcontrol.wait), K split over the warps of a CTA, mma columns = the
//    sub-blocks of a block so each lane scales its own partial sums.
//  * qmv_mma_kernel (Q4_K, M = 2..4): the same streaming, mma columns =
//    tokens, sub-block scales folded into the fp16 A operand exactly.
//  * qmv_x16_kernel (any type, up to 4 tokens per pass): direct global loads,
//    16-row tiles, the sparse-column mapping of the M = 1 kernel.
//  * qmv_tma_kernel / qmv_direct_kernel: dp4a on 15-bit fixed-point x planes;
//    kept only for M > 4 shapes the tensor-core GEMM does not take (Q6_K with
//    K % 2048 != 0 and N % 8 != 0, Q8_0 with K % 256 != 0).
//  * Epilogues: + residual (matvec_add), silu(gate) * up (SwiGLU pair),
//    per-4-row argmax partials (LM head), fp16 store.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdio.h>

#include "qgemm.cuh"

#include "common.cuh"

namespace t2c {
namespace {

constexpr int kThreads = 128;  // x-prologue / consumer threads
constexpr int kWarps = kThreads / 32;
constexpr int kMaxStreams = 3;
constexpr int kMaxStages = 8;

enum Mode : int { MODE_ROWS = 0, MODE_SWIGLU = 1, MODE_ARGMAX = 2 };

struct QStream {
    const uint8_t *w;
    __half *y;
    const __half *res;
    int64_t n;
    int64_t row_bytes;
    int64_t rs_begin;  // first row-set (direct) / row block (streamed) index of this stream
    int fmt;
    // streamed-kernel geometry
    int rb;            // rows per row block (SwiGLU: gate + up rows)
    int seg_blocks;    // GGUF blocks per staged row segment
    int seg_bytes;     // bytes per staged row segment
    int chunks;        // segments per row (K / (seg_blocks * block_values))
    int lpr;           // lanes per row group
    int whole;         // 1: a stage is rb full contiguous rows (one copy)
};

struct QParams {
    // tensor-core kernel: 2-D TMA maps of the Q4_K weights (u32 words, [N, row_bytes / 4],
    // box 72 x 16 = 16 rows x one 288-byte segment)
    alignas(64) CUtensorMap tmap[kMaxStreams];
    QStream s[kMaxStreams];
    int nstreams;
    int mode;
    const __half *x;
    const float *norm_w;
    float eps;
    int M;         // tokens in this launch chunk (<= MT)
    int K;
    int units;     // 64-value units per row (direct kernel)
    int lpr;       // lanes per row-set (direct kernel)
    int64_t total_rowsets;  // direct: row-sets; streamed: row blocks
    int stages;
    int stage_bytes;
    // MODE_ARGMAX: best (score, row) per group of 4 rows, [M, G]
    float *ps;
    uint32_t *pt;
    int64_t G;
    // tensor-core kernel: row-block groups of wpb warps, bpc groups per CTA, nseg segments per row
    int wpb;
    int bpc;
    int nseg;
    int xseg_per_warp;  // M = 1 kernel: x segments held per warp
    // M = 1 kernel, row-parallel tensor parallelism: the output summed over ar_tp ranks in the
    // epilogue (ar_tp < 2: off).  ar_peer[r]: rank r's IPC-mapped buffer (flags, two fp32 regions)
    uint8_t *ar_peer[8];
    uint32_t *ar_counter;  // this rank's [epoch, arrivals]
    int ar_rank, ar_tp;
    int64_t ar_nmax;
};

// Fused row-parallel reduction buffer of a rank:
//   [flags: kArMaxCtas x kArMaxRanks u32][parity 0: kArMaxRanks slots of n_max fp32][parity 1: same]
// slot s of a parity region holds rank s's partials, pushed there by rank s.
constexpr int kArMaxRanks = 8;
constexpr int kArMaxCtas = 512;
constexpr int kArMaxRows = 16384;
constexpr int64_t kArFlagBytes = static_cast<int64_t>(kArMaxCtas) * kArMaxRanks * 4;

// x planes in shared memory.  xh/xl rows are padded by 16 bytes after every
// 64 values (row stride KP = K * 5 / 4) so that the 16-byte fragments that
// consecutive lanes read for consecutive 64-value units fall in distinct
// banks.
struct XPlanes {
    const int8_t *xh;    // [MT][KP]
    const int8_t *xl;    // [MT][KP]
    const float *sx;     // [MT][K/32]
    const int *xq16;     // [MT][K/16] integer sums of (128 xh + xl) over 16 values
    const float4 *meta;  // [MT][K/64]: sx[2u], sx[2u+1], xsum[2u], xsum[2u+1]
    int kp;
    __device__ __forceinline__ int off(int m, int k) const { return m * kp + k + ((k >> 6) << 4); }
};

__host__ __device__ __forceinline__ int padded_k(int K) { return K + (K >> 2); }

// ------------------------------------------------------------- loads
template <bool SMEM>
__device__ __forceinline__ uint4 ld_v4(const uint8_t *p) {
    if constexpr (SMEM) {
        uint4 v;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                     : "r"(smem_u32(p)));
        return v;
    } else {
        return ldg_nc_v4(p);
    }
}
template <bool SMEM>
__device__ __forceinline__ uint32_t ld_u32(const uint8_t *p) {
    if constexpr (SMEM) {
        uint32_t v;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)));
        return v;
    } else {
        return ldg_nc_u32(p);
    }
}
template <bool SMEM>
__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) {
    if constexpr (SMEM) {
        unsigned short v;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(smem_u32(p)));
        return v;
    } else {
        return ldg_nc_u16(p);
    }
}

// 16 bytes starting at a 2-byte aligned address (aligned words + funnel shift).
template <bool SMEM>
__device__ __forceinline__ uint4 ld16_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint8_t *base = reinterpret_cast<const uint8_t *>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3) * 8u;
    const uint32_t w0 = ld_u32<SMEM>(base), w1 = ld_u32<SMEM>(base + 4), w2 = ld_u32<SMEM>(base + 8);
    const uint32_t w3 = ld_u32<SMEM>(base + 12);
    const uint32_t w4 = sh ? ld_u32<SMEM>(base + 16) : 0u;
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

// ---------------------------------------------------------------- x prologue
// Chunks of 8 fp16 values (16 bytes).  Thread t owns chunks t, t + kThreads,
// ...; the four chunks of a 32-value sub-block sit on four consecutive lanes,
// so sub-block maxima and 16-value sums are two/one xor-shuffles away.  Loads
// are issued kRound chunks at a time so their latencies overlap.  Only the
// kThreads consumer threads run this (CONSUMER_BAR: sync on named barrier 1).
constexpr int kRound = 4;

__device__ __forceinline__ void unpack8(const uint4 &v, float f[8]) {
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

template <int MT, int NT>
__device__ __forceinline__ void sync_threads_nt() {
    if constexpr (NT == kThreads) {
        __syncthreads();
    } else {
        asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
    }
}

// NT threads (0..NT-1) build the x planes; ends with a barrier over them.
template <int MT, int NT>
__device__ void prepare_x(const QParams &p, int8_t *xh, int8_t *xl, float *sx, int *xq16, float4 *meta, float *red) {
    constexpr int kThreads = NT;
    constexpr int kWarps = NT / 32;
    const int K = p.K;
    const int KP = padded_k(K);
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int chunks_per_row = K >> 3;
    const int total = MT * chunks_per_row;
    const uint4 *xv = reinterpret_cast<const uint4 *>(p.x);
    float inv_rms[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) inv_rms[m] = 1.0f;
    if (p.norm_w != nullptr) {
        float ss[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ss[m] = 0.0f;
        for (int base = 0; base < total; base += kThreads * kRound) {
            uint4 v[kRound];
#pragma unroll
            for (int i = 0; i < kRound; ++i) {
                const int c = base + i * kThreads + tid;
                const int m = c / chunks_per_row;
                v[i] = (c < total && m < p.M) ? xv[c] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < kRound; ++i) {
                const int c = base + i * kThreads + tid;
                const int m = c / chunks_per_row;
                float f[8];
                unpack8(v[i], f);
                float part = 0.0f;
#pragma unroll
                for (int e = 0; e < 8; ++e) part = fmaf(f[e], f[e], part);
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    if (mm == m) ss[mm] += part;
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[warp * MT + m] = t;
        }
        sync_threads_nt<MT, NT>();
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float t = 0.0f;
            for (int w = 0; w < kWarps; ++w) t += red[w * MT + m];
            inv_rms[m] = rsqrtf(t / static_cast<float>(K) + p.eps);
        }
    }
    for (int base = 0; base < total; base += kThreads * kRound) {
        uint4 v[kRound];
#pragma unroll
        for (int i = 0; i < kRound; ++i) {
            const int c = base + i * kThreads + tid;
            const int m = c / chunks_per_row;
            v[i] = (c < total && m < p.M) ? xv[c] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kRound; ++i) {
            const int c = base + i * kThreads + tid;
            if (base + i * kThreads >= total) break;  // uniform across the CTA
            const int m = c / chunks_per_row;
            const int k = (c - m * chunks_per_row) * 8;
            float f[8];
            unpack8(v[i], f);
            if (p.norm_w != nullptr && c < total) {
                float r = 1.0f;
#pragma unroll
                for (int mm = 0; mm < MT; ++mm)
                    if (mm == m) r = inv_rms[mm];
                const float4 w0 = *reinterpret_cast<const float4 *>(p.norm_w + k);
                const float4 w1 = *reinterpret_cast<const float4 *>(p.norm_w + k + 4);
                const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = f[e] * r * wv[e];
            }
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(f[e]));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            const float inv = amax > 0.0f ? 16383.0f / amax : 0.0f;
            uint32_t hw[2] = {0u, 0u}, lw[2] = {0u, 0u};
            int sum = 0;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                int q = __float2int_rn(f[e] * inv);
                q = max(-16383, min(16383, q));
                sum += q;
                hw[e >> 2] |= (static_cast<uint32_t>(q >> 7) & 0xffu) << (8 * (e & 3));
                lw[e >> 2] |= (static_cast<uint32_t>(q & 127)) << (8 * (e & 3));
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            if (c < total) {
                const int o = m * KP + k + ((k >> 6) << 4);
                *reinterpret_cast<uint2 *>(xh + o) = make_uint2(hw[0], hw[1]);
                *reinterpret_cast<uint2 *>(xl + o) = make_uint2(lw[0], lw[1]);
                if ((lane & 1) == 0) xq16[c >> 1] = sum;
                if ((lane & 3) == 0) sx[c >> 2] = amax / 16383.0f;
            }
        }
    }
    sync_threads_nt<MT, NT>();
    // per-64-value unit metadata (two sub-blocks)
    const int units = MT * (K >> 6);
    for (int u = tid; u < units; u += NT) {
        const float s0 = sx[2 * u], s1 = sx[2 * u + 1];
        const float x0 = s0 * static_cast<float>(xq16[4 * u] + xq16[4 * u + 1]);
        const float x1 = s1 * static_cast<float>(xq16[4 * u + 2] + xq16[4 * u + 3]);
        meta[u] = make_float4(s0, s1, x0, x1);
    }
    sync_threads_nt<MT, NT>();
}

__device__ __forceinline__ uint32_t pack_half2_bits(__half lo, __half hi) {
    return static_cast<uint32_t>(__half_as_ushort(lo)) | (static_cast<uint32_t>(__half_as_ushort(hi)) << 16);
}

// fp16 x of the 2..4-token tensor-core kernel.  Per batch row, the K values
// rounded to fp16 once (as the reference's fp16 activations) in
// pair-interleaved 4-value chunks (x0, x2, x1, x3), with 16 bytes of padding
// after every 16 chunks (the B fragments of the four lanes of a quad then
// fall in distinct banks): row stride xf_row_bytes(K).  Then per row and
// super-block the 8 sub-block sums as fp16 pairs (hi[8], lo[8]) with
// hi = fp16(sum), lo = fp16(sum - hi), the B operand of the min-term mma.
__host__ __device__ __forceinline__ int xf_row_bytes(int K) { return 2 * K + (K >> 6) * 16; }
__host__ __device__ __forceinline__ int xf_chunk_off(int c) { return 8 * c + 16 * (c >> 4); }

template <int MT, int NT>
__device__ void prepare_x_f16(const QParams &p, uint8_t *xperm, uint8_t *xsum, float *red) {
    const int K = p.K;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    constexpr int kW = NT / 32;
    const int chunks_per_row = K >> 3;
    const int total = MT * chunks_per_row;
    const uint4 *xv = reinterpret_cast<const uint4 *>(p.x);
    const int rb = xf_row_bytes(K), sb_per_row = K >> 8;
    float inv_rms[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) inv_rms[m] = 1.0f;
    if (p.norm_w != nullptr) {
        float ss[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ss[m] = 0.0f;
        for (int c = tid; c < total; c += NT) {
            const int m = c / chunks_per_row;
            if (m >= p.M) continue;
            float f[8];
            unpack8(xv[c], f);
            float part = 0.0f;
#pragma unroll
            for (int e = 0; e < 8; ++e) part = fmaf(f[e], f[e], part);
#pragma unroll
            for (int mm = 0; mm < MT; ++mm)
                if (mm == m) ss[mm] += part;
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float t = warp_sum(ss[m]);
            if (lane == 0) red[warp * MT + m] = t;
        }
        sync_threads_nt<MT, NT>();
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float t = 0.0f;
            for (int w = 0; w < kW; ++w) t += red[w * MT + m];
            inv_rms[m] = rsqrtf(t / static_cast<float>(K) + p.eps);
        }
    }
    // NT and chunks_per_row are multiples of 4, so lanes 4i .. 4i + 3 always
    // hold the four 8-value chunks of one 32-value sub-block
    for (int base = 0; base < total; base += NT) {
        const int c = base + tid;
        const int m = c / chunks_per_row;
        const int k = (c - m * chunks_per_row) * 8;
        float f[8];
        if (c < total && m < p.M) {
            unpack8(xv[c], f);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.0f;
        }
        if (p.norm_w != nullptr && c < total) {
            float r = 1.0f;
#pragma unroll
            for (int mm = 0; mm < MT; ++mm)
                if (mm == m) r = inv_rms[mm];
            const float4 w0 = *reinterpret_cast<const float4 *>(p.norm_w + k);
            const float4 w1 = *reinterpret_cast<const float4 *>(p.norm_w + k + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * r * wv[e];
        }
        __half h[8];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            h[e] = __float2half_rn(f[e]);
            sum += __half2float(h[e]);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (c < total) {
            const int cc = k >> 2;  // first 4-value chunk
            *reinterpret_cast<uint4 *>(xperm + m * rb + xf_chunk_off(cc)) =
                make_uint4(pack_half2_bits(h[0], h[2]), pack_half2_bits(h[1], h[3]), pack_half2_bits(h[4], h[6]),
                           pack_half2_bits(h[5], h[7]));
            if ((lane & 3) == 0) {
                const int j = k >> 5;  // sub-block of the row
                const __half hi = __float2half_rn(sum);
                const __half lo = __float2half_rn(sum - __half2float(hi));
                uint8_t *dst = xsum + (m * sb_per_row + (j >> 3)) * 32 + 2 * (j & 7);
                st_u16(dst, __half_as_ushort(hi));
                st_u16(dst + 16, __half_as_ushort(lo));
            }
        }
    }
    sync_threads_nt<MT, NT>();
}

// ------------------------------------------------------------- Q4_K unit
// Unit = group G (32 bytes) of block b: low nibbles are sub-block 2G
// (k0 .. k0+31), high nibbles sub-block 2G+1 (k0+32 .. k0+63).
// rows[r]: start of the row segment holding block b (nullptr: no row);
// kbase: absolute k of block 0 of the segment.
template <int MT, int NR, bool SMEM>
__device__ __forceinline__ void unit_q4k(const uint8_t *const rows[NR], int b, int G, int kbase, int K,
                                         const XPlanes &xp, float acc[NR][MT]) {
    const int k0 = kbase + b * 256 + G * 64;
    const int j0 = k0 >> 5;
    (void)K;
    uint4 hdr[NR], q0[NR], q1[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (rows[r] != nullptr) {
            const uint8_t *blk = rows[r] + b * 144;
            hdr[r] = ld_v4<SMEM>(blk);
            q0[r] = ld_v4<SMEM>(blk + 16 + G * 32);
            q1[r] = ld_v4<SMEM>(blk + 32 + G * 32);
        } else {
            hdr[r] = make_uint4(0, 0, 0, 0);
            q0[r] = hdr[r];
            q1[r] = hdr[r];
        }
    }
    // 6-bit scale/min codes for sub-blocks 2G and 2G+1 (quantize/vulkan.py:331-342
    // packing), decoded without divergent branches; small integers become
    // floats through the 2^23 mantissa trick.
    const int i0 = (2 * G) & 3;
    const bool low = G < 2;
    float ds0[NR], ds1[NR], dm0[NR], dm1[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const float d = half_bits_to_float(hdr[r].x);
        const float dmin = half_bits_to_float(hdr[r].x >> 16);
        const uint32_t y = hdr[r].y >> (8 * i0), z = hdr[r].z >> (8 * i0), w = hdr[r].w >> (8 * i0);
        const uint32_t hi_sc = ((y >> 6) & 0x3u) | (((y >> 14) & 0x3u) << 8);      // 2 high bits, bytes 0/1
        const uint32_t hi_mn = ((z >> 6) & 0x3u) | (((z >> 14) & 0x3u) << 8);
        const uint32_t sc_pair = low ? (y & 0x3F3Fu) : ((w & 0x0F0Fu) | (hi_sc << 4));
        const uint32_t mn_pair = low ? (z & 0x3F3Fu) : (((w >> 4) & 0x0F0Fu) | (hi_mn << 4));
        const float sc0 = __uint_as_float(0x4B000000u | (sc_pair & 0xffu)) - 8388608.0f;
        const float sc1 = __uint_as_float(0x4B000000u | (sc_pair >> 8)) - 8388608.0f;
        const float mn0 = __uint_as_float(0x4B000000u | (mn_pair & 0xffu)) - 8388608.0f;
        const float mn1 = __uint_as_float(0x4B000000u | (mn_pair >> 8)) - 8388608.0f;
        ds0[r] = d * sc0;
        ds1[r] = d * sc1 * 0.0625f;  // high nibbles enter dp4a as 16*q
        dm0[r] = dmin * mn0;
        dm1[r] = dmin * mn1;
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int4 *xhv = reinterpret_cast<const int4 *>(xp.xh + xp.off(m, k0));
        const int4 *xlv = reinterpret_cast<const int4 *>(xp.xl + xp.off(m, k0));
        const int4 hA0 = xhv[0], hA1 = xhv[1], hB0 = xhv[2], hB1 = xhv[3];
        const int4 lA0 = xlv[0], lA1 = xlv[1], lB0 = xlv[2], lB1 = xlv[3];
        const float4 mt = xp.meta[m * (K >> 6) + (j0 >> 1)];
        const float s0 = mt.x, s1 = mt.y, xs0 = mt.z, xs1 = mt.w;
        const int xhA[8] = {hA0.x, hA0.y, hA0.z, hA0.w, hA1.x, hA1.y, hA1.z, hA1.w};
        const int xlA[8] = {lA0.x, lA0.y, lA0.z, lA0.w, lA1.x, lA1.y, lA1.z, lA1.w};
        const int xhB[8] = {hB0.x, hB0.y, hB0.z, hB0.w, hB1.x, hB1.y, hB1.z, hB1.w};
        const int xlB[8] = {lB0.x, lB0.y, lB0.z, lB0.w, lB1.x, lB1.y, lB1.z, lB1.w};
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const uint32_t wA[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
            int hiL = 0, loL = 0, hiH = 0, loH = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t lo4 = wA[i] & 0x0F0F0F0Fu;
                const uint32_t hi4 = wA[i] & 0xF0F0F0F0u;
                hiL = dp4a_us(lo4, xhA[i], hiL);
                loL = dp4a_us(lo4, xlA[i], loL);
                hiH = dp4a_us(hi4, xhB[i], hiH);
                loH = dp4a_us(hi4, xlB[i], loH);
            }
            const float TL = static_cast<float>(hiL * 128 + loL);
            const float TH = static_cast<float>(hiH * 128 + loH);
            float a = acc[r][m];
            a = fmaf(ds0[r] * s0, TL, a);
            a = fmaf(ds1[r] * s1, TH, a);
            a = fmaf(-dm0[r], xs0, a);
            a = fmaf(-dm1[r], xs1, a);
            acc[r][m] = a;
        }
    }
}

// ------------------------------------------------------------- Q6_K unit
// Unit = (block b, half s, l-half lh): values i = 128 s + 32 c + 16 lh + l,
// c = 0..3, l = 0..15 (quantize/vulkan.py:542-564 layout).
template <int MT, int NR, bool SMEM>
__device__ __forceinline__ void unit_q6k(const uint8_t *const rows[NR], int b, int sl, int kbase, int K,
                                         const XPlanes &xp, float acc[NR][MT]) {
    const int s = sl >> 1, lh = sl & 1;
    const int kk = kbase + b * 256 + s * 128 + lh * 16;
    uint4 qa[NR], qb[NR], qh[NR];
    float dsc[NR][4];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (rows[r] != nullptr) {
            const uint8_t *blk = rows[r] + b * 210;
            qa[r] = ld16_a2<SMEM>(blk + 64 * s + 16 * lh);
            qb[r] = ld16_a2<SMEM>(blk + 64 * s + 32 + 16 * lh);
            qh[r] = ld16_a2<SMEM>(blk + 128 + 32 * s + 16 * lh);
            const float d = half_bits_to_float(ld_u16<SMEM>(blk + 208));
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t pair = ld_u16<SMEM>(blk + 192 + 8 * s + 2 * c);
                const int8_t code = static_cast<int8_t>((pair >> (8 * lh)) & 0xffu);
                dsc[r][c] = d * static_cast<float>(code);
            }
        } else {
            qa[r] = make_uint4(0, 0, 0, 0);
            qb[r] = qa[r];
            qh[r] = qa[r];
#pragma unroll
            for (int c = 0; c < 4; ++c) dsc[r][c] = 0.0f;
        }
    }
    const int sub_per_row = K >> 5;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int k = kk + 32 * c;
            const int4 xh4 = *reinterpret_cast<const int4 *>(xp.xh + xp.off(m, k));
            const int4 xl4 = *reinterpret_cast<const int4 *>(xp.xl + xp.off(m, k));
            const float sxv = xp.sx[m * sub_per_row + (k >> 5)];
            const int q16 = xp.xq16[m * sub_per_row * 2 + (k >> 4)];
            const int xhw[4] = {xh4.x, xh4.y, xh4.z, xh4.w};
            const int xlw[4] = {xl4.x, xl4.y, xl4.z, xl4.w};
#pragma unroll
            for (int r = 0; r < NR; ++r) {
                const uint4 ql = (c & 1) ? qb[r] : qa[r];
                const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
                const uint32_t hw[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
                int hi = 0, lo = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t l4 = (c >> 1) ? ((lw[i] >> 4) & 0x0F0F0F0Fu) : (lw[i] & 0x0F0F0F0Fu);
                    const uint32_t h2 = ((hw[i] >> (2 * c)) & 0x03030303u) << 4;
                    const uint32_t level = l4 | h2;
                    hi = dp4a_us(level, xhw[i], hi);
                    lo = dp4a_us(level, xlw[i], lo);
                }
                const int T = hi * 128 + lo - 32 * q16;
                acc[r][m] = fmaf(dsc[r][c] * sxv, static_cast<float>(T), acc[r][m]);
            }
        }
    }
}

// ------------------------------------------------------------- Q8_0 unit
// Unit = blocks 2u and 2u+1 of the segment (68 bytes, 4-byte aligned).
template <int MT, int NR, bool SMEM>
__device__ __forceinline__ void unit_q8_0(const uint8_t *const rows[NR], int u, int kbase, int K,
                                          const XPlanes &xp, float acc[NR][MT]) {
    uint32_t qa[NR][8], qb[NR][8];
    float da[NR], db[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (rows[r] != nullptr) {
            const uint8_t *p = rows[r] + u * 68;
            uint32_t w[17];
#pragma unroll
            for (int i = 0; i < 17; ++i) w[i] = ld_u32<SMEM>(p + 4 * i);
            da[r] = half_bits_to_float(w[0]);
            db[r] = half_bits_to_float(w[8] >> 16);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qa[r][i] = __funnelshift_r(w[i], w[i + 1], 16);
                qb[r][i] = w[9 + i];
            }
        } else {
            da[r] = 0.0f;
            db[r] = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qa[r][i] = 0;
                qb[r][i] = 0;
            }
        }
    }
    const int k0 = kbase + u * 64;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int4 *xhv = reinterpret_cast<const int4 *>(xp.xh + xp.off(m, k0));
        const int4 *xlv = reinterpret_cast<const int4 *>(xp.xl + xp.off(m, k0));
        const int4 h0 = xhv[0], h1 = xhv[1], h2 = xhv[2], h3 = xhv[3];
        const int4 l0 = xlv[0], l1 = xlv[1], l2 = xlv[2], l3 = xlv[3];
        const int xhA[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int xlA[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const int xhB[8] = {h2.x, h2.y, h2.z, h2.w, h3.x, h3.y, h3.z, h3.w};
        const int xlB[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
        const float4 mt = xp.meta[m * (K >> 6) + (k0 >> 6)];
        const float sA = mt.x, sB = mt.y;
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            int hA = 0, lA = 0, hB = 0, lB = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                hA = dp4a_ss(static_cast<int>(qa[r][i]), xhA[i], hA);
                lA = dp4a_ss(static_cast<int>(qa[r][i]), xlA[i], lA);
                hB = dp4a_ss(static_cast<int>(qb[r][i]), xhB[i], hB);
                lB = dp4a_ss(static_cast<int>(qb[r][i]), xlB[i], lB);
            }
            float a = acc[r][m];
            a = fmaf(da[r] * sA, static_cast<float>(hA * 128 + lA), a);
            a = fmaf(db[r] * sB, static_cast<float>(hB * 128 + lB), a);
            acc[r][m] = a;
        }
    }
}

// Runs unit `u` of a row segment starting at absolute k `kbase` for NR rows.
// Q4_K / Q6_K: 4 units per block; Q8_0: u indexes block pairs.
template <int MT, int NR, bool SMEM>
__device__ __forceinline__ void run_unit(int fmt, const uint8_t *const rows[NR], int u, int kbase, int K,
                                         const XPlanes &xp, float acc[NR][MT]) {
    if (fmt == T2C_Q4_K) {
        unit_q4k<MT, NR, SMEM>(rows, u >> 2, u & 3, kbase, K, xp, acc);
    } else if (fmt == T2C_Q6_K) {
        unit_q6k<MT, NR, SMEM>(rows, u >> 2, u & 3, kbase, K, xp, acc);
    } else {
        unit_q8_0<MT, NR, SMEM>(rows, u, kbase, K, xp, acc);
    }
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

// Epilogue for NR rows.  ROWS mode: row r is output n[r] of stream st.
// SWIGLU mode: rows (r, r+1) are (gate, up) of output n[r].  n < 0: no row.
template <int MT, int NR>
__device__ __forceinline__ void store_rows(const QParams &p, const QStream &st, const int64_t n[NR],
                                           const float acc[NR][MT], bool swiglu) {
    if (p.mode == MODE_ARGMAX) {
        // rows n[0..NR) are consecutive and start on a multiple of 4
        if (n[0] < 0) return;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m >= p.M) continue;
            float best = acc[0][m];
            uint32_t tok = static_cast<uint32_t>(n[0]);
#pragma unroll
            for (int r = 1; r < NR; ++r) {
                if (n[r] >= 0 && acc[r][m] > best) {
                    best = acc[r][m];
                    tok = static_cast<uint32_t>(n[r]);
                }
            }
            const int64_t g = n[0] >> 2;
            p.ps[m * p.G + g] = best;
            p.pt[m * p.G + g] = tok;
        }
        return;
    }
    if (swiglu) {
#pragma unroll
        for (int r = 0; r + 1 < NR; r += 2) {
            if (n[r] < 0) continue;
#pragma unroll
            for (int m = 0; m < MT; ++m)
                if (m < p.M) st.y[m * st.n + n[r]] = __float2half_rn(silu(acc[r][m]) * acc[r + 1][m]);
        }
        return;
    }
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        if (n[r] < 0) continue;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < p.M) {
                const int64_t o = m * st.n + n[r];
                float v = acc[r][m];
                if (st.res) v += __half2float(st.res[o]);
                st.y[o] = __float2half_rn(v);
            }
        }
    }
}

template <int MT, int NR>
__device__ __forceinline__ void reduce_lanes(float acc[NR][MT], int lpr) {
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float v = acc[r][m];
            for (int o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[r][m] = v;
        }
}

// =============================================================== direct kernel
// A row-set = 2 rows (ROWS: rows n0, n0+1 of one stream; SWIGLU: gate row n0
// and up row n0), processed by `lpr` lanes that split the 64-value units.
constexpr int kDirectRows = 2;

template <int MT, int FMT>
__global__ void __launch_bounds__(kThreads, (MT == 1 ? 5 : 2)) qmv_direct_kernel(const QParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = p.K;
    float4 *meta = reinterpret_cast<float4 *>(smem);
    int8_t *xh = reinterpret_cast<int8_t *>(meta + MT * (K >> 6));
    int8_t *xl = xh + MT * padded_k(K);
    float *sx = reinterpret_cast<float *>(xl + MT * padded_k(K));
    int *xq16 = reinterpret_cast<int *>(sx + MT * (K >> 5));
    float *red = reinterpret_cast<float *>(xq16 + MT * (K >> 4));

    pdl_wait();
    pdl_trigger();
    prepare_x<MT, kThreads>(p, xh, xl, sx, xq16, meta, red);

    const XPlanes xp{xh, xl, sx, xq16, meta, padded_k(K)};
    const int lane = threadIdx.x & 31;
    const int lpr = p.lpr;
    const int sub = lane / lpr;
    const int sub_lane = lane - sub * lpr;
    const int subs_per_warp = 32 / lpr;
    const int64_t gsub = (static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5)) * subs_per_warp + sub;
    const int64_t gsub_stride = static_cast<int64_t>(gridDim.x) * kWarps * subs_per_warp;
    const bool swiglu = p.mode == MODE_SWIGLU;

    // Every sub-warp runs the same number of iterations so the shuffles always
    // see full warps; row-sets past the end are masked out.
    const int64_t iters = (p.total_rowsets + gsub_stride - 1) / gsub_stride;
    for (int64_t it = 0; it < iters; ++it) {
        const int64_t rs = gsub + it * gsub_stride;
        const uint8_t *rows[kDirectRows] = {nullptr, nullptr};
        int64_t n[kDirectRows] = {-1, -1};
        int fmt = T2C_Q4_K;
        int si = 0;
        if (rs < p.total_rowsets) {
            if (swiglu) {
                fmt = p.s[0].fmt;
                rows[0] = p.s[0].w + rs * p.s[0].row_bytes;
                rows[1] = p.s[1].w + rs * p.s[1].row_bytes;
                n[0] = rs;
                n[1] = rs;
            } else {
#pragma unroll
                for (int i = 1; i < kMaxStreams; ++i)
                    if (i < p.nstreams && rs >= p.s[i].rs_begin) si = i;
                const QStream &st = p.s[si];
                fmt = st.fmt;
                const int64_t n0 = (rs - st.rs_begin) * kDirectRows;
                rows[0] = st.w + n0 * st.row_bytes;
                n[0] = n0;
                if (n0 + 1 < st.n) {
                    rows[1] = rows[0] + st.row_bytes;
                    n[1] = n0 + 1;
                }
            }
        }
        if (FMT != 0) fmt = FMT;
        float acc[kDirectRows][MT];
#pragma unroll
        for (int r = 0; r < kDirectRows; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        if (rs < p.total_rowsets) {
            for (int u = sub_lane; u < p.units; u += lpr) run_unit<MT, kDirectRows, false>(fmt, rows, u, 0, K, xp, acc);
        }
        reduce_lanes<MT, kDirectRows>(acc, lpr);
        if (p.mode == MODE_ARGMAX) {
            // Rows 4g..4g+3 are row-sets 2g and 2g+1, held by sub-warps sub and
            // sub+1 of this warp (lpr <= 16, so row-set parity = sub parity).
            // The even sub-warp merges its partner's best; ties keep the lower id.
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                float best = -INFINITY;
                uint32_t tok = 0xffffffffu;
                if (rs < p.total_rowsets && m < p.M) {
                    best = acc[0][m];
                    tok = static_cast<uint32_t>(n[0]);
                    if (n[1] >= 0 && acc[1][m] > best) {
                        best = acc[1][m];
                        tok = static_cast<uint32_t>(n[1]);
                    }
                }
                const float other = __shfl_down_sync(0xffffffffu, best, lpr);
                const uint32_t other_tok = __shfl_down_sync(0xffffffffu, tok, lpr);
                if (sub_lane == 0 && (sub & 1) == 0 && rs < p.total_rowsets && m < p.M) {
                    if (other_tok != 0xffffffffu && other > best) {
                        best = other;
                        tok = other_tok;
                    }
                    p.ps[m * p.G + (rs >> 1)] = best;
                    p.pt[m * p.G + (rs >> 1)] = tok;
                }
            }
            continue;
        }
        if (sub_lane == 0 && rs < p.total_rowsets) store_rows<MT, kDirectRows>(p, p.s[si], n, acc, swiglu);
    }
}

// ============================================================= streamed kernel
// Persistent CTAs of four warps, several CTAs per SM.  Every warp runs its
// own pipeline: lane 0 streams the warp's row blocks HBM -> shared memory with
// 1-D bulk async copies into a private ring of `stages` buffers (completion
// on one mbarrier per buffer) and refills a buffer as soon as the warp has
// decoded it, so each warp keeps `stages` copies in flight and no warp waits
// for another.  Stage = one row block x one K segment: rb rows, each a
// contiguous segment of seg_bytes (or, for `whole` streams, rb full rows
// copied at once).  Row group g of kNR rows is served by lpr lanes (one
// 64-value unit per lane per stage; x fragments reused across the kNR rows).
// SwiGLU row blocks hold rb/2 gate rows then the rb/2 matching up rows; a
// row group is then two outputs (gate, up, gate, up).
constexpr int kNR = 4;
constexpr int kConsumerWarps = kWarps;
constexpr int kConsumerThreads = kThreads;
constexpr size_t kStageHead = 512;  // full barriers [kWarps][kMaxStages]

__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
// 16 bytes at a 2-byte aligned shared address.
__device__ __forceinline__ uint4 lds128_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8), w3 = lds32(b + 12);
    const uint32_t w4 = sh ? lds32(b + 16) : 0u;
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}

__device__ __forceinline__ float small_u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// x planes as shared addresses.
struct XS {
    uint32_t xh, xl, meta, sx, xq16;
    int kp, u64, s32;  // padded row stride, K/64, K/32
    __device__ __forceinline__ uint32_t off(int m, int k) const {
        return static_cast<uint32_t>(m * kp + k + ((k >> 6) << 4));
    }
};

// Q4_K: rows[r] = shared address of the 144-byte block, G = group, k0 = first value.
template <int MT>
__device__ __forceinline__ void lane_q4k(const uint32_t rows[kNR], int G, int k0, const XS &x,
                                         float acc[kNR][MT]) {
    const int i0 = (2 * G) & 3;
    const bool low = G < 2;
    uint4 q0[kNR], q1[kNR];
    float ds0[kNR], ds1[kNR], dm0[kNR], dm1[kNR];
#pragma unroll
    for (int r = 0; r < kNR; ++r) {
        const uint4 h = lds128(rows[r]);
        q0[r] = lds128(rows[r] + 16 + 32 * G);
        q1[r] = lds128(rows[r] + 32 + 32 * G);
        const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
        const uint32_t y = h.y >> (8 * i0), z = h.z >> (8 * i0), w = h.w >> (8 * i0);
        const uint32_t hs = ((y >> 6) & 0x3u) | (((y >> 14) & 0x3u) << 8);
        const uint32_t hm = ((z >> 6) & 0x3u) | (((z >> 14) & 0x3u) << 8);
        const uint32_t scp = low ? (y & 0x3F3Fu) : ((w & 0x0F0Fu) | (hs << 4));
        const uint32_t mnp = low ? (z & 0x3F3Fu) : (((w >> 4) & 0x0F0Fu) | (hm << 4));
        ds0[r] = d * small_u2f(scp & 0xffu);
        ds1[r] = d * small_u2f(scp >> 8) * 0.0625f;  // high nibbles enter dp4a as 16*q
        dm0[r] = dmin * small_u2f(mnp & 0xffu);
        dm1[r] = dmin * small_u2f(mnp >> 8);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const uint32_t xo = x.off(m, k0);
        const uint4 hA0 = lds128(x.xh + xo), hA1 = lds128(x.xh + xo + 16), hB0 = lds128(x.xh + xo + 32),
                    hB1 = lds128(x.xh + xo + 48);
        const uint4 lA0 = lds128(x.xl + xo), lA1 = lds128(x.xl + xo + 16), lB0 = lds128(x.xl + xo + 32),
                    lB1 = lds128(x.xl + xo + 48);
        const uint4 mt = lds128(x.meta + 16u * static_cast<uint32_t>(m * x.u64 + (k0 >> 6)));
        const float s0 = __uint_as_float(mt.x), s1 = __uint_as_float(mt.y);
        const float xs0 = __uint_as_float(mt.z), xs1 = __uint_as_float(mt.w);
        const uint32_t xhA[8] = {hA0.x, hA0.y, hA0.z, hA0.w, hA1.x, hA1.y, hA1.z, hA1.w};
        const uint32_t xlA[8] = {lA0.x, lA0.y, lA0.z, lA0.w, lA1.x, lA1.y, lA1.z, lA1.w};
        const uint32_t xhB[8] = {hB0.x, hB0.y, hB0.z, hB0.w, hB1.x, hB1.y, hB1.z, hB1.w};
        const uint32_t xlB[8] = {lB0.x, lB0.y, lB0.z, lB0.w, lB1.x, lB1.y, lB1.z, lB1.w};
#pragma unroll
        for (int r = 0; r < kNR; ++r) {
            const uint32_t wq[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
            int hiL = 0, loL = 0, hiH = 0, loH = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t lo4 = wq[i] & 0x0F0F0F0Fu, hi4 = wq[i] & 0xF0F0F0F0u;
                hiL = dp4a_us(lo4, static_cast<int>(xhA[i]), hiL);
                loL = dp4a_us(lo4, static_cast<int>(xlA[i]), loL);
                hiH = dp4a_us(hi4, static_cast<int>(xhB[i]), hiH);
                loH = dp4a_us(hi4, static_cast<int>(xlB[i]), loH);
            }
            float a = acc[r][m];
            a = fmaf(ds0[r] * s0, static_cast<float>(hiL * 128 + loL), a);
            a = fmaf(ds1[r] * s1, static_cast<float>(hiH * 128 + loH), a);
            a = fmaf(-dm0[r], xs0, a);
            a = fmaf(-dm1[r], xs1, a);
            acc[r][m] = a;
        }
    }
}

// Q6_K: rows[r] = shared address of the 210-byte block; sl = 2 s + lh; kk = value index of (s, lh, c=0, l=0).
template <int MT>
__device__ __forceinline__ void lane_q6k(const uint32_t rows[kNR], int sl, int kk, const XS &x,
                                         float acc[kNR][MT]) {
    const int s = sl >> 1, lh = sl & 1;
    uint4 qa[kNR], qb[kNR], qh[kNR];
    float dsc[kNR][4];
#pragma unroll
    for (int r = 0; r < kNR; ++r) {
        qa[r] = lds128_a2(rows[r] + 64 * s + 16 * lh);
        qb[r] = lds128_a2(rows[r] + 64 * s + 32 + 16 * lh);
        qh[r] = lds128_a2(rows[r] + 128 + 32 * s + 16 * lh);
        const float d = half_bits_to_float(lds16(rows[r] + 208));
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t pair = lds16(rows[r] + 192 + 8 * s + 2 * c);
            dsc[r][c] = d * static_cast<float>(static_cast<int8_t>((pair >> (8 * lh)) & 0xffu));
        }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int k = kk + 32 * c;
            const uint4 xh4 = lds128(x.xh + x.off(m, k)), xl4 = lds128(x.xl + x.off(m, k));
            const float sxv = __uint_as_float(lds32(x.sx + 4u * static_cast<uint32_t>(m * x.s32 + (k >> 5))));
            const int q16 = static_cast<int>(lds32(x.xq16 + 4u * static_cast<uint32_t>(m * x.s32 * 2 + (k >> 4))));
            const uint32_t xhw[4] = {xh4.x, xh4.y, xh4.z, xh4.w};
            const uint32_t xlw[4] = {xl4.x, xl4.y, xl4.z, xl4.w};
#pragma unroll
            for (int r = 0; r < kNR; ++r) {
                const uint4 ql = (c & 1) ? qb[r] : qa[r];
                const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
                const uint32_t hw[4] = {qh[r].x, qh[r].y, qh[r].z, qh[r].w};
                int hi = 0, lo = 0;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t l4 = (c >> 1) ? ((lw[i] >> 4) & 0x0F0F0F0Fu) : (lw[i] & 0x0F0F0F0Fu);
                    const uint32_t level = l4 | (((hw[i] >> (2 * c)) & 0x03030303u) << 4);
                    hi = dp4a_us(level, static_cast<int>(xhw[i]), hi);
                    lo = dp4a_us(level, static_cast<int>(xlw[i]), lo);
                }
                acc[r][m] = fmaf(dsc[r][c] * sxv, static_cast<float>(hi * 128 + lo - 32 * q16), acc[r][m]);
            }
        }
    }
}

// Q8_0: rows[r] = shared address of the block pair (68 bytes, 4-byte aligned); k0 = first value.
template <int MT>
__device__ __forceinline__ void lane_q8_0(const uint32_t rows[kNR], int k0, const XS &x, float acc[kNR][MT]) {
    uint32_t qa[kNR][8], qb[kNR][8];
    float da[kNR], db[kNR];
#pragma unroll
    for (int r = 0; r < kNR; ++r) {
        uint32_t w[17];
#pragma unroll
        for (int i = 0; i < 17; ++i) w[i] = lds32(rows[r] + 4 * i);
        da[r] = half_bits_to_float(w[0]);
        db[r] = half_bits_to_float(w[8] >> 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            qa[r][i] = __funnelshift_r(w[i], w[i + 1], 16);
            qb[r][i] = w[9 + i];
        }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const uint32_t xo = x.off(m, k0);
        const uint4 h0 = lds128(x.xh + xo), h1 = lds128(x.xh + xo + 16), h2 = lds128(x.xh + xo + 32),
                    h3 = lds128(x.xh + xo + 48);
        const uint4 l0 = lds128(x.xl + xo), l1 = lds128(x.xl + xo + 16), l2 = lds128(x.xl + xo + 32),
                    l3 = lds128(x.xl + xo + 48);
        const uint4 mt = lds128(x.meta + 16u * static_cast<uint32_t>(m * x.u64 + (k0 >> 6)));
        const float sA = __uint_as_float(mt.x), sB = __uint_as_float(mt.y);
        const uint32_t xhA[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t xlA[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const uint32_t xhB[8] = {h2.x, h2.y, h2.z, h2.w, h3.x, h3.y, h3.z, h3.w};
        const uint32_t xlB[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
#pragma unroll
        for (int r = 0; r < kNR; ++r) {
            int hA = 0, lA = 0, hB = 0, lB = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                hA = dp4a_ss(static_cast<int>(qa[r][i]), static_cast<int>(xhA[i]), hA);
                lA = dp4a_ss(static_cast<int>(qa[r][i]), static_cast<int>(xlA[i]), lA);
                hB = dp4a_ss(static_cast<int>(qb[r][i]), static_cast<int>(xhB[i]), hB);
                lB = dp4a_ss(static_cast<int>(qb[r][i]), static_cast<int>(xlB[i]), lB);
            }
            float a = acc[r][m];
            a = fmaf(da[r] * sA, static_cast<float>(hA * 128 + lA), a);
            a = fmaf(db[r] * sB, static_cast<float>(hB * 128 + lB), a);
            acc[r][m] = a;
        }
    }
}

__device__ __forceinline__ int stream_of(const QParams &p, int64_t block) {
    int si = 0;
#pragma unroll
    for (int i = 1; i < kMaxStreams; ++i)
        if (i < p.nstreams && block >= p.s[i].rs_begin) si = i;
    return si;
}

__device__ __forceinline__ int64_t block_first_row(const QParams &p, int si, int64_t block) {
    const int rows = p.mode == MODE_SWIGLU ? p.s[0].rb / 2 : p.s[si].rb;
    return (block - p.s[si].rs_begin) * rows;
}

// Issues the bulk copies of one stage and arms its full barrier.
__device__ __forceinline__ void issue_stage(const QParams &p, int64_t block, int chunk, uint8_t *stage,
                                            uint64_t *bar) {
    const int si = stream_of(p, block);
    const int64_t row0 = block_first_row(p, si, block);
    const QStream &st = p.s[si];
    if (p.mode == MODE_SWIGLU) {
        const int half = st.rb / 2;
        const int64_t left = p.s[0].n - row0;
        const int nv = left < half ? static_cast<int>(left) : half;
        mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nv) * 2u * st.seg_bytes);
        for (int g = 0; g < 2; ++g) {
            const QStream &sg = p.s[g];
            for (int r = 0; r < nv; ++r) {
                const uint8_t *src = sg.w + (row0 + r) * sg.row_bytes + static_cast<int64_t>(chunk) * st.seg_bytes;
                bulk_g2s(stage + (g * half + r) * st.seg_bytes, src, st.seg_bytes, bar);
            }
        }
        return;
    }
    const int64_t left = st.n - row0;
    const int nv = left < st.rb ? static_cast<int>(left) : st.rb;
    if (st.whole) {
        const uint32_t bytes = static_cast<uint32_t>(nv * st.row_bytes);
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(stage, st.w + row0 * st.row_bytes, bytes, bar);
        return;
    }
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(nv) * st.seg_bytes);
    for (int r = 0; r < nv; ++r) {
        const uint8_t *src = st.w + (row0 + r) * st.row_bytes + static_cast<int64_t>(chunk) * st.seg_bytes;
        bulk_g2s(stage + r * st.seg_bytes, src, st.seg_bytes, bar);
    }
}

// Advances a warp's item cursor (row block, K segment) by one.
__device__ __forceinline__ void next_item(const QParams &p, int64_t &block, int &chunk, int64_t block_stride) {
    if (++chunk == p.s[stream_of(p, block)].chunks) {
        chunk = 0;
        block += block_stride;
    }
}

template <int MT, int FMT>
__global__ void __launch_bounds__(kConsumerThreads) qmv_tma_kernel(const QParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = p.K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem) + warp * kMaxStages;
    uint8_t *stages = smem + kStageHead + static_cast<size_t>(warp) * S * p.stage_bytes;
    float4 *meta = reinterpret_cast<float4 *>(smem + kStageHead + static_cast<size_t>(kWarps) * S * p.stage_bytes);
    int8_t *xh = reinterpret_cast<int8_t *>(meta + MT * (K >> 6));
    int8_t *xl = xh + MT * padded_k(K);
    float *sx = reinterpret_cast<float *>(xl + MT * padded_k(K));
    int *xq16 = reinterpret_cast<int *>(sx + MT * (K >> 5));
    float *red = reinterpret_cast<float *>(xq16 + MT * (K >> 4));
    const int64_t block_stride = static_cast<int64_t>(gridDim.x) * kWarps;
    const int64_t first_block = static_cast<int64_t>(blockIdx.x) * kWarps + warp;

    // Weights are static: start streaming before the dependency on the
    // previous kernel in the stream resolves.
    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
        int64_t block = first_block;
        int chunk = 0;
        for (int i = 0; i < S && block < p.total_rowsets; ++i) {
            issue_stage(p, block, chunk, stages + static_cast<size_t>(i) * p.stage_bytes, &full[i]);
            next_item(p, block, chunk, block_stride);
        }
    }
    pdl_wait();
    pdl_trigger();
    prepare_x<MT, kConsumerThreads>(p, xh, xl, sx, xq16, meta, red);  // ends with __syncthreads
    const XS x{smem_u32(xh), smem_u32(xl), smem_u32(meta), smem_u32(sx), smem_u32(xq16), padded_k(K), K >> 6,
               K >> 5};
    const bool swiglu = p.mode == MODE_SWIGLU;
    const uint32_t stages_addr = smem_u32(stages);

    int s = 0;
    uint32_t phase = 0;
    int64_t ahead_block = first_block;  // cursor S items ahead of the one consumed
    int ahead_chunk = 0;
    for (int i = 0; i < S; ++i) next_item(p, ahead_block, ahead_chunk, block_stride);
    for (int64_t block = first_block; block < p.total_rowsets; block += block_stride) {
        const int si = stream_of(p, block);
        const QStream &st = p.s[si];
        const int64_t row0 = block_first_row(p, si, block);
        const int fmt = FMT != 0 ? FMT : st.fmt;
        const int lpr = st.lpr;
        const int group = lane / lpr, glane = lane - group * lpr;
        const int units = fmt == T2C_Q8_0 ? st.seg_blocks / 2 : st.seg_blocks * 4;
        const int seg_stride = st.whole ? static_cast<int>(st.row_bytes) : st.seg_bytes;
        const int seg_values = st.seg_blocks * (fmt == T2C_Q8_0 ? 32 : 256);
        uint32_t roff[kNR];
        int64_t n[kNR];
#pragma unroll
        for (int r = 0; r < kNR; ++r) {
            int srow;
            if (swiglu) {
                const int o = 2 * group + (r >> 1);
                srow = (r & 1) * (st.rb / 2) + o;
                n[r] = row0 + o < p.s[0].n ? row0 + o : -1;
            } else {
                srow = group * kNR + r;
                n[r] = row0 + srow < st.n ? row0 + srow : -1;
            }
            roff[r] = static_cast<uint32_t>(srow * seg_stride);
        }
        float acc[kNR][MT];
#pragma unroll
        for (int r = 0; r < kNR; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        for (int c = 0; c < st.chunks; ++c) {
            if (!mbar_wait(&full[s], phase)) {
                // Copies never completed: report and leave without touching the stage.
                report_device_error(T2C_ETIMEOUT);
                return;
            }
            const uint32_t stage = stages_addr + static_cast<uint32_t>(s) * static_cast<uint32_t>(p.stage_bytes);
            const int kseg = c * seg_values;
            for (int u = glane; u < units; u += lpr) {
                uint32_t rows[kNR];
                if (fmt == T2C_Q4_K) {
#pragma unroll
                    for (int r = 0; r < kNR; ++r) rows[r] = stage + roff[r] + (u >> 2) * 144;
                    lane_q4k<MT>(rows, u & 3, kseg + (u >> 2) * 256 + (u & 3) * 64, x, acc);
                } else if (fmt == T2C_Q6_K) {
#pragma unroll
                    for (int r = 0; r < kNR; ++r) rows[r] = stage + roff[r] + (u >> 2) * 210;
                    const int sl = u & 3;
                    lane_q6k<MT>(rows, sl, kseg + (u >> 2) * 256 + (sl >> 1) * 128 + (sl & 1) * 16, x, acc);
                } else {
#pragma unroll
                    for (int r = 0; r < kNR; ++r) rows[r] = stage + roff[r] + u * 68;
                    lane_q8_0<MT>(rows, kseg + u * 64, x, acc);
                }
            }
            // Refill this buffer with the item S positions ahead (async-proxy
            // writes after the warp's generic reads).
            __syncwarp();
            if (lane == 0 && ahead_block < p.total_rowsets) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_stage(p, ahead_block, ahead_chunk, stages + static_cast<size_t>(s) * p.stage_bytes, &full[s]);
            }
            next_item(p, ahead_block, ahead_chunk, block_stride);
            if (++s == S) {
                s = 0;
                phase ^= 1u;
            }
        }
        reduce_lanes<MT, kNR>(acc, lpr);
        if (glane == 0) store_rows<MT, kNR>(p, st, n, acc, swiglu);
    }
}

// ============================================================ tensor-core kernel
// Q4_K matvec for M <= 4 with int8 tensor-core tiles (mma.sync m16n8k32
// s8 x s8 -> s32): one instruction forms the 16-row x 32-value integer dot
// products of a sub-block for all (batch row, x plane) columns, so a warp
// spends ~0.05 instructions per weight instead of ~0.13 with dp4a.
//   A (16 x 32): weight nibbles of 16 rows for one 32-value sub-block.  Lane
//     (g = lane/4, t = lane%4) takes bytes 8t..8t+7 of the sub-block's 32-byte
//     group for rows g and g+8; low nibbles form sub-block 2q, high nibbles 2q+1.
//     The k order inside the tile is permuted (slots 4t..4t+3 <- values
//     8t..8t+3, slots 16+4t.. <- 8t+4..8t+7) identically for A and B.
//   B (32 x 8): column n = 2m + plane holds x plane (xh, xl) of batch row m.
//   D: lane (g, t) receives rows g, g+8 for batch row m = t, both planes, and
//     applies the sub-block scale d*sc (taken by shuffle from the lane that
//     decoded it), the x scale and the min term.
// Streaming is the same as qmv_tma_kernel (warp-private rings of 1-D bulk
// copies into shared memory, bounded mbarrier waits, weights requested before
// griddepcontrol.wait), with 16-row blocks and 2-super-block (288-byte) row
// segments (a 288-byte row stride keeps the 8-byte fragment reads free of
// bank conflicts).  K is split across the warps of a CTA: the 8 warps form
// bpc groups of wpb warps; group j takes row block (iteration base + j) and
// its warps take segments w, w + wpb, ...; the partial sums meet in shared
// memory at the end of every CTA iteration.
constexpr int kMmaWarps = 8;
constexpr int kMmaThreads = kMmaWarps * 32;
constexpr int kMmaSegBlocks = 2;
constexpr int kMmaSegBytes = kMmaSegBlocks * 144;
constexpr int kMmaRows = 16;




__device__ __forceinline__ void mma_f16_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// fp16 x of the 2..4-token kernel (prepare_x_f16): shared addresses.
struct XF {
    uint32_t perm, sum;
    int row_bytes, sum_row;  // xf_row_bytes(K), (K / 256) * 32
};

__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// Small non-negative integer v (< 2048) times 2^-e as fp16 bits, duplicated in both halves.
__device__ __forceinline__ uint32_t half2_dup(float v) {
    const uint32_t b = __half_as_ushort(__float2half_rn(v));
    return b | (b << 16);
}

// One 144-byte super-block of a 16-row group for up to 4 batch rows:
// acc[0] row g, acc[1] row g+8, batch row t (mma m16n8k16, f16 inputs, fp32
// accumulators).  Lane (g, t) reads group t of rows g, g + 8 (low nibbles:
// sub-block 2t, high nibbles: sub-block 2t + 1).  Each nibble becomes an fp16
// subnormal by masking (q * 2^-24 or 16 q * 2^-24) and is multiplied by its
// sub-block scale code (sc, or sc / 16 for the high nibbles) in one f16x2
// multiply: sc * q * 2^-24 exactly (sc * q < 1024), so one accumulator holds
// the whole super-block.  B column n carries batch row n / 2 (clamped to
// M - 1): D column 2t of lane (g, t) is batch row t.  The min term
// sum_j m_j * xsum_j comes from one more mma (A = m codes, B = the hi / lo
// fp16 parts of the sub-block sums).  The k order inside an mma follows the
// pair-interleaved x chunks: word j, byte parity p of group t fill k-slots
// {2t, 2t + 1} with bytes 4j + p, 4j + p + 2 (low nibbles) and
// {2t + 8, 2t + 9} with their high nibbles.
__device__ __forceinline__ void q4k_codes(const uint4 h, int t, uint32_t &sc0, uint32_t &sc1, uint32_t &m0,
                                          uint32_t &m1) {
    const int i0 = (2 * t) & 3;
    const bool low = t < 2;
    const uint32_t y = h.y >> (8 * i0), z = h.z >> (8 * i0), w = h.w >> (8 * i0);
    const uint32_t hs = ((y >> 6) & 0x3u) | (((y >> 14) & 0x3u) << 8);
    const uint32_t hm = ((z >> 6) & 0x3u) | (((z >> 14) & 0x3u) << 8);
    const uint32_t scp = low ? (y & 0x3F3Fu) : ((w & 0x0F0Fu) | (hs << 4));
    const uint32_t mnp = low ? (z & 0x3F3Fu) : (((w >> 4) & 0x0F0Fu) | (hm << 4));
    sc0 = scp & 0xffu;
    sc1 = scp >> 8;
    m0 = mnp & 0xffu;
    m1 = mnp >> 8;
}

__device__ __forceinline__ void mma_q4k_block(uint32_t rowg, uint32_t row_stride, int kabs, const XF &x, int lane,
                                              int M, float acc[2]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t rowg8 = rowg + 8u * row_stride;
    const uint4 hg = lds128(rowg), hg8 = lds128(rowg8);
    uint32_t scl[2], sch[2], mm[2];
    float d[2], dmin[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint4 h = r ? hg8 : hg;
        uint32_t c0, c1, n0, n1;
        q4k_codes(h, t, c0, c1, n0, n1);
        scl[r] = half2_dup(static_cast<float>(c0));
        sch[r] = half2_dup(static_cast<float>(c1) * 0.0625f);
        mm[r] = pack_half2_bits(__float2half_rn(static_cast<float>(n0)), __float2half_rn(static_cast<float>(n1)));
        d[r] = half_bits_to_float(h.x) * 16777216.0f;
        dmin[r] = half_bits_to_float(h.x >> 16);
    }
    const uint4 w0 = lds128(rowg + 16 + 32 * t), w1 = lds128(rowg + 32 + 32 * t);
    const uint4 v0 = lds128(rowg8 + 16 + 32 * t), v1 = lds128(rowg8 + 32 + 32 * t);
    const int bm = min(g >> 1, M - 1);
    const int sb = kabs >> 8;
    const uint32_t xb = x.perm + static_cast<uint32_t>(bm * x.row_bytes + 576 * sb + 144 * t);
    uint32_t bl[16], bh[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 a = lds128(xb + 16 * i), b = lds128(xb + 64 + 16 * i);
        bl[4 * i] = a.x;
        bl[4 * i + 1] = a.y;
        bl[4 * i + 2] = a.z;
        bl[4 * i + 3] = a.w;
        bh[4 * i] = b.x;
        bh[4 * i + 1] = b.y;
        bh[4 * i + 2] = b.z;
        bh[4 * i + 3] = b.w;
    }
    const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const uint32_t V[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    float D[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t w = W[j], v = V[j];
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            const uint32_t a[4] = {hmul2_bits(w & 0x000F000Fu, scl[0]), hmul2_bits(v & 0x000F000Fu, scl[1]),
                                   hmul2_bits(w & 0x00F000F0u, sch[0]), hmul2_bits(v & 0x00F000F0u, sch[1])};
            mma_f16_16816(D, a, bl[2 * j + p], bh[2 * j + p]);
            w >>= 8;
            v >>= 8;
        }
    }
    const uint32_t xs = x.sum + static_cast<uint32_t>(bm * x.sum_row + 32 * sb + 4 * t);
    const uint32_t am[4] = {mm[0], mm[1], mm[0], mm[1]};
    float E[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    mma_f16_16816(E, am, lds32(xs), lds32(xs + 16));
    acc[0] += fmaf(d[0], D[0], -dmin[0] * E[0]);
    acc[1] += fmaf(d[1], D[2], -dmin[1] * E[2]);
}

// Item cursor of one warp: CTA iteration `it`, j-th item of the warp in that
// iteration.  Items of a row block are its segments seg0, seg0 + wpb, ...;
// with SwiGLU every segment is two items (gate rows, then up rows).
struct MmaCursor {
    int64_t it;
    int j;
};

__device__ __forceinline__ int64_t mma_block(const QParams &p, int64_t it, int warp) {
    return (static_cast<int64_t>(blockIdx.x) + it * gridDim.x) * p.bpc + warp / p.wpb;
}

__device__ __forceinline__ int mma_items(const QParams &p, int warp) {
    const int segs = (p.nseg - warp % p.wpb + p.wpb - 1) / p.wpb;
    return p.mode == MODE_SWIGLU ? 2 * segs : segs;
}

__device__ __forceinline__ bool mma_valid(const QParams &p, const MmaCursor &c, int warp, int64_t iters) {
    return c.it < iters && mma_block(p, c.it, warp) < p.total_rowsets;
}

__device__ __forceinline__ void mma_advance(const QParams &p, MmaCursor &c, int warp) {
    if (++c.j == mma_items(p, warp)) {
        c.j = 0;
        ++c.it;
    }
}

// Issues item j of a row block: one 16-row x 288-byte TMA box.
__device__ __forceinline__ void mma_issue(const QParams &p, int warp, int64_t block, int j, uint8_t *stage,
                                          uint64_t *bar) {
    const bool swiglu = p.mode == MODE_SWIGLU;
    const int si = swiglu ? (j & 1) : stream_of(p, block);
    const int seg = warp % p.wpb + (swiglu ? (j >> 1) : j) * p.wpb;
    const int row0 = static_cast<int>((block - p.s[swiglu ? 0 : si].rs_begin) * kMmaRows);
    // rows past N are zero-filled by the TMA unit and still count toward the transaction bytes
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kMmaRows * kMmaSegBytes));
    tma_load_2d(stage, &p.tmap[si], seg * (kMmaSegBytes / 4), row0, bar);
}

// Split-K partials of a row block meet in shared memory: each warp of the
// block's group stores its rows in its own slot, and the last to arrive adds
// the group's slots in warp order and applies the epilogue.  The slots of
// (iteration % kMmaSlots, group) are reused once the previous use is done
// (generation counter); the wait for that is bounded.
constexpr int kMmaSlots = 4;
struct MmaSlot {
    float v[2][kMmaRows][4];  // one warp's partial sums: [gate/up or value][row][batch row]
    int arrived;
    int gen;
};

__device__ __forceinline__ bool slot_wait_gen(volatile int *gen, int want) {
    if (*gen == want) return true;
    const uint64_t start = global_timer_ns();
    while (*gen != want) {
        __nanosleep(64);
        if (global_timer_ns() - start > 2000000000ull) return false;
    }
    return true;
}

template <int MT>
__device__ __forceinline__ void mma_finish_block(const QParams &p, int64_t block, const float v[2][2], int lane,
                                                 const float *res_pre = nullptr) {
    const bool swiglu = p.mode == MODE_SWIGLU;
    const int g = lane >> 2, t = lane & 3;
    const int si = swiglu ? 0 : stream_of(p, block);
    const QStream &st = p.s[si];
    const int64_t row0 = (block - st.rs_begin) * kMmaRows;
    const int64_t na = row0 + g, nb = row0 + g + 8;
    if (p.mode == MODE_ARGMAX) {
        // groups of 4 rows: lanes (g, t) with g in one quad; ties keep the lower row
        float best[2] = {na < st.n ? v[0][0] : -INFINITY, nb < st.n ? v[0][1] : -INFINITY};
        uint32_t tok[2] = {static_cast<uint32_t>(na), static_cast<uint32_t>(nb)};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
            for (int o = 4; o <= 8; o <<= 1) {
                const float ob = __shfl_xor_sync(0xffffffffu, best[h], o);
                const uint32_t ot = __shfl_xor_sync(0xffffffffu, tok[h], o);
                if (ob > best[h] || (ob == best[h] && ot < tok[h])) {
                    best[h] = ob;
                    tok[h] = ot;
                }
            }
        }
        if ((g & 3) == 0 && t < p.M) {
            if (na < st.n) {
                p.ps[t * p.G + (na >> 2)] = best[0];
                p.pt[t * p.G + (na >> 2)] = tok[0];
            }
            if (nb < st.n) {
                p.ps[t * p.G + (nb >> 2)] = best[1];
                p.pt[t * p.G + (nb >> 2)] = tok[1];
            }
        }
        return;
    }
    if (t >= p.M) return;
    const int64_t rows[2] = {na, nb};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (rows[h] >= st.n) continue;
        const int64_t o = t * st.n + rows[h];
        float val;
        if (swiglu) {
            val = silu(v[0][h]) * v[1][h];
        } else {
            val = v[0][h];
            if (res_pre) {
                val += res_pre[h];
            } else if (st.res) {
                val += __half2float(st.res[o]);
            }
        }
        st.y[o] = __float2half_rn(val);
    }
}

template <int MT>
__global__ void __launch_bounds__(kMmaThreads, 1) qmv_mma_kernel(const __grid_constant__ QParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = p.K;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    const bool swiglu = p.mode == MODE_SWIGLU;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem) + warp * kMaxStages;
    uint8_t *stages = smem + kStageHead + static_cast<size_t>(warp) * S * p.stage_bytes;
    MmaSlot *slots = reinterpret_cast<MmaSlot *>(smem + kStageHead + static_cast<size_t>(kMmaWarps) * S * p.stage_bytes);
    uint8_t *xperm = reinterpret_cast<uint8_t *>(slots + kMmaSlots * kMmaWarps);
    uint8_t *xsum = xperm + MT * xf_row_bytes(K);
    float *pred = reinterpret_cast<float *>(xsum + MT * (K >> 8) * 32);
    const int64_t iters = (p.total_rowsets + static_cast<int64_t>(gridDim.x) * p.bpc - 1) /
                          (static_cast<int64_t>(gridDim.x) * p.bpc);
    const int group = warp / p.wpb;

    MmaCursor ahead{0, 0};
    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
        for (int i = 0; i < S && mma_valid(p, ahead, warp, iters); ++i) {
            mma_issue(p, warp, mma_block(p, ahead.it, warp), ahead.j, stages + static_cast<size_t>(i) * p.stage_bytes,
                      &full[i]);
            mma_advance(p, ahead, warp);
        }
    }
    for (int i = threadIdx.x; i < kMmaSlots * kMmaWarps * static_cast<int>(sizeof(MmaSlot) / 4); i += kMmaThreads)
        reinterpret_cast<int *>(slots)[i] = 0;
    pdl_wait();
    pdl_trigger();
    prepare_x_f16<MT, kMmaThreads>(p, xperm, xsum, pred);  // ends with a CTA barrier
    const XF x{smem_u32(xperm), smem_u32(xsum), xf_row_bytes(K), (K >> 8) * 32};
    ahead = MmaCursor{0, 0};
    for (int i = 0; i < S && mma_valid(p, ahead, warp, iters); ++i) mma_advance(p, ahead, warp);

    const uint32_t stages_addr = smem_u32(stages);
    const int items = mma_items(p, warp);
    const int g = lane >> 2, t = lane & 3;
    int s = 0;
    uint32_t phase = 0;
    bool failed = false;
    for (int64_t it = 0; it < iters; ++it) {
        const int64_t block = mma_block(p, it, warp);
        if (block >= p.total_rowsets) break;  // later iterations have no block either
        float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        for (int j = 0; j < items; ++j) {
            if (!failed && !mbar_wait(&full[s], phase)) {
                report_device_error(T2C_ETIMEOUT);
                failed = true;
            }
            if (!failed) {
                const uint32_t stage = stages_addr + static_cast<uint32_t>(s) * static_cast<uint32_t>(p.stage_bytes);
                const bool up = swiglu && (j & 1);
                const int seg = warp % p.wpb + (swiglu ? (j >> 1) : j) * p.wpb;
                const int kseg = seg * kMmaSegBlocks * 256;
                float part[2] = {0.0f, 0.0f};
#pragma unroll
                for (int sb = 0; sb < kMmaSegBlocks; ++sb)
                    mma_q4k_block(stage + static_cast<uint32_t>(g * kMmaSegBytes + sb * 144), kMmaSegBytes,
                                  kseg + sb * 256, x, lane, p.M, part);
                acc[0][0] += up ? 0.0f : part[0];
                acc[0][1] += up ? 0.0f : part[1];
                acc[1][0] += up ? part[0] : 0.0f;
                acc[1][1] += up ? part[1] : 0.0f;
                __syncwarp();
                if (lane == 0 && mma_valid(p, ahead, warp, iters)) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mma_issue(p, warp, mma_block(p, ahead.it, warp), ahead.j,
                              stages + static_cast<size_t>(s) * p.stage_bytes, &full[s]);
                }
                if (mma_valid(p, ahead, warp, iters)) mma_advance(p, ahead, warp);
            }
            if (++s == S) {
                s = 0;
                phase ^= 1u;
            }
        }
        if (p.wpb == 1) {
            mma_finish_block<MT>(p, block, acc, lane);
            continue;
        }
        // each warp parks its partial sums in its own slot; the group's last warp adds them in warp
        // order (a fixed summation order: results do not depend on which warp finishes first).  The
        // group's first slot carries the arrival count and the generation.
        MmaSlot *const base = slots + (it % kMmaSlots) * kMmaWarps + group * p.wpb;
        MmaSlot *const mine = slots + (it % kMmaSlots) * kMmaWarps + warp;
        if (!slot_wait_gen(&base->gen, static_cast<int>(it / kMmaSlots))) {
            report_device_error(T2C_ETIMEOUT);
            failed = true;
            continue;
        }
        if (t < p.M) {  // lane (g, t) holds rows g, g+8 of batch row t
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                mine->v[r][g][t] = acc[r][0];
                mine->v[r][g + 8][t] = acc[r][1];
            }
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&base->arrived, 1) == p.wpb - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence_block();
        float v[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        const int tm = t < p.M ? t : 0;
        for (int w = 0; w < p.wpb; ++w) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                v[r][0] += *reinterpret_cast<volatile float *>(&base[w].v[r][g][tm]);
                v[r][1] += *reinterpret_cast<volatile float *>(&base[w].v[r][g + 8][tm]);
            }
        }
        mma_finish_block<MT>(p, block, v, lane);
        __syncwarp();
        if (lane == 0) {
            base->arrived = 0;
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&base->gen) = base->gen + 1;
        }
    }
}

// ------------------------------------------------ M = 1 kernel, per-warp x
// Same streaming and split-K as qmv_mma_kernel, but each warp prepares only
// the x values of its own K-segments (after, when there is a fused RMSNorm,
// a warp-local sum of squares over the whole row), so the prologue has no
// CTA barrier and x costs ~1.1 KB of shared memory per segment: two CTAs fit
// on an SM.  x keeps the reference's arithmetic: the (normalized) values are
// rounded to fp16 once, like the reference's fp16 activation tensor, and enter
// the fp16 tensor-core products unchanged.  Per 512-value segment:
//   [0, 1024)     fp16 x in pair-interleaved 4-value chunks (x0, x2, x1, x3),
//                 so that every 32-bit word is one mma B pair (k, k + 2);
//   [1024, 1088)  fp32 sums of the segment's 16 sub-blocks (32 values each);
//   [1088, 1152)  zeros: the B source of lanes whose mma column is unused.
constexpr int kM1SegSum = 1024;
constexpr int kM1SegZero = 1088;
constexpr int kM1SegBytes = 1152;
constexpr int kM1MaxSegs = 16;                   // per warp (K <= 65536)
constexpr int kM1XReg = 4;                       // segments whose x loads are issued together

// x values [k0, k0 + 512) of a segment: lane l holds values 16 l .. 16 l + 15.
__device__ __forceinline__ void m1_load_x(const QParams &p, int k0, int lane, float f[16]) {
    const uint4 *xv = reinterpret_cast<const uint4 *>(p.x + k0 + 16 * lane);
    unpack8(xv[0], f);
    unpack8(xv[1], f + 8);
}
__device__ __forceinline__ void m1_load_norm(const QParams &p, int k0, int lane, float w[16]) {
    const float4 *wv = reinterpret_cast<const float4 *>(p.norm_w + k0 + 16 * lane);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float4 w4 = wv[i];
        w[4 * i] = w4.x;
        w[4 * i + 1] = w4.y;
        w[4 * i + 2] = w4.z;
        w[4 * i + 3] = w4.w;
    }
}

// Rounds one segment of x (f, already scaled by the RMSNorm when there is
// one) to fp16 and writes it, its sub-block sums and the zero area.
__device__ __forceinline__ void m1_prepare_segment(const float f[16], uint8_t *area, int lane) {
    __half h[16];
    float sum = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        h[e] = __float2half_rn(f[e]);
        sum += __half2float(h[e]);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);  // lanes 2i, 2i+1 = sub-block i
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[2 * i] = pack_half2_bits(h[4 * i], h[4 * i + 2]);
        w[2 * i + 1] = pack_half2_bits(h[4 * i + 1], h[4 * i + 3]);
    }
    *reinterpret_cast<uint4 *>(area + 32 * lane) = make_uint4(w[0], w[1], w[2], w[3]);
    *reinterpret_cast<uint4 *>(area + 32 * lane + 16) = make_uint4(w[4], w[5], w[6], w[7]);
    if ((lane & 1) == 0) *reinterpret_cast<float *>(area + kM1SegSum + 4 * (lane >> 1)) = sum;
    if (lane < 4) *reinterpret_cast<uint4 *>(area + kM1SegZero + 16 * lane) = make_uint4(0u, 0u, 0u, 0u);
}

// Residual values of rows g, g + 8 of row block `blk` (lane t == 0), read
// well before the epilogue that adds them.
__device__ __forceinline__ void m1_load_res(const QParams &p, int blk, int lane, float rv[2]) {
    rv[0] = rv[1] = 0.0f;
    if (p.mode != MODE_ROWS || (lane & 3) != 0) return;
    const QStream &st = p.s[p.nstreams > 1 ? stream_of(p, blk) : 0];
    if (st.res == nullptr) return;
    const int64_t row = (blk - st.rs_begin) * kMmaRows + (lane >> 2);
    if (row < st.n) rv[0] = __half2float(st.res[row]);
    if (row + 8 < st.n) rv[1] = __half2float(st.res[row + 8]);
}

// Fragment mapping of the M = 1 kernel (mma m16n8k16, f16 inputs, fp32
// accumulators; A = 16 weight rows, B = x).  Lane (g, t) reads group t (bytes
// 32 t .. 32 t + 31 of the 128 nibble bytes) of rows g and g + 8 of a Q4_K
// block: the low nibbles are sub-block 2t, the high nibbles sub-block 2t + 1.
// The nibbles enter the mma as fp16 subnormals by masking alone: q * 2^-24
// (low) and 16 q * 2^-24 (high), exact.  mma (j, p) (word j, byte parity p)
// gives lane t's k-slots {2t, 2t + 1} the low nibbles of bytes 4j + p and
// 4j + p + 2, and k-slots {2t + 8, 2t + 9} their high nibbles.  B column 2t
// carries the x values of the low slots of lane t, column 2t + 1 those of its
// high slots, zero elsewhere, so D columns 2t, 2t + 1 of lane (g, t) are
// exactly the sums q * x over sub-blocks 2t and 2t + 1 of rows g, g + 8: every
// lane applies the scales of its own two sub-blocks, and the four lanes of a
// quad are summed per row block at the end.
struct M1Lane {
    uint32_t aoff;           // group t's bytes in a 144-byte block
    uint32_t b0off, b0step;  // B source of the low slots (segment-relative; step per super-block)
    uint32_t b1off, b1step;  // B source of the high slots
    uint32_t soff;           // sums of sub-blocks 2t, 2t + 1 of super-block 0
    // scale decode of sub-blocks 2t, 2t + 1: header bytes (2t, 2t + 1) mod 4 by byte_perm `sel`, then
    // codes = (W & mw) | ((Y >> sy) & my) (t < 2: the 6-bit bytes of Y; t >= 2: low / high nibbles of W
    // with the top two bits of Y / Z)
    uint32_t sel, mw, my, sy;
};

__device__ __forceinline__ M1Lane m1_lane(int lane) {
    const int g = lane >> 2, t = lane & 3, h = g - 2 * t;
    M1Lane L;
    L.aoff = static_cast<uint32_t>(16 + 32 * t);
    L.b0off = h == 0 ? static_cast<uint32_t>(128 * t) : static_cast<uint32_t>(kM1SegZero);
    L.b0step = h == 0 ? 512u : 0u;
    L.b1off = h == 1 ? static_cast<uint32_t>(128 * t + 64) : static_cast<uint32_t>(kM1SegZero);
    L.b1step = h == 1 ? 512u : 0u;
    L.soff = static_cast<uint32_t>(kM1SegSum + 8 * t);
    const uint32_t b = static_cast<uint32_t>((2 * t) & 3);
    L.sel = 0x4400u | ((b + 1) << 4) | b;
    L.mw = t < 2 ? 0u : 0x0F0Fu;
    L.my = t < 2 ? 0x3F3Fu : 0x3030u;
    L.sy = t < 2 ? 0u : 2u;
    return L;
}

// d * sc * 2^24, d * sc * 2^20 (the high nibbles enter as 16 q) and dmin * m
// of sub-blocks 2t, 2t + 1 of one Q4_K header.  Codes become floats through
// the 2^23 mantissa trick folded into one exact fma: s * (2^23 + c) - s * 2^23.
__device__ __forceinline__ void m1_scales(const uint4 h, const M1Lane &L, float ds[2], float dm[2]) {
    const uint32_t Y = __byte_perm(h.y, 0u, L.sel), Z = __byte_perm(h.z, 0u, L.sel), W = __byte_perm(h.w, 0u, L.sel);
    const uint32_t scp = (W & L.mw) | ((Y >> L.sy) & L.my);
    const uint32_t mnp = ((W >> 4) & L.mw) | ((Z >> L.sy) & L.my);
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const float d24 = d * 16777216.0f, d20 = d * 1048576.0f;
    ds[0] = fmaf(d24, __uint_as_float(__byte_perm(scp, 0x4B000000u, 0x7540u)), -d24 * 8388608.0f);
    ds[1] = fmaf(d20, __uint_as_float(__byte_perm(scp, 0x4B000000u, 0x7541u)), -d20 * 8388608.0f);
    dm[0] = fmaf(dmin, __uint_as_float(__byte_perm(mnp, 0x4B000000u, 0x7540u)), -dmin * 8388608.0f);
    dm[1] = fmaf(dmin, __uint_as_float(__byte_perm(mnp, 0x4B000000u, 0x7541u)), -dmin * 8388608.0f);
}

// One 144-byte block (super-block sb of the segment) of a 16-row group whose
// rows are kMmaSegBytes apart; acc = rows g, g + 8.
__device__ __forceinline__ void m1_block(const uint8_t *rowg, const uint8_t *xseg, int sb, const M1Lane &L,
                                         float acc[2]) {
    const uint8_t *rowg8 = rowg + 8 * kMmaSegBytes;
    const uint4 hg = *reinterpret_cast<const uint4 *>(rowg), hg8 = *reinterpret_cast<const uint4 *>(rowg8);
    float ds[2][2], dm[2][2];
    m1_scales(hg, L, ds[0], dm[0]);
    m1_scales(hg8, L, ds[1], dm[1]);
    const uint4 w0 = *reinterpret_cast<const uint4 *>(rowg + L.aoff);
    const uint4 w1 = *reinterpret_cast<const uint4 *>(rowg + L.aoff + 16);
    const uint4 v0 = *reinterpret_cast<const uint4 *>(rowg8 + L.aoff);
    const uint4 v1 = *reinterpret_cast<const uint4 *>(rowg8 + L.aoff + 16);
    const uint8_t *b0p = xseg + L.b0off + sb * L.b0step;
    const uint8_t *b1p = xseg + L.b1off + sb * L.b1step;
    uint32_t bl[16], bh[16];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 a = *reinterpret_cast<const uint4 *>(b0p + 16 * i);
        const uint4 b = *reinterpret_cast<const uint4 *>(b1p + 16 * i);
        bl[4 * i] = a.x;
        bl[4 * i + 1] = a.y;
        bl[4 * i + 2] = a.z;
        bl[4 * i + 3] = a.w;
        bh[4 * i] = b.x;
        bh[4 * i + 1] = b.y;
        bh[4 * i + 2] = b.z;
        bh[4 * i + 3] = b.w;
    }
    const uint32_t W[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
    const uint32_t V[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    // two accumulator chains (even / odd byte parity) halve the dependent mma latency
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f}, e[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        // byte shifts on the multiply pipe (high half of w * 2^24), the masks on the logic pipe
        const uint32_t w = W[j], v = V[j], w8 = __umulhi(w, 1u << 24), v8 = __umulhi(v, 1u << 24);
        const uint32_t a0[4] = {w & 0x000F000Fu, v & 0x000F000Fu, w & 0x00F000F0u, v & 0x00F000F0u};
        const uint32_t a1[4] = {w8 & 0x000F000Fu, v8 & 0x000F000Fu, w8 & 0x00F000F0u, v8 & 0x00F000F0u};
        mma_f16_16816(d, a0, bl[2 * j], bh[2 * j]);
        mma_f16_16816(e, a1, bl[2 * j + 1], bh[2 * j + 1]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] += e[i];
    const float2 xs = *reinterpret_cast<const float2 *>(xseg + L.soff + 32 * sb);
    // ds carries the 2^24 (low) and 2^20 (high) of the subnormal weights
    acc[0] += fmaf(ds[0][0], d[0], fmaf(ds[0][1], d[1], -fmaf(dm[0][0], xs.x, dm[0][1] * xs.y)));
    acc[1] += fmaf(ds[1][0], d[2], fmaf(ds[1][1], d[3], -fmaf(dm[1][0], xs.x, dm[1][1] * xs.y)));
}

// Split-K slot of the M = 1 kernel: each warp of a row block's group stores
// its partial sums in its own column; the last warp to arrive adds the
// columns in warp order (the result does not depend on arrival order).
struct M1Slot {
    float v[2][kMmaRows][kMmaWarps];  // [gate/up or value][row][warp of the group]
    int arrived;
    int gen;
};

// Item j of row block `blk` (segment seg0 + j * wpb; SwiGLU: gate / up
// alternate) as one 16-row x 288-byte TMA box.
__device__ __forceinline__ void m1_issue(const QParams &p, int blk, int j, int seg0, uint8_t *stage, uint64_t *bar) {
    const bool swiglu = p.mode == MODE_SWIGLU;
    int si = 0, jj = j;
    if (swiglu) {
        si = j & 1;
        jj = j >> 1;
    } else if (p.nstreams > 1) {
        si = stream_of(p, blk);
    }
    const int row0 = (blk - static_cast<int>(p.s[swiglu ? 0 : si].rs_begin)) * kMmaRows;
    // rows past N are zero-filled by the TMA unit and still count toward the transaction bytes
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(kMmaRows * kMmaSegBytes));
    tma_load_2d(stage, &p.tmap[si], (seg0 + jj * p.wpb) * (kMmaSegBytes / 4), row0, bar);
}

// Row-parallel tensor parallelism (M = 1), push side: the fp32 partials of block blk's 16 rows
// (lanes t == 0: rows g and g + 8) go into slot `rank` of every rank's region of this launch's
// epoch parity (plain stores, over NVLink for the peers).
__device__ __forceinline__ float *ar_slot(const QParams &p, int owner, uint32_t epoch, int src) {
    return reinterpret_cast<float *>(p.ar_peer[owner] + kArFlagBytes) +
           (static_cast<int64_t>(epoch & 1u) * kArMaxRanks + src) * p.ar_nmax;
}
__device__ __forceinline__ void m1_ar_push(const QParams &p, int64_t blk, const float v[2][2], int lane, uint32_t epoch) {
    if ((lane & 3) != 0) return;
    const int g = lane >> 2;
    const int64_t row0 = (blk - p.s[0].rs_begin) * kMmaRows;
    for (int q = 0; q < p.ar_tp; ++q) {
        float *dst = ar_slot(p, q, epoch, p.ar_rank);
        dst[row0 + g] = v[0][0];
        dst[row0 + g + 8] = v[0][1];
    }
}

// Pull side, once per CTA after all of its blocks are pushed: a system-scope release of this
// launch's epoch into flag (CTA, rank) of every rank, a bounded acquire-wait for every
// rank's flag (CTA, peer) (the peer's CTA of the same index pushed the same blocks), then every
// row of the CTA's blocks = residual + the ranks' partials summed in rank order (the same
// order on every rank: every rank holds the same bits).  Each rank reads a parity region
// before its next launch releases the flags, and a region is rewritten only two launches later.
// A peer that does not arrive within a second: T2C_ETIMEOUT, the rows keep this rank's partial.
__device__ __forceinline__ void m1_ar_finish(const QParams &p, uint32_t epoch) {
    const int tid = threadIdx.x, tp = p.ar_tp, rank = p.ar_rank, cta = blockIdx.x;
    __syncthreads();
    if (tid < tp)  // a system-scope release: every lane's pushes are ordered before it by the barrier above
        ar_store_release(reinterpret_cast<uint32_t *>(p.ar_peer[tid]) + cta * kArMaxRanks + rank, epoch);
    __syncthreads();
    int arrived = 1;
    if (tid < tp) {
        const uint32_t *flag = reinterpret_cast<const uint32_t *>(p.ar_peer[rank]) + cta * kArMaxRanks + tid;
        if (ar_load_acquire(flag) < epoch) {
            const uint64_t start = global_timer_ns();
            while (ar_load_acquire(flag) < epoch) {
                if (global_timer_ns() - start > 1000000000ull) {
                    arrived = 0;
                    report_device_error(T2C_ETIMEOUT);
                    break;
                }
            }
        }
    }
    const bool ok = __syncthreads_and(arrived) != 0;
    const QStream &st = p.s[0];
    const int total = static_cast<int>(p.total_rowsets), step = static_cast<int>(gridDim.x) * p.bpc;
    // the CTA's rows: groups g of blocks first + g + i * step, 16 rows each
    const int per_pass = p.bpc * kMmaRows;
    for (int64_t pass = 0;; ++pass) {
        const int64_t first = static_cast<int64_t>(cta) * p.bpc + pass * step;
        if (first >= total) break;
        for (int e = tid; e < per_pass; e += blockDim.x) {
            const int64_t blk = first + e / kMmaRows;
            if (blk >= total) continue;
            const int64_t row = (blk - st.rs_begin) * kMmaRows + e % kMmaRows;
            if (row >= st.n) continue;
            float acc;
            if (ok) {
                acc = 0.0f;
                for (int q = 0; q < tp; ++q) acc += __ldcv(ar_slot(p, rank, epoch, q) + row);
            } else {
                acc = __ldcv(ar_slot(p, rank, epoch, rank) + row);
            }
            if (st.res != nullptr) acc += __half2float(st.res[row]);
            st.y[row] = __float2half_rn(acc);
        }
    }
}

__global__ void __launch_bounds__(kMmaThreads, 2) qmv_m1_kernel(const __grid_constant__ QParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = p.stages;
    const bool swiglu = p.mode == MODE_SWIGLU;
    // per-warp constants: row-block group, first segment, items per row block
    const int group = warp / p.wpb, seg0 = warp % p.wpb;
    const int nsegw = (p.nseg - seg0 + p.wpb - 1) / p.wpb;
    const int items = swiglu ? 2 * nsegw : nsegw;
    const int total = static_cast<int>(p.total_rowsets);
    const int step = static_cast<int>(gridDim.x) * p.bpc;
    const int first = static_cast<int>(blockIdx.x) * p.bpc + group;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem) + warp * kMaxStages;
    uint8_t *stages = smem + kStageHead + static_cast<size_t>(warp) * S * p.stage_bytes;
    uint8_t *xarea = smem + kStageHead + static_cast<size_t>(kMmaWarps) * S * p.stage_bytes +
                     static_cast<size_t>(warp) * p.xseg_per_warp * kM1SegBytes;
    M1Slot *slots = reinterpret_cast<M1Slot *>(smem + kStageHead + static_cast<size_t>(kMmaWarps) * S * p.stage_bytes +
                                                 static_cast<size_t>(kMmaWarps) * p.xseg_per_warp * kM1SegBytes);

    // producer cursor (warp-uniform; lane 0 issues)
    int pblk = first, pj = 0;
    if (lane == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
    }
    for (int i = 0; i < S && pblk < total; ++i) {
        if (lane == 0) m1_issue(p, pblk, pj, seg0, stages + static_cast<size_t>(i) * p.stage_bytes, &full[i]);
        if (++pj == items) {
            pj = 0;
            pblk += step;
        }
    }
    for (int i = threadIdx.x; i < kMmaSlots * p.bpc * static_cast<int>(sizeof(M1Slot) / 4); i += kMmaThreads)
        reinterpret_cast<int *>(slots)[i] = 0;
    // RMSNorm weights of the first segment: weights, like the matrix rows, are
    // never written by the preceding kernel, so they load before the wait
    float nw[16];
    const bool norm = p.norm_w != nullptr;
    if (norm && nsegw > 0) m1_load_norm(p, seg0 * (kMmaSegBlocks * 256), lane, nw);
    __syncthreads();  // slot zeroing visible to every warp
    pdl_wait();
    pdl_trigger();
    float rv[2];
    if (first < total) m1_load_res(p, first, lane, rv);
    // tensor-parallel epoch of this launch (the counter moves on only after every CTA has read it)
    const uint32_t ar_epoch = p.ar_tp > 1 ? *reinterpret_cast<volatile const uint32_t *>(p.ar_counter) + 1u : 0u;
    // this warp's x segments (the first one stays in registers); with a fused
    // RMSNorm the wpb warps of a group (which together hold every segment of
    // the row) add their sums of squares through shared memory (one CTA barrier)
    // every x load of this warp's first kM1XReg segments is issued before any is used: one
    // round trip to L2 instead of one per segment (x was just written by the preceding kernel)
    uint4 xr[kM1XReg][2];
#pragma unroll
    for (int j = 0; j < kM1XReg; ++j) {
        if (j < nsegw) {
            const uint4 *xv = reinterpret_cast<const uint4 *>(p.x + (seg0 + j * p.wpb) * (kMmaSegBlocks * 256) + 16 * lane);
            xr[j][0] = xv[0];
            xr[j][1] = xv[1];
        }
    }
    float inv_rms = 1.0f;
    if (norm) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < kM1XReg; ++j) {
            if (j < nsegw) {
                float f[16];
                unpack8(xr[j][0], f);
                unpack8(xr[j][1], f + 8);
#pragma unroll
                for (int e = 0; e < 16; ++e) ss = fmaf(f[e], f[e], ss);
            }
        }
        for (int j = kM1XReg; j < nsegw; ++j) {
            float f[16];
            m1_load_x(p, (seg0 + j * p.wpb) * (kMmaSegBlocks * 256), lane, f);
#pragma unroll
            for (int e = 0; e < 16; ++e) ss = fmaf(f[e], f[e], ss);
        }
        ss = warp_sum(ss);
        float *sq = reinterpret_cast<float *>(slots + kMmaSlots * p.bpc);
        if (lane == 0) sq[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = group * p.wpb; w < (group + 1) * p.wpb; ++w) tot += sq[w];
        inv_rms = rsqrtf(tot / static_cast<float>(p.K) + p.eps);
    }
    auto prep = [&](int j, float f[16]) {
        const int k0 = (seg0 + j * p.wpb) * (kMmaSegBlocks * 256);
        float w[16];
        if (norm) {
            if (j == 0) {
#pragma unroll
                for (int e = 0; e < 16; ++e) w[e] = nw[e];
            } else {
                m1_load_norm(p, k0, lane, w);
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) f[e] *= inv_rms * w[e];
        }
        m1_prepare_segment(f, xarea + j * kM1SegBytes, lane);
    };
#pragma unroll
    for (int j = 0; j < kM1XReg; ++j) {
        if (j < nsegw) {
            float f[16];
            unpack8(xr[j][0], f);
            unpack8(xr[j][1], f + 8);
            prep(j, f);
        }
    }
    for (int j = kM1XReg; j < nsegw; ++j) {
        float f[16];
        m1_load_x(p, (seg0 + j * p.wpb) * (kMmaSegBlocks * 256), lane, f);
        prep(j, f);
    }
    __syncwarp();

    const M1Lane L = m1_lane(lane);
    const int g = lane >> 2, t = lane & 3;
    int s = 0, it = 0;
    uint32_t phase = 0;
    bool failed = false;
    for (int blk = first; blk < total; blk += step, ++it) {
        if (it > 0) m1_load_res(p, blk, lane, rv);
        float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        for (int j = 0; j < items; ++j) {
            if (!failed && !mbar_wait(&full[s], phase)) {
                report_device_error(T2C_ETIMEOUT);
                failed = true;
            }
            if (!failed) {
                const uint8_t *stage = stages + static_cast<size_t>(s) * p.stage_bytes + g * kMmaSegBytes;
                const uint8_t *xseg = xarea + (swiglu ? (j >> 1) : j) * kM1SegBytes;
                float part[2] = {0.0f, 0.0f};
#pragma unroll
                for (int sb = 0; sb < kMmaSegBlocks; ++sb) m1_block(stage + sb * 144, xseg, sb, L, part);
                if (swiglu && (j & 1)) {
                    acc[1][0] += part[0];
                    acc[1][1] += part[1];
                } else {
                    acc[0][0] += part[0];
                    acc[0][1] += part[1];
                }
                __syncwarp();
                if (pblk < total) {
                    if (lane == 0) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        m1_issue(p, pblk, pj, seg0, stages + static_cast<size_t>(s) * p.stage_bytes, &full[s]);
                    }
                    if (++pj == items) {
                        pj = 0;
                        pblk += step;
                    }
                }
            }
            if (++s == S) {
                s = 0;
                phase ^= 1u;
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                acc[r][h] += __shfl_xor_sync(0xffffffffu, acc[r][h], 1);
                acc[r][h] += __shfl_xor_sync(0xffffffffu, acc[r][h], 2);
            }
        if (p.wpb == 1) {
            if (p.ar_tp > 1)
                m1_ar_push(p, blk, acc, lane, ar_epoch);
            else
                mma_finish_block<1>(p, blk, acc, lane, rv);
            continue;
        }
        M1Slot *slot = slots + (it % kMmaSlots) * p.bpc + group;
        if (!slot_wait_gen(&slot->gen, it / kMmaSlots)) {
            report_device_error(T2C_ETIMEOUT);
            failed = true;
            continue;
        }
        if (t == 0) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                slot->v[r][g][seg0] = acc[r][0];
                slot->v[r][g + 8][seg0] = acc[r][1];
            }
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&slot->arrived, 1) == p.wpb - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence_block();
        float v[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        for (int w = 0; w < p.wpb; ++w) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                v[r][0] += *reinterpret_cast<volatile float *>(&slot->v[r][g][w]);
                v[r][1] += *reinterpret_cast<volatile float *>(&slot->v[r][g + 8][w]);
            }
        }
        if (p.ar_tp > 1)
            m1_ar_push(p, blk, v, lane, ar_epoch);
        else
            mma_finish_block<1>(p, blk, v, lane, rv);
        __syncwarp();
        if (lane == 0) {
            slot->arrived = 0;
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&slot->gen) = slot->gen + 1;
        }
    }
    if (p.ar_tp > 1) {
        m1_ar_finish(p, ar_epoch);
        // the launch's epoch moves on once every CTA is past its last read of it
        __syncthreads();
        if (threadIdx.x == 0) {
            const uint32_t epoch = ar_epoch;
            __threadfence();
            if (atomicAdd(&p.ar_counter[1], 1u) == gridDim.x - 1) {
                p.ar_counter[1] = 0u;
                __threadfence();
                *reinterpret_cast<volatile uint32_t *>(p.ar_counter) = epoch;
            }
        }
    }
}

// ======================================================= exact fp16-x kernel
// qmv_x16_kernel<MT>: up to MT = 4 tokens per pass (the weight words of a unit
// are loaded once and serve every token; more tokens take further passes),
// weight streams of any GGUF type (Q4_K, Q6_K, Q8_0, mixed in one fused QKV),
// modes ROWS (+ residual), SWIGLU and ARGMAX.  x keeps the
// reference's arithmetic: the (normalized) values are rounded to fp16 once
// and enter fp16 tensor-core products unchanged; every weight code enters as
// an exactly representable fp16 value and the block scales are applied in
// fp32, so the only differences from the reference's fp32 loop are fp32
// summation order and the fp16 store.
//   * Tiles of 16 rows (mma m16n8k16 A); the 8 warps of a CTA take bpc tiles
//     at a time with wpb warps per tile splitting K into 256-value units
//     (partial sums meet in shared memory in warp order: deterministic).
//   * Weights come straight from global memory (ld.global.nc), each lane
//     loading the bytes of its own two rows; x (fp16, natural order) and the
//     fp32 sums of its 32-value blocks are staged in shared memory.
//   * Columns of the mma carry scale groups, not tokens: lane t's k-slots
//     {2t, 2t + 1} belong to one group and {2t + 8, 2t + 9} to another, and
//     B column 2t (2t + 1) holds x only in the first (second) pair of slots,
//     so D columns 2t, 2t + 1 of lane (g, t) are group sums that lane t
//     scales itself; the four lanes of a quad are added at the end.
//       Q4_K: group t of each block (low nibbles: sub-block 2t, high: 2t + 1),
//             nibbles as fp16 subnormals (q * 2^-24, 16 q * 2^-24) by masking;
//             d * sc and dmin * m * xsum per sub-block in fp32.
//       Q6_K: per (half s, 16-value half lh, quarter pair cp): quarters cp and
//             cp + 2 at positions 16 lh + 4t .. + 3; the 6-bit levels L become
//             fp16 1024 + L by byte permutes and L - 32 by one f16x2 subtract
//             (exact); d * sc of the two 16-value groups in fp32.
//       Q8_0: blocks 2t and 2t + 1 of each 8-block unit; q + 128 as fp16
//             subnormals, d * (D - 128 * xsum) in fp32.
constexpr int kXWarps = 8;
constexpr int kXThreads = kXWarps * 32;

__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) { return ldg_nc_u32(p); }

// 32-bit word at a 2-byte aligned address.
__device__ __forceinline__ uint32_t ldg32_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3u) == 0) return ldg32(p);
    return __funnelshift_r(ldg32(p - 2), ldg32(p + 2), 16);
}

__device__ __forceinline__ uint32_t hsub2_bits(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ void mma_f16_16816_zc(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.0f));
}

// x of one token: fp16 [K] in natural order, fp32 sums of 32-value blocks [K / 32].
// Token m of the pass: x row m of p.x into xs + m * 2K (fp16) and xsum + m * K / 32.
__device__ void x16_prepare_token(const QParams &p, int m, uint8_t *xs, float *xsum, float *red) {
    const int K = p.K;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int chunks = K >> 3;
    const uint4 *xv = reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(m) * K);
    xs += static_cast<size_t>(m) * 2 * K;
    xsum += static_cast<size_t>(m) * (K >> 5);
    red += m * kXWarps;
    float inv_rms = 1.0f;
    if (p.norm_w != nullptr) {
        float ss = 0.0f;
        for (int c = tid; c < chunks; c += kXThreads) {
            float f[8];
            unpack8(xv[c], f);
#pragma unroll
            for (int e = 0; e < 8; ++e) ss = fmaf(f[e], f[e], ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
        for (int w = 0; w < kXWarps; ++w) tot += red[w];
        inv_rms = rsqrtf(tot / static_cast<float>(K) + p.eps);
    }
    // kXThreads and chunks are multiples of 4: lanes 4i .. 4i + 3 hold the chunks of one 32-value block
    for (int base = 0; base < chunks; base += kXThreads) {
        const int c = base + tid;
        float f[8];
        if (c < chunks) {
            unpack8(xv[c], f);
        } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.0f;
        }
        if (p.norm_w != nullptr && c < chunks) {
            const float4 w0 = *reinterpret_cast<const float4 *>(p.norm_w + 8 * c);
            const float4 w1 = *reinterpret_cast<const float4 *>(p.norm_w + 8 * c + 4);
            const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = f[e] * inv_rms * wv[e];
        }
        __half h[8];
        float sum = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            h[e] = __float2half_rn(f[e]);
            sum += __half2float(h[e]);
        }
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (c < chunks) {
            *reinterpret_cast<uint4 *>(xs + 16 * c) =
                make_uint4(pack_half2_bits(h[0], h[1]), pack_half2_bits(h[2], h[3]), pack_half2_bits(h[4], h[5]),
                           pack_half2_bits(h[6], h[7]));
            if ((lane & 3) == 0) xsum[c >> 2] = sum;
        }
    }
}

// x of the pass's p.M tokens (rows past p.M of a MT-token pass are zero), then one CTA barrier.
template <int MT>
__device__ void x16_prepare(const QParams &p, uint8_t *xs, float *xsum, float *red) {
#pragma unroll 1
    for (int m = 0; m < p.M; ++m) x16_prepare_token(p, m, xs, xsum, red);
    const int K = p.K;
    for (int i = threadIdx.x + p.M * (2 * K / 16); i < MT * (2 * K / 16); i += kXThreads)
        reinterpret_cast<uint4 *>(xs)[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = threadIdx.x + p.M * (K >> 5); i < MT * (K >> 5); i += kXThreads) xsum[i] = 0.0f;
    __syncthreads();
}

// Per-lane constants of the sparse-column mapping.
struct XLane {
    int g, t;
    uint32_t b0on, b1on;  // all-ones when this lane's B column takes the first / second slot pair
    uint32_t sel, mw, my, sy;  // Q4_K scale decode of sub-blocks 2t, 2t + 1 (as M1Lane)
};

__device__ __forceinline__ XLane x_lane(int lane) {
    XLane L;
    L.g = lane >> 2;
    L.t = lane & 3;
    const int h = L.g - 2 * L.t;
    L.b0on = h == 0 ? 0xffffffffu : 0u;
    L.b1on = h == 1 ? 0xffffffffu : 0u;
    const uint32_t b = static_cast<uint32_t>((2 * L.t) & 3);
    L.sel = 0x4400u | ((b + 1) << 4) | b;
    L.mw = L.t < 2 ? 0u : 0x0F0Fu;
    L.my = L.t < 2 ? 0x3F3Fu : 0x3030u;
    L.sy = L.t < 2 ? 0u : 2u;
    return L;
}

// d * sc * 2^24, d * sc * 2^20 and dmin * m of sub-blocks 2t, 2t + 1 (see m1_scales).
__device__ __forceinline__ void x_q4k_scales(const uint4 h, const XLane &L, float ds[2], float dm[2]) {
    const uint32_t Y = __byte_perm(h.y, 0u, L.sel), Z = __byte_perm(h.z, 0u, L.sel), W = __byte_perm(h.w, 0u, L.sel);
    const uint32_t scp = (W & L.mw) | ((Y >> L.sy) & L.my);
    const uint32_t mnp = ((W >> 4) & L.mw) | ((Z >> L.sy) & L.my);
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const float d24 = d * 16777216.0f, d20 = d * 1048576.0f;
    ds[0] = fmaf(d24, __uint_as_float(__byte_perm(scp, 0x4B000000u, 0x7540u)), -d24 * 8388608.0f);
    ds[1] = fmaf(d20, __uint_as_float(__byte_perm(scp, 0x4B000000u, 0x7541u)), -d20 * 8388608.0f);
    dm[0] = fmaf(dmin, __uint_as_float(__byte_perm(mnp, 0x4B000000u, 0x7540u)), -dmin * 8388608.0f);
    dm[1] = fmaf(dmin, __uint_as_float(__byte_perm(mnp, 0x4B000000u, 0x7541u)), -dmin * 8388608.0f);
}

// Unit u (256 values) of two rows (ra, rb: row starts, nullptr when past N) for Q4_K; the weight words are
// loaded once and serve each of the MT tokens (x of token m at xs + m * xstride, its sums at
// xsum + m * sstride).
template <int MT>
__device__ __forceinline__ void x16_q4k(const uint8_t *ra, const uint8_t *rb, int u, const uint8_t *xs,
                                        const float *xsum, int xstride, int sstride, const XLane &L,
                                        float acc[MT][2]) {
    const uint4 z4 = make_uint4(0u, 0u, 0u, 0u);
    const uint8_t *ba = ra ? ra + 144 * u : nullptr, *bb = rb ? rb + 144 * u : nullptr;
    const uint4 ha = ba ? ldg_nc_v4(ba) : z4, hb = bb ? ldg_nc_v4(bb) : z4;
    const uint4 wa0 = ba ? ldg_nc_v4(ba + 16 + 32 * L.t) : z4, wa1 = ba ? ldg_nc_v4(ba + 32 + 32 * L.t) : z4;
    const uint4 wb0 = bb ? ldg_nc_v4(bb + 16 + 32 * L.t) : z4, wb1 = bb ? ldg_nc_v4(bb + 32 + 32 * L.t) : z4;
    float ds[2][2], dm[2][2];
    x_q4k_scales(ha, L, ds[0], dm[0]);
    x_q4k_scales(hb, L, ds[1], dm[1]);
    const uint32_t A[8] = {wa0.x, wa0.y, wa0.z, wa0.w, wa1.x, wa1.y, wa1.z, wa1.w};
    const uint32_t B[8] = {wb0.x, wb0.y, wb0.z, wb0.w, wb1.x, wb1.y, wb1.z, wb1.w};
#pragma unroll 1
    for (int m = 0; m < MT; ++m) {
        // B: lo (hi) values of group t' = this lane's t for the lanes whose column takes them
        const uint8_t *xb = xs + m * xstride + 2 * (256 * u + 64 * L.t) + (L.b1on ? 64 : 0);
        uint32_t bx[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4 v = *reinterpret_cast<const uint4 *>(xb + 16 * i);
            bx[4 * i] = v.x;
            bx[4 * i + 1] = v.y;
            bx[4 * i + 2] = v.z;
            bx[4 * i + 3] = v.w;
        }
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f}, e[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            // bytes (4j, 4j + 1) then (4j + 2, 4j + 3): x pairs in natural order
            const uint32_t a01 = __byte_perm(A[j], 0u, 0x4140u), a23 = __byte_perm(A[j], 0u, 0x4342u);
            const uint32_t b01 = __byte_perm(B[j], 0u, 0x4140u), b23 = __byte_perm(B[j], 0u, 0x4342u);
            const uint32_t f0[4] = {a01 & 0x000F000Fu, b01 & 0x000F000Fu, a01 & 0x00F000F0u, b01 & 0x00F000F0u};
            const uint32_t f1[4] = {a23 & 0x000F000Fu, b23 & 0x000F000Fu, a23 & 0x00F000F0u, b23 & 0x00F000F0u};
            mma_f16_16816(d, f0, bx[2 * j] & L.b0on, bx[2 * j] & L.b1on);
            mma_f16_16816(e, f1, bx[2 * j + 1] & L.b0on, bx[2 * j + 1] & L.b1on);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) d[i] += e[i];
        const float2 xs2 = *reinterpret_cast<const float2 *>(xsum + m * sstride + 8 * u + 2 * L.t);
        acc[m][0] += fmaf(ds[0][0], d[0], fmaf(ds[0][1], d[1], -fmaf(dm[0][0], xs2.x, dm[0][1] * xs2.y)));
        acc[m][1] += fmaf(ds[1][0], d[2], fmaf(ds[1][1], d[3], -fmaf(dm[1][0], xs2.x, dm[1][1] * xs2.y)));
    }
}

// All 32-bit words one lane needs from a Q6_K block (at a 2-byte aligned
// address).  Lane t owns quarter c = t >> 1 and 16-value half lh = t & 1 of
// both 128-value halves s: ql words [s][j] at 64 s + 32 c + 16 lh + 4j (low
// nibbles: quarter c, high nibbles: quarter c + 2), qh words [s][j] at
// 128 + 32 s + 16 lh + 4j, the 16 int8 scales (sign-flipped) and d.
struct Q6Words {
    uint32_t ql[8], qh[8], sc[4];
    float d;
};

// Words [4 Q + (half ? 2 : 0), + 16) bytes of the 32 bytes w[0..7] (Q, half compile-time in the caller's switch).
template <int Q>
__device__ __forceinline__ void q6_pick4(const uint32_t w[8], bool half, uint32_t *out) {
#pragma unroll
    for (int i = 0; i < 4; ++i) out[i] = half ? __funnelshift_r(w[Q + i], w[Q + i + 1], 16) : w[Q + i];
}

__device__ __forceinline__ void q6_load(const uint8_t *b, int t, Q6Words &q) {
    if (b == nullptr) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            q.ql[i] = 0u;
            q.qh[i] = 0u;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) q.sc[i] = 0x80808080u;
        q.d = 0.0f;
        return;
    }
    // five 16-byte pieces (ql at lo_off and lo_off + 64, qh at hi_off and hi_off + 32, the scales at 192),
    // all at the block's offset sh within their aligned 16-byte windows: every window is loaded before
    // any word is taken apart.  A window holds at least one byte of the block, so it stays inside any
    // allocation of 16-byte granularity.
    const int lo_off = 32 * (t >> 1) + 16 * (t & 1), hi_off = 128 + 16 * (t & 1);
    const uintptr_t ab = reinterpret_cast<uintptr_t>(b);
    const int sh = static_cast<int>(ab & 15u);
    const uint8_t *base = reinterpret_cast<const uint8_t *>(ab - static_cast<uintptr_t>(sh));
    const int offs[5] = {lo_off, lo_off + 64, hi_off, hi_off + 32, 192};
    uint32_t w[5][8];
#pragma unroll
    for (int c = 0; c < 5; ++c) {
        const uint4 v0 = ldg_nc_v4(base + offs[c]);
        const uint4 v1 = sh ? ldg_nc_v4(base + offs[c] + 16) : make_uint4(0u, 0u, 0u, 0u);
        w[c][0] = v0.x;
        w[c][1] = v0.y;
        w[c][2] = v0.z;
        w[c][3] = v0.w;
        w[c][4] = v1.x;
        w[c][5] = v1.y;
        w[c][6] = v1.z;
        w[c][7] = v1.w;
    }
    const uint32_t dw = ldg_nc_u16(b + 208);
    uint32_t *dst[5] = {q.ql, q.ql + 4, q.qh, q.qh + 4, q.sc};
    const bool half = (sh & 2) != 0;
    switch (sh >> 2) {
        case 0:
#pragma unroll
            for (int c = 0; c < 5; ++c) q6_pick4<0>(w[c], half, dst[c]);
            break;
        case 1:
#pragma unroll
            for (int c = 0; c < 5; ++c) q6_pick4<1>(w[c], half, dst[c]);
            break;
        case 2:
#pragma unroll
            for (int c = 0; c < 5; ++c) q6_pick4<2>(w[c], half, dst[c]);
            break;
        default:
#pragma unroll
            for (int c = 0; c < 5; ++c) q6_pick4<3>(w[c], half, dst[c]);
            break;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) q.sc[i] ^= 0x80808080u;
    q.d = half_bits_to_float(dw);
}

// Byte t of a sign-flipped scale word times d, exact: (2^23 + 128 + sc) - (2^23 + 128) is exact in fp32,
// and so is d * sc.
__device__ __forceinline__ float q6_ds(uint32_t scx, uint32_t sel, float d) {
    return d * (__uint_as_float(__byte_perm(scx, 0x4B000000u, sel)) - 8388736.0f);
}

// Unit u (one 210-byte super-block) of two rows for Q6_K.  Per half s, lane t
// accumulates its two 16-value groups (quarter c = t >> 1 and c + 2, half
// lh = t & 1) over 8 mma and scales them once: groups 8s + t and 8s + t + 4.
template <int MT>
__device__ __forceinline__ void x16_q6k(const uint8_t *ra, const uint8_t *rb, int u, const uint8_t *xs, int xstride,
                                        const XLane &L, float acc[MT][2]) {
    Q6Words A, B;
    q6_load(ra ? ra + 210 * u : nullptr, L.t, A);
    q6_load(rb ? rb + 210 * u : nullptr, L.t, B);
    const uint32_t k1056 = 0x64206420u;  // fp16 1056 = 1024 + 32 in both halves
    const int c = L.t >> 1;
    const uint32_t shl = static_cast<uint32_t>(4 - 2 * c), shr = static_cast<uint32_t>(2 * c);
    const uint32_t sel = 0x7540u + static_cast<uint32_t>(L.t);
#pragma unroll 1
    for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        // x of this lane's group (quarter c) or of quarter c + 2 (64 values on) for the high-slot lanes
        const uint8_t *xb = xs + m * xstride + 2 * (256 * u + 128 * s + 32 * c + 16 * (L.t & 1)) + (L.b1on ? 128 : 0);
        const uint4 x0 = *reinterpret_cast<const uint4 *>(xb), x1 = *reinterpret_cast<const uint4 *>(xb + 16);
        const uint32_t bx[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float D[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t qla = A.ql[4 * s + j], qha = A.qh[4 * s + j];
            const uint32_t qlb = B.ql[4 * s + j], qhb = B.qh[4 * s + j];
            const uint32_t la = (qla & 0x0F0F0F0Fu) | ((qha << shl) & 0x30303030u);
            const uint32_t lb = (qlb & 0x0F0F0F0Fu) | ((qhb << shl) & 0x30303030u);
            const uint32_t ha = ((qla >> 4) & 0x0F0F0F0Fu) | ((qha >> shr) & 0x30303030u);
            const uint32_t hb = ((qlb >> 4) & 0x0F0F0F0Fu) | ((qhb >> shr) & 0x30303030u);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                const uint32_t ps = h2 ? 0x4342u : 0x4140u;
                const uint32_t a[4] = {hsub2_bits(__byte_perm(la, 0x64646464u, ps), k1056),
                                       hsub2_bits(__byte_perm(lb, 0x64646464u, ps), k1056),
                                       hsub2_bits(__byte_perm(ha, 0x64646464u, ps), k1056),
                                       hsub2_bits(__byte_perm(hb, 0x64646464u, ps), k1056)};
                const uint32_t b = bx[2 * j + h2];
                mma_f16_16816(D, a, b & L.b0on, b & L.b1on);
            }
        }
        acc[m][0] += fmaf(q6_ds(A.sc[2 * s], sel, A.d), D[0], q6_ds(A.sc[2 * s + 1], sel, A.d) * D[1]);
        acc[m][1] += fmaf(q6_ds(B.sc[2 * s], sel, B.d), D[2], q6_ds(B.sc[2 * s + 1], sel, B.d) * D[3]);
    }
}

// Unit u (8 blocks = 272 bytes, 256 values) of two rows for Q8_0: lane t takes blocks 2t and 2t + 1.
// int8 codes as exact fp16: 1024 + 128 + q by byte permutes, minus 1152 by one f16x2 subtract.
template <int MT>
__device__ __forceinline__ void x16_q80(const uint8_t *ra, const uint8_t *rb, int u, const uint8_t *xs, int xstride,
                                        const XLane &L, float acc[MT][2]) {
    const uint8_t *ba = ra ? ra + 272 * u + 68 * L.t : nullptr, *bb = rb ? rb + 272 * u + 68 * L.t : nullptr;
    uint32_t wa[17], wb[17];
#pragma unroll
    for (int i = 0; i < 17; ++i) {
        wa[i] = ba ? ldg32(ba + 4 * i) : 0u;
        wb[i] = bb ? ldg32(bb + 4 * i) : 0u;
    }
    // block 2t: d = bytes 0-1, q = bytes 2..33; block 2t + 1: d = bytes 34-35, q = bytes 36..67
    const float da0 = half_bits_to_float(wa[0]), da1 = half_bits_to_float(wa[8] >> 16);
    const float db0 = half_bits_to_float(wb[0]), db1 = half_bits_to_float(wb[8] >> 16);
    const uint32_t k1152 = 0x64806480u;  // fp16 1152 = 1024 + 128
#pragma unroll 1
    for (int m = 0; m < MT; ++m) {
    const uint8_t *xb = xs + m * xstride + 2 * (256 * u + 64 * L.t) + (L.b1on ? 64 : 0);
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f}, e[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t qa0 = __funnelshift_r(wa[j], wa[j + 1], 16) ^ 0x80808080u;  // block 2t, values 4j..4j+3
        const uint32_t qb0 = __funnelshift_r(wb[j], wb[j + 1], 16) ^ 0x80808080u;
        const uint32_t qa1 = wa[9 + j] ^ 0x80808080u;  // block 2t + 1
        const uint32_t qb1 = wb[9 + j] ^ 0x80808080u;
        const uint2 xv = *reinterpret_cast<const uint2 *>(xb + 8 * j);
        const uint32_t f0[4] = {hsub2_bits(__byte_perm(qa0, 0x64646464u, 0x4140u), k1152),
                                hsub2_bits(__byte_perm(qb0, 0x64646464u, 0x4140u), k1152),
                                hsub2_bits(__byte_perm(qa1, 0x64646464u, 0x4140u), k1152),
                                hsub2_bits(__byte_perm(qb1, 0x64646464u, 0x4140u), k1152)};
        const uint32_t f1[4] = {hsub2_bits(__byte_perm(qa0, 0x64646464u, 0x4342u), k1152),
                                hsub2_bits(__byte_perm(qb0, 0x64646464u, 0x4342u), k1152),
                                hsub2_bits(__byte_perm(qa1, 0x64646464u, 0x4342u), k1152),
                                hsub2_bits(__byte_perm(qb1, 0x64646464u, 0x4342u), k1152)};
        mma_f16_16816(d, f0, xv.x & L.b0on, xv.x & L.b1on);
        mma_f16_16816(e, f1, xv.y & L.b0on, xv.y & L.b1on);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] += e[i];
    acc[m][0] += fmaf(da0, d[0], da1 * d[1]);
    acc[m][1] += fmaf(db0, d[2], db1 * d[3]);
    }
}

template <int MT>
__device__ __forceinline__ void x16_unit(int fmt, const uint8_t *ra, const uint8_t *rb, int u, const uint8_t *xs,
                                         const float *xsum, int K, const XLane &L, float acc[MT][2]) {
    if (fmt == T2C_Q4_K) {
        x16_q4k<MT>(ra, rb, u, xs, xsum, 2 * K, K >> 5, L, acc);
    } else if (fmt == T2C_Q6_K) {
        x16_q6k<MT>(ra, rb, u, xs, 2 * K, L, acc);
    } else {
        x16_q80<MT>(ra, rb, u, xs, 2 * K, L, acc);
    }
}

template <int MT>
__global__ void __launch_bounds__(kXThreads, 2) qmv_x16_kernel(const __grid_constant__ QParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int K = p.K;
    uint8_t *xs = smem;                                          // [MT][K] fp16
    float *xsum = reinterpret_cast<float *>(smem + MT * 2 * K);  // [MT][K / 32]
    float *red = xsum + MT * (K >> 5);                           // [MT][warps]
    float *part = red + MT * kXWarps;                            // [warp][token][gate/up][16 rows]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const XLane L = x_lane(lane);
    pdl_wait();
    pdl_trigger();
    x16_prepare<MT>(p, xs, xsum, red);
    const bool swiglu = p.mode == MODE_SWIGLU;
    const int wpb = p.wpb, bpc = kXWarps / wpb;
    const int grp = warp / wpb, wig = warp - grp * wpb;
    const int units = K >> 8;
    for (int64_t base = static_cast<int64_t>(blockIdx.x) * bpc; base < p.total_rowsets;
         base += static_cast<int64_t>(gridDim.x) * bpc) {
        const int64_t tile = base + grp;
        float acc[MT][2][2];
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m][0][0] = acc[m][0][1] = acc[m][1][0] = acc[m][1][1] = 0.0f;
        if (tile < p.total_rowsets) {
            const int si = swiglu ? 0 : stream_of(p, tile);
            const int64_t row0 = (tile - p.s[si].rs_begin) * kMmaRows;
#pragma unroll 1
            for (int wi = 0; wi < (swiglu ? 2 : 1); ++wi) {
                const QStream &st = p.s[swiglu ? wi : si];
                const int64_t na = row0 + L.g, nb = row0 + L.g + 8;
                const uint8_t *ra = na < st.n ? st.w + na * st.row_bytes : nullptr;
                const uint8_t *rb = nb < st.n ? st.w + nb * st.row_bytes : nullptr;
                float a2[MT][2];
#pragma unroll
                for (int m = 0; m < MT; ++m) a2[m][0] = a2[m][1] = 0.0f;
#pragma unroll 1
                for (int u = wig; u < units; u += wpb) x16_unit<MT>(st.fmt, ra, rb, u, xs, xsum, K, L, a2);
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    acc[m][wi][0] = a2[m][0];
                    acc[m][wi][1] = a2[m][1];
                }
            }
#pragma unroll
            for (int m = 0; m < MT; ++m)
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        acc[m][r][h] += __shfl_xor_sync(0xffffffffu, acc[m][r][h], 1);
                        acc[m][r][h] += __shfl_xor_sync(0xffffffffu, acc[m][r][h], 2);
                    }
        }
        if (wpb > 1) {
            if (L.t == 0) {
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        part[((warp * MT + m) * 2 + r) * 16 + L.g] = acc[m][r][0];
                        part[((warp * MT + m) * 2 + r) * 16 + L.g + 8] = acc[m][r][1];
                    }
            }
            __syncthreads();
            if (wig == 0) {
#pragma unroll
                for (int m = 0; m < MT; ++m)
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        float v0 = 0.0f, v1 = 0.0f;
                        for (int w = warp; w < warp + wpb; ++w) {
                            v0 += part[((w * MT + m) * 2 + r) * 16 + L.g];
                            v1 += part[((w * MT + m) * 2 + r) * 16 + L.g + 8];
                        }
                        acc[m][r][0] = v0;
                        acc[m][r][1] = v1;
                    }
            }
            __syncthreads();
        }
        if (wig == 0 && tile < p.total_rowsets) {
            // every lane of a quad holds all tokens' sums; lane t stores token t (the dense layout the
            // epilogue expects)
            float v[2][2] = {{acc[0][0][0], acc[0][0][1]}, {acc[0][1][0], acc[0][1][1]}};
#pragma unroll
            for (int m = 1; m < MT; ++m)
                if (L.t == m) {
                    v[0][0] = acc[m][0][0];
                    v[0][1] = acc[m][0][1];
                    v[1][0] = acc[m][1][0];
                    v[1][1] = acc[m][1][1];
                }
            mma_finish_block<MT>(p, tile, v, lane);
        }
    }
}

// ================================================================== launchers
size_t x_smem_bytes(int MT, int K) {
    return static_cast<size_t>(MT) * (K / 64) * 16 + static_cast<size_t>(MT) * padded_k(K) * 2 +
           static_cast<size_t>(MT) * (K / 32) * 4 + static_cast<size_t>(MT) * (K / 16) * 4 +
           static_cast<size_t>(kConsumerWarps) * 8 * 4;
}

constexpr size_t kSmemLimit = 220 * 1024;

int pick_mt(int64_t M, int K) {
    const size_t budget = 96 * 1024;
    int mt = 8;
    while (mt > 1 && (mt / 2 >= M || x_smem_bytes(mt, K) > budget)) mt /= 2;
    return mt;
}

template <typename Kernel>
int ensure_smem_attr(Kernel kernel, bool &configured_flag) {
    if (!configured_flag) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)) !=
            cudaSuccess) {
            return set_error(T2C_ECUDA, "qmv: cudaFuncSetAttribute failed");
        }
        configured_flag = true;
    }
    return T2C_OK;
}

int device_slot() {
    int device = 0;
    cudaGetDevice(&device);
    return device < 0 ? 0 : (device > 63 ? 63 : device);
}

template <typename Kernel>
int launch_pdl(Kernel kernel, int blocks, int threads, size_t smem, cudaStream_t stream, const QParams &p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, p);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "qmv launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

template <int MT, int FMT>
int launch_direct(QParams p, cudaStream_t stream) {
    static bool configured[64] = {false};
    const size_t smem = x_smem_bytes(MT, p.K);
    int rc = ensure_smem_attr(qmv_direct_kernel<MT, FMT>, configured[device_slot()]);
    if (rc) return rc;
    const int subs_per_block = kWarps * (32 / p.lpr);
    int64_t blocks = (p.total_rowsets + subs_per_block - 1) / subs_per_block;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qmv_direct_kernel<MT, FMT>, kThreads, smem) !=
            cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    const int64_t max_blocks = static_cast<int64_t>(sm_count()) * per_sm;
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    return launch_pdl(qmv_direct_kernel<MT, FMT>, static_cast<int>(blocks), kThreads, smem, stream, p);
}

int tma_stages(int mt, const QParams &p);

template <int MT, int FMT>
int launch_tma(QParams p, cudaStream_t stream) {
    static bool configured[64] = {false};
    p.stages = tma_stages(MT, p);
    if (p.stages < 2) return set_error(T2C_EUNSUPPORTED, "qmv: stage of %d bytes does not fit", p.stage_bytes);
    const size_t smem =
        kStageHead + static_cast<size_t>(kWarps) * p.stages * p.stage_bytes + x_smem_bytes(MT, p.K);
    int rc = ensure_smem_attr(qmv_tma_kernel<MT, FMT>, configured[device_slot()]);
    if (rc) return rc;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qmv_tma_kernel<MT, FMT>, kConsumerThreads, smem) !=
            cudaSuccess ||
        per_sm < 1) {
        per_sm = 1;
    }
    int64_t blocks = (p.total_rowsets + kWarps - 1) / kWarps;
    const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
    if (blocks > cap) blocks = cap;
    return launch_pdl(qmv_tma_kernel<MT, FMT>, static_cast<int>(blocks), kConsumerThreads, smem, stream, p);
}

template <int FMT>
int launch_fmt_mt(const QParams &c, int mt, bool tma, cudaStream_t stream) {
    if (tma) {
        switch (mt) {
            case 1: return launch_tma<1, FMT>(c, stream);
            case 2: return launch_tma<2, FMT>(c, stream);
            case 4: return launch_tma<4, FMT>(c, stream);
            default: return launch_tma<8, FMT>(c, stream);
        }
    }
    switch (mt) {
        case 1: return launch_direct<1, FMT>(c, stream);
        case 2: return launch_direct<2, FMT>(c, stream);
        case 4: return launch_direct<4, FMT>(c, stream);
        default: return launch_direct<8, FMT>(c, stream);
    }
}

int launch_fmt(const QParams &c, int mt, bool tma, cudaStream_t stream) {
    int fmt = c.s[0].fmt;
    for (int i = 1; i < c.nstreams; ++i)
        if (c.s[i].fmt != fmt) fmt = 0;
    switch (fmt) {
        case T2C_Q4_K: return launch_fmt_mt<T2C_Q4_K>(c, mt, tma, stream);
        case T2C_Q6_K: return launch_fmt_mt<T2C_Q6_K>(c, mt, tma, stream);
        case T2C_Q8_0: return launch_fmt_mt<T2C_Q8_0>(c, mt, tma, stream);
        default: return launch_fmt_mt<0>(c, mt, tma, stream);
    }
}

// Ring depth per warp of the streamed kernel: about kStreamBytesPerSm of
// weights in flight per SM, spread over the CTAs that fit (>= 2 buffers per
// warp, 0 when nothing fits).
constexpr size_t kSmPerSmem = 227 * 1024;
constexpr size_t kStreamBytesPerSm = 160 * 1024;

int tma_stages(int mt, const QParams &p) {
    const size_t xbytes = x_smem_bytes(mt, p.K);
    const size_t stage = static_cast<size_t>(p.stage_bytes);
    for (int ctas = 4; ctas >= 1; --ctas) {
        int stages = static_cast<int>(kStreamBytesPerSm / ctas / (kWarps * stage));
        if (stages < 2) stages = 2;
        if (stages > kMaxStages) stages = kMaxStages;
        const size_t per_cta = kStageHead + kWarps * stages * stage + xbytes + 1024;
        if (per_cta * ctas <= kSmPerSmem && per_cta <= kSmemLimit) return stages;
    }
    return 0;
}

int launch_chunked(QParams p, int64_t M, bool tma, cudaStream_t stream) {
    const int mt = pick_mt(M, p.K);
    const int64_t K = p.K;
    for (int64_t m0 = 0; m0 < M; m0 += mt) {
        QParams c = p;
        c.M = static_cast<int>((M - m0) < mt ? (M - m0) : mt);
        c.x = p.x + m0 * K;
        for (int i = 0; i < p.nstreams; ++i) {
            if (c.s[i].y) c.s[i].y = p.s[i].y + m0 * p.s[i].n;
            if (c.s[i].res) c.s[i].res = p.s[i].res + m0 * p.s[i].n;
        }
        if (p.mode == MODE_ARGMAX) {
            c.ps = p.ps + m0 * p.G;
            c.pt = p.pt + m0 * p.G;
        }
        int rc = launch_fmt(c, mt, tma, stream);
        if (rc != T2C_OK) return rc;
    }
    return T2C_OK;
}

int validate_common(int64_t M, int64_t K, const void *x) {
    if (x == nullptr) return set_error(T2C_EINVAL, "x is NULL");
    if (M <= 0 || K <= 0) return set_error(T2C_EINVAL, "M=%lld K=%lld must be positive", (long long)M, (long long)K);
    if (K % 64 != 0) return set_error(T2C_EINVAL, "K=%lld must be a multiple of 64", (long long)K);
    if (K > 65536) return set_error(T2C_EUNSUPPORTED, "K=%lld above 65536", (long long)K);
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) return set_error(T2C_EINVAL, "x must be 16-byte aligned");
    return T2C_OK;
}

int validate_weight(int wtype, const void *w, int64_t K) {
    if (w == nullptr) return set_error(T2C_EINVAL, "weight is NULL");
    if (wtype == T2C_Q4_K) {
        if (K % 256) return set_error(T2C_EINVAL, "Q4_K needs K %% 256 == 0, got %lld", (long long)K);
        if (reinterpret_cast<uintptr_t>(w) % 16) return set_error(T2C_EINVAL, "Q4_K weight must be 16-byte aligned");
    } else if (wtype == T2C_Q6_K) {
        if (K % 256) return set_error(T2C_EINVAL, "Q6_K needs K %% 256 == 0, got %lld", (long long)K);
        if (reinterpret_cast<uintptr_t>(w) % 4) return set_error(T2C_EINVAL, "Q6_K weight must be 4-byte aligned");
    } else if (wtype == T2C_Q8_0) {
        if (K % 64) return set_error(T2C_EUNSUPPORTED, "Q8_0 kernel needs K %% 64 == 0, got %lld", (long long)K);
        if (reinterpret_cast<uintptr_t>(w) % 4) return set_error(T2C_EINVAL, "Q8_0 weight must be 4-byte aligned");
    } else {
        return set_error(T2C_EUNSUPPORTED, "weight type %d not supported", wtype);
    }
    return T2C_OK;
}

int lanes_for(int units) {
    int lpr = 32;
    while (lpr > 4 && lpr > units) lpr >>= 1;
    return lpr;
}

// Streamed geometry of one stream, or false when it cannot be bulk-copied
// (every copy must start 16-byte aligned and move a multiple of 16 bytes).
// Rows per row block: 4 consumer warps x (32 / lpr) groups x 4 rows.
bool tma_geometry(QStream &st, int64_t K, bool swiglu) {
    if (reinterpret_cast<uintptr_t>(st.w) % 16) return false;
    const int block_values = st.fmt == T2C_Q8_0 ? 32 : 256;
    const int block_bytes = st.fmt == T2C_Q4_K ? 144 : (st.fmt == T2C_Q6_K ? 210 : 34);
    const int nb = static_cast<int>(K / block_values);
    int seg_blocks = st.fmt == T2C_Q8_0 ? 32 : 8;
    if (seg_blocks > nb) seg_blocks = nb;
    while (nb % seg_blocks) --seg_blocks;
    const bool seg_ok = (st.row_bytes % 16 == 0) && ((seg_blocks * block_bytes) % 16 == 0) &&
                        (st.fmt != T2C_Q8_0 || seg_blocks % 2 == 0);
    if (seg_ok) {
        st.whole = 0;
        st.seg_blocks = seg_blocks;
        st.seg_bytes = seg_blocks * block_bytes;
        st.chunks = nb / seg_blocks;
    } else {
        if (swiglu) return false;
        if (st.fmt == T2C_Q8_0 && nb % 2) return false;
        st.whole = 1;
        st.seg_blocks = nb;
        st.seg_bytes = static_cast<int>(st.row_bytes);
        st.chunks = 1;
    }
    const int units = st.fmt == T2C_Q8_0 ? st.seg_blocks / 2 : st.seg_blocks * 4;
    st.lpr = lanes_for(units);
    if (st.lpr < 8) return false;
    st.rb = (32 / st.lpr) * kNR;
    if (st.whole && ((st.rb * st.row_bytes) % 16 != 0 || st.n % st.rb != 0)) return false;
    return true;
}

// Chooses the streamed kernel when every stream can be bulk-copied.
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
int encode_weight_map(CUtensorMap *map, const uint8_t *w, int64_t n, int64_t row_bytes) {
    static PFN_cuTensorMapEncodeTiled encode = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
    }();
    if (encode == nullptr || row_bytes % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0) return T2C_EUNSUPPORTED;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 4), static_cast<cuuint64_t>(n)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {kMmaSegBytes / 4, kMmaRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? T2C_OK : T2C_EUNSUPPORTED;
}

size_t mma_fixed_smem(int MT, int K) {
    return kStageHead + kMmaSlots * kMmaWarps * sizeof(MmaSlot) + static_cast<size_t>(MT) * xf_row_bytes(K) +
           static_cast<size_t>(MT) * (K / 256) * 32 + static_cast<size_t>(kMmaWarps) * MT * 4;
}

template <int MT>
int launch_mma(QParams p, cudaStream_t stream) {
    static bool configured[64] = {false};
    const size_t fixed = mma_fixed_smem(MT, p.K);
    const size_t per_stage = static_cast<size_t>(kMmaWarps) * p.stage_bytes;
    p.stages = fixed >= kSmemLimit ? 0 : static_cast<int>((kSmemLimit - fixed) / per_stage);
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    if (p.stages < 2) return set_error(T2C_EUNSUPPORTED, "qmv_mma: stages do not fit");
    const size_t smem = fixed + per_stage * p.stages;
    int rc = ensure_smem_attr(qmv_mma_kernel<MT>, configured[device_slot()]);
    if (rc) return rc;
    // the same number of CTA iterations for every CTA
    const int64_t groups = (p.total_rowsets + p.bpc - 1) / p.bpc;
    const int64_t iters = (groups + sm_count() - 1) / sm_count();
    const int64_t blocks = (groups + iters - 1) / iters;
    return launch_pdl(qmv_mma_kernel<MT>, static_cast<int>(blocks), kMmaThreads, smem, stream, p);
}

int launch_m1(QParams p, cudaStream_t stream) {
    static bool configured[64] = {false};
    p.xseg_per_warp = (p.nseg + p.wpb - 1) / p.wpb;
    if (p.xseg_per_warp > kM1MaxSegs) return set_error(T2C_EUNSUPPORTED, "qmv_m1: K too large");
    const size_t fixed = kStageHead + static_cast<size_t>(kMmaWarps) * p.xseg_per_warp * kM1SegBytes +
                         static_cast<size_t>(kMmaSlots) * p.bpc * sizeof(M1Slot) + kMmaWarps * sizeof(float);
    const size_t per_stage = static_cast<size_t>(kMmaWarps) * p.stage_bytes;
    // two CTAs per SM when two stages per warp fit in half of the shared memory, else one CTA with more stages
    const size_t half = 113 * 1024;
    int per_sm = 1;
    if (fixed + 2 * per_stage <= half) {
        per_sm = 2;
        p.stages = static_cast<int>((half - fixed) / per_stage);
    } else {
        p.stages = fixed >= kSmemLimit ? 0 : static_cast<int>((kSmemLimit - fixed) / per_stage);
    }
    if (p.stages > kMaxStages) p.stages = kMaxStages;
    if (p.stages < 2) return set_error(T2C_EUNSUPPORTED, "qmv_m1: stages do not fit");
    const size_t smem = fixed + per_stage * p.stages;
    int rc = ensure_smem_attr(qmv_m1_kernel, configured[device_slot()]);
    if (rc) return rc;
    int64_t blocks = (p.total_rowsets + p.bpc - 1) / p.bpc;
    if (blocks > static_cast<int64_t>(sm_count()) * per_sm) blocks = static_cast<int64_t>(sm_count()) * per_sm;
    // the fused tensor-parallel reduction waits on the peers' CTA of the same index: every CTA resident
    if (p.ar_tp > 1 && blocks > kArMaxCtas) return set_error(T2C_EUNSUPPORTED, "qmv_m1: too many CTAs to reduce");
    return launch_pdl(qmv_m1_kernel, static_cast<int>(blocks), kMmaThreads, smem, stream, p);
}


// Tensor-core path when every stream is Q4_K, M <= 4 and K splits into 512-value segments.
int try_mma(QParams p, int64_t M, cudaStream_t stream, bool &used) {
    used = false;
    if (M > 4 || p.K % (kMmaSegBlocks * 256) != 0) return T2C_OK;
    for (int i = 0; i < p.nstreams; ++i)
        if (p.s[i].fmt != T2C_Q4_K) return T2C_OK;
    const bool swiglu = p.mode == MODE_SWIGLU;
    // K above 8192: the 2..4-token kernel's x planes over all of K leave too little shared memory
    // for weight stages, so each token takes its own pass of the M = 1 kernel instead
    const bool per_token = M > 1 && p.K > 8192;
    const int MT = (M <= 1 || per_token) ? 1 : (M <= 2 ? 2 : 4);
    p.stage_bytes = kMmaRows * kMmaSegBytes;
    if (mma_fixed_smem(MT, p.K) + 2 * static_cast<size_t>(kMmaWarps) * p.stage_bytes > kSmemLimit) return T2C_OK;
    p.nseg = p.K / (kMmaSegBlocks * 256);
    p.wpb = 1;
    while (p.wpb * 2 <= kMmaWarps && p.wpb * 2 <= p.nseg) p.wpb *= 2;
    p.bpc = kMmaWarps / p.wpb;
    int64_t blocks = 0;
    for (int i = 0; i < p.nstreams; ++i) {
        p.s[i].rs_begin = blocks;
        blocks += (p.s[i].n + kMmaRows - 1) / kMmaRows;
        if (swiglu) break;
    }
    if (swiglu) p.s[1].rs_begin = blocks;
    p.total_rowsets = blocks;
    p.M = static_cast<int>(M);
    for (int i = 0; i < (swiglu ? 2 : p.nstreams); ++i) {
        if (p.s[i].n > INT32_MAX || encode_weight_map(&p.tmap[i], p.s[i].w, p.s[i].n, p.s[i].row_bytes) != T2C_OK)
            return T2C_OK;  // no map: the dp4a kernels serve this call
    }
    used = true;
    if (per_token) {
        for (int64_t t = 0; t < M; ++t) {
            QParams q = p;
            q.M = 1;
            q.x = p.x + t * p.K;
            for (int i = 0; i < kMaxStreams; ++i) {
                if (q.s[i].y != nullptr) q.s[i].y += t * q.s[i].n;
                if (q.s[i].res != nullptr) q.s[i].res += t * q.s[i].n;
            }
            const int rc = launch_m1(q, stream);
            if (rc) return rc;
        }
        return T2C_OK;
    }
    switch (MT) {
        case 1: return launch_m1(p, stream);
        case 2: return launch_mma<2>(p, stream);
        default: return launch_mma<4>(p, stream);
    }
}

bool batched_kernel_serves(int64_t M, int64_t K) { return M > 4 && M <= 16 && (K <= 8192 || M <= 8); }

// M > 4, Q4_K / Q6_K / Q8_0 streams, no fused RMSNorm: tcgen05 GEMM (fused QKV in one launch when the
// formats agree, else one launch per weight).
int try_gemm(const QParams &p, int64_t M, cudaStream_t stream, bool &used) {
    used = false;
    if (M <= 4) return T2C_OK;
    const int fmt = p.s[0].fmt;
    // Q4_K at 5..16 tokens with K <= 8192, or 5..8 tokens at any K: the batched exact kernel (fused
    // RMSNorm allowed).  Beyond that the tcgen05 GEMM measured faster (per launch from 16 tokens at
    // K = 12288, where the x slices leave room for only two weight stages per warp; over a whole
    // batch-32 decode step at 32 tokens).
    if (batched_kernel_serves(M, p.K) && p.mode != MODE_ARGMAX) {
        bool all_q4k = true;
        for (int i = 0; i < (p.mode == MODE_SWIGLU ? 2 : p.nstreams); ++i) all_q4k = all_q4k && p.s[i].fmt == T2C_Q4_K;
        if (all_q4k) {
            QGemmArgs b = {};
            b.fmt = T2C_Q4_K;
            b.K = p.K;
            b.M = M;
            b.x = p.x;
            if (p.mode == MODE_SWIGLU) {
                b.nw = 1;
                b.w[0] = p.s[0].w;
                b.w_up = p.s[1].w;
                b.N[0] = p.s[0].n;
                b.y[0] = p.s[0].y;
            } else {
                b.nw = p.nstreams;
                for (int i = 0; i < p.nstreams; ++i) {
                    b.w[i] = p.s[i].w;
                    b.N[i] = p.s[i].n;
                    b.y[i] = p.s[i].y;
                    b.res[i] = p.s[i].res;
                }
            }
            const int rc = qbatch(b, p.norm_w, p.eps, stream);
            if (rc != T2C_EUNSUPPORTED) {
                used = true;
                return rc;
            }
        }
    }
    if (p.norm_w != nullptr) return T2C_OK;
    if (fmt != T2C_Q4_K && fmt != T2C_Q6_K && fmt != T2C_Q8_0) return T2C_OK;
    bool same = true;
    for (int i = 1; i < (p.mode == MODE_SWIGLU ? 2 : p.nstreams); ++i) same = same && p.s[i].fmt == fmt;
    QGemmArgs a = {};
    a.fmt = fmt;
    a.K = p.K;
    a.M = M;
    a.x = p.x;
    if (p.mode == MODE_SWIGLU) {
        if (!same) return T2C_OK;
        a.nw = 1;
        a.w[0] = p.s[0].w;
        a.w_up = p.s[1].w;
        a.N[0] = p.s[0].n;
        a.y[0] = p.s[0].y;
    } else if (p.mode == MODE_ARGMAX) {
        a.nw = 1;
        a.w[0] = p.s[0].w;
        a.N[0] = p.s[0].n;
        a.ps = p.ps;
        a.pt = p.pt;
        a.G = p.G;
    } else if (same) {
        // all weights of a fused QKV in one launch
        a.nw = p.nstreams;
        for (int i = 0; i < p.nstreams; ++i) {
            a.w[i] = p.s[i].w;
            a.N[i] = p.s[i].n;
            a.y[i] = p.s[i].y;
            a.res[i] = p.s[i].res;
        }
    } else {
        // mixed formats (Q4_K_M: Q6_K v): one launch per weight, all or nothing
        for (int i = 0; i < p.nstreams; ++i) {
            const int fi = p.s[i].fmt;
            const bool ok_fmt = fi == T2C_Q4_K || fi == T2C_Q8_0 || (fi == T2C_Q6_K && (p.K % 2048 == 0 || p.s[i].n % 8 == 0));
            if (!ok_fmt || reinterpret_cast<uintptr_t>(p.s[i].w) % 16) return T2C_OK;
        }
        for (int i = 0; i < p.nstreams; ++i) {
            QGemmArgs one = a;
            one.fmt = p.s[i].fmt;
            one.nw = 1;
            one.w[0] = p.s[i].w;
            one.N[0] = p.s[i].n;
            one.y[0] = p.s[i].y;
            one.res[0] = p.s[i].res;
            const int rc = qgemm(one, stream);
            if (rc == T2C_EUNSUPPORTED && i == 0) return T2C_OK;
            if (rc != T2C_OK) return rc == T2C_EUNSUPPORTED ? set_error(T2C_EUNSUPPORTED, "qgemm: weight %d", i) : rc;
        }
        used = true;
        return T2C_OK;
    }
    const int rc = qgemm(a, stream);
    if (rc == T2C_EUNSUPPORTED) return T2C_OK;  // nothing launched: the matvec kernels serve this call
    used = true;
    return rc;
}

// Exact fp16-x kernel, one launch per token (any GGUF type, K % 256 == 0).
size_t x16_smem_bytes(int MT, int K) {
    return static_cast<size_t>(MT) * (2 * static_cast<size_t>(K) + static_cast<size_t>(K / 32) * 4) +
           static_cast<size_t>(MT) * kXWarps * 4 + static_cast<size_t>(kXWarps) * MT * 2 * 16 * 4;
}

template <int MT>
int launch_x16_mt(const QParams &p, int64_t tiles, cudaStream_t stream) {
    static bool configured[64] = {false};
    const size_t smem = x16_smem_bytes(MT, p.K);
    int rc = ensure_smem_attr(qmv_x16_kernel<MT>, configured[device_slot()]);
    if (rc) return rc;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qmv_x16_kernel<MT>, kXThreads, smem) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    const int bpc = kXWarps / p.wpb;
    int64_t blocks = (tiles + bpc - 1) / bpc;
    const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm;
    if (blocks > cap) blocks = cap;
    return launch_pdl(qmv_x16_kernel<MT>, static_cast<int>(blocks), kXThreads, smem, stream, p);
}

// Up to 4 tokens per pass (weights read once for all of them); more tokens take passes of 4.
int launch_x16(QParams p, int64_t M, cudaStream_t stream) {
    const bool swiglu = p.mode == MODE_SWIGLU;
    int64_t tiles = 0;
    for (int i = 0; i < p.nstreams; ++i) {
        p.s[i].rs_begin = tiles;
        tiles += (p.s[i].n + kMmaRows - 1) / kMmaRows;
        if (swiglu) break;  // gate and up rows form one set of tiles
    }
    if (swiglu) p.s[1].rs_begin = tiles;  // never selected
    p.total_rowsets = tiles;
    const int units = p.K / 256;
    // warps per tile (split K): enough warps in flight for the whole GPU, at most one unit each
    const int64_t want = static_cast<int64_t>(sm_count()) * 2 * kXWarps;
    int wpb = 1;
    while (wpb < kXWarps && tiles * wpb < want && wpb * 2 <= units) wpb *= 2;
    p.wpb = wpb;
    int cap = 4;
    while (cap > 1 && x16_smem_bytes(cap, p.K) > kSmemLimit) cap /= 2;
    if (x16_smem_bytes(cap, p.K) > kSmemLimit) return set_error(T2C_EUNSUPPORTED, "qmv_x16: K too large");
    for (int64_t t0 = 0; t0 < M; t0 += cap) {
        const int mt = static_cast<int>(M - t0 < cap ? M - t0 : cap);
        QParams q = p;
        q.M = mt;
        q.x = p.x + t0 * p.K;
        for (int i = 0; i < kMaxStreams; ++i) {
            if (q.s[i].y != nullptr) q.s[i].y += t0 * q.s[i].n;
            if (q.s[i].res != nullptr) q.s[i].res += t0 * q.s[i].n;
        }
        if (p.mode == MODE_ARGMAX) {
            q.ps = p.ps + t0 * p.G;
            q.pt = p.pt + t0 * p.G;
        }
        const int rc = mt == 1 ? launch_x16_mt<1>(q, tiles, stream)
                       : mt == 2 ? launch_x16_mt<2>(q, tiles, stream)
                                 : launch_x16_mt<4>(q, tiles, stream);
        if (rc) return rc;
    }
    return T2C_OK;
}

int run_linear(QParams p, int64_t M, cudaStream_t stream) {
    bool used = false;
    const int rc_gemm = try_gemm(p, M, stream, used);
    if (used) return rc_gemm;
    const int rc_mma = try_mma(p, M, stream, used);
    if (used) return rc_mma;
    if (M <= 4 && p.K % 256 == 0) return launch_x16(p, M, stream);
    bool tma = true;
    const bool swiglu = p.mode == MODE_SWIGLU;
    int stage_bytes = 0;
    for (int i = 0; i < p.nstreams && tma; ++i) {
        QStream &st = p.s[i];
        if (!tma_geometry(st, p.K, swiglu)) {
            tma = false;
            break;
        }
        const int bytes = st.rb * st.seg_bytes;
        if (bytes > stage_bytes) stage_bytes = bytes;
    }
    if (tma) {
        p.stage_bytes = stage_bytes;
        if (tma_stages(pick_mt(M, p.K), p) < 2) tma = false;
    }
    if (tma) {
        int64_t blocks = 0;
        for (int i = 0; i < p.nstreams; ++i) {
            QStream &st = p.s[i];
            st.rs_begin = blocks;
            const int64_t rows_per_block = swiglu ? st.rb / 2 : st.rb;
            blocks += (st.n + rows_per_block - 1) / rows_per_block;
            if (swiglu) break;  // gate and up form one stream of outputs
        }
        if (swiglu) p.s[1].rs_begin = blocks;  // never selected
        p.total_rowsets = blocks;
        p.stage_bytes = stage_bytes;
        return launch_chunked(p, M, true, stream);
    }
    // direct kernel: row-sets of 2 rows (ROWS, ARGMAX) or 1 output (SWIGLU)
    p.units = p.K / 64;
    p.lpr = lanes_for(p.units);
    if (p.mode == MODE_ARGMAX && p.lpr > 16) p.lpr = 16;  // row-set pairs share a warp
    int64_t rs = 0;
    for (int i = 0; i < p.nstreams; ++i) {
        p.s[i].rs_begin = rs;
        rs += swiglu ? p.s[i].n : (p.s[i].n + kDirectRows - 1) / kDirectRows;
        if (swiglu) break;
    }
    if (swiglu) p.s[1].rs_begin = rs;
    p.total_rowsets = rs;
    return launch_chunked(p, M, false, stream);
}

}  // namespace

cudaError_t status_qlinear(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c

using namespace t2c;

extern "C" int t2c_linear_multi(int count, const int *wtypes, const void *const *ws, void *const *ys,
                                const void *const *residuals, const int64_t *Ns, const void *x,
                                const float *norm_weight, float eps, int64_t M, int64_t K, void *stream) {
    if (count < 1 || count > kMaxStreams) return set_error(T2C_EINVAL, "count=%d must be 1..3", count);
    int rc = validate_common(M, K, x);
    if (rc) return rc;
    QParams p = {};
    p.nstreams = count;
    p.mode = MODE_ROWS;
    p.x = static_cast<const __half *>(x);
    p.norm_w = norm_weight;
    p.eps = eps;
    p.K = static_cast<int>(K);
    for (int i = 0; i < count; ++i) {
        if ((rc = validate_weight(wtypes[i], ws[i], K))) return rc;
        if (ys[i] == nullptr || Ns[i] <= 0) return set_error(T2C_EINVAL, "stream %d: bad output or N", i);
        p.s[i].w = static_cast<const uint8_t *>(ws[i]);
        p.s[i].y = static_cast<__half *>(ys[i]);
        p.s[i].res = residuals ? static_cast<const __half *>(residuals[i]) : nullptr;
        p.s[i].n = Ns[i];
        p.s[i].row_bytes = row_bytes(wtypes[i], K);
        p.s[i].fmt = wtypes[i];
    }
    return run_linear(p, M, as_stream(stream));
}

extern "C" int t2c_linear(int wtype, const void *x, const void *w, const void *residual, void *y, int64_t M,
                          int64_t N, int64_t K, void *stream) {
    const int types[1] = {wtype};
    const void *wp[1] = {w};
    void *yp[1] = {y};
    const void *rp[1] = {residual};
    const int64_t np[1] = {N};
    return t2c_linear_multi(1, types, wp, yp, rp, np, x, nullptr, 0.0f, M, K, stream);
}

extern "C" int64_t t2c_linear_allreduce_buffer_bytes(int64_t n_max) {
    return kArFlagBytes + 2 * static_cast<int64_t>(kArMaxRanks) * n_max * 4;
}

extern "C" int t2c_linear_allreduce(int wtype, const void *x, const void *w, const void *residual, void *y,
                                    int64_t M, int64_t N, int64_t K, void *const *bufs, int rank, int tp,
                                    uint32_t *counter, int64_t n_max, void *stream) {
    int rc = validate_common(M, K, x);
    if (rc) return rc;
    if ((rc = validate_weight(wtype, w, K))) return rc;
    if (y == nullptr || N <= 0) return set_error(T2C_EINVAL, "linear_allreduce: bad output or N");
    if (!bufs || !counter || tp < 2 || tp > kArMaxRanks || rank < 0 || rank >= tp)
        return set_error(T2C_EINVAL, "linear_allreduce: bad rank / tp / buffers");
    for (int q = 0; q < tp; ++q)
        if (!bufs[q] || reinterpret_cast<uintptr_t>(bufs[q]) % 256)
            return set_error(T2C_EINVAL, "linear_allreduce: bad peer buffer %d", q);
    if (M != 1 || wtype != T2C_Q4_K || N % kMmaRows || N > n_max || N > kArMaxRows || K % (kMmaSegBlocks * 256) ||
        n_max % 4)
        return set_error(T2C_EUNSUPPORTED, "linear_allreduce: 1 token, Q4_K, N a multiple of 16 up to %d, "
                                           "K a multiple of %d", kArMaxRows, kMmaSegBlocks * 256);
    QParams p = {};
    p.nstreams = 1;
    p.mode = MODE_ROWS;
    p.x = static_cast<const __half *>(x);
    p.K = static_cast<int>(K);
    p.s[0].w = static_cast<const uint8_t *>(w);
    p.s[0].y = static_cast<__half *>(y);
    p.s[0].res = static_cast<const __half *>(residual);
    p.s[0].n = N;
    p.s[0].row_bytes = row_bytes(wtype, K);
    p.s[0].fmt = wtype;
    for (int q = 0; q < tp; ++q) p.ar_peer[q] = static_cast<uint8_t *>(bufs[q]);
    p.ar_counter = counter;
    p.ar_rank = rank;
    p.ar_tp = tp;
    p.ar_nmax = n_max;
    bool used = false;
    rc = try_mma(p, M, as_stream(stream), used);
    if (!used) return set_error(T2C_EUNSUPPORTED, "linear_allreduce: the M = 1 tensor-core kernel does not serve this shape");
    return rc;
}

extern "C" int t2c_linear_swiglu(int wtype, const void *x, const void *w_gate, const void *w_up, void *y,
                                 const float *norm_weight, float eps, int64_t M, int64_t N, int64_t K,
                                 void *stream) {
    int rc = validate_common(M, K, x);
    if (rc) return rc;
    if ((rc = validate_weight(wtype, w_gate, K)) || (rc = validate_weight(wtype, w_up, K))) return rc;
    if (y == nullptr || N <= 0) return set_error(T2C_EINVAL, "bad output or N");
    QParams p = {};
    p.nstreams = 2;
    p.mode = MODE_SWIGLU;
    p.x = static_cast<const __half *>(x);
    p.norm_w = norm_weight;
    p.eps = eps;
    p.K = static_cast<int>(K);
    const int64_t rb = row_bytes(wtype, K);
    p.s[0].w = static_cast<const uint8_t *>(w_gate);
    p.s[0].y = static_cast<__half *>(y);
    p.s[0].n = N;
    p.s[0].row_bytes = rb;
    p.s[0].fmt = wtype;
    p.s[1] = p.s[0];
    p.s[1].w = static_cast<const uint8_t *>(w_up);
    p.s[1].y = nullptr;
    return run_linear(p, M, as_stream(stream));
}

extern "C" int t2c_lm_head_argmax(int wtype, const void *x, const void *w, float *partial_scores,
                                  uint32_t *partial_tokens, const float *norm_weight, float eps, int64_t M,
                                  int64_t N, int64_t K, void *stream) {
    int rc = validate_common(M, K, x);
    if (rc) return rc;
    if ((rc = validate_weight(wtype, w, K))) return rc;
    if (!partial_scores || !partial_tokens || N <= 0) return set_error(T2C_EINVAL, "lm_head_argmax: bad output");
    QParams p = {};
    p.nstreams = 1;
    p.mode = MODE_ARGMAX;
    p.x = static_cast<const __half *>(x);
    p.norm_w = norm_weight;
    p.eps = eps;
    p.K = static_cast<int>(K);
    p.s[0].w = static_cast<const uint8_t *>(w);
    p.s[0].n = N;
    p.s[0].row_bytes = row_bytes(wtype, K);
    p.s[0].fmt = wtype;
    p.ps = partial_scores;
    p.pt = partial_tokens;
    p.G = (N + 3) / 4;
    return run_linear(p, M, as_stream(stream));
}

extern "C" int64_t t2c_linear_f32_scratch_bytes(int64_t M, int64_t N, int64_t K) {
    return (M * K * 2 + 255) / 256 * 256 + M * N * 2;
}

extern "C" int t2c_linear_f32(int wtype, const float *x, const void *w, float *y, int64_t M, int64_t N, int64_t K,
                              void *scratch, int64_t scratch_bytes, void *stream) {
    int rc = validate_common(M, K, x);
    if (rc) return rc;
    if ((rc = validate_weight(wtype, w, K))) return rc;
    if (y == nullptr || N <= 0) return set_error(T2C_EINVAL, "linear_f32: bad output or N");
    if (scratch == nullptr || reinterpret_cast<uintptr_t>(scratch) % 256 ||
        scratch_bytes < t2c_linear_f32_scratch_bytes(M, N, K))
        return set_error(T2C_ESCRATCH, "linear_f32: scratch needs %lld bytes (256-byte aligned)",
                         (long long)t2c_linear_f32_scratch_bytes(M, N, K));
    // x rounded to fp16 (the reference's cooperative-matrix operands are fp16 as well)
    __half *x16 = static_cast<__half *>(scratch);
    __half *y16 = reinterpret_cast<__half *>(static_cast<uint8_t *>(scratch) + (M * K * 2 + 255) / 256 * 256);
    if ((rc = t2c_cast(x, T2C_F32, x16, T2C_F16, M * K, stream))) return rc;
    const cudaStream_t s = as_stream(stream);
    if (M > 4 && (wtype == T2C_Q4_K || wtype == T2C_Q8_0 || wtype == T2C_Q6_K)) {
        // tensor-core GEMM writing fp32 directly from the TMEM accumulators
        QGemmArgs a = {};
        a.fmt = wtype;
        a.nw = 1;
        a.w[0] = static_cast<const uint8_t *>(w);
        a.N[0] = N;
        a.K = K;
        a.M = M;
        a.x = x16;
        a.yf[0] = y;
        rc = qgemm(a, s);
        if (rc != T2C_EUNSUPPORTED) return rc;
    }
    // other shapes: the fp16 kernels, then widen
    if ((rc = t2c_linear(wtype, x16, w, nullptr, y16, M, N, K, stream))) return rc;
    return t2c_cast(y16, T2C_F16, y, T2C_F32, M * N, stream);
}

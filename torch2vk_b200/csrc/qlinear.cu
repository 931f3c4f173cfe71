// Quantized linear for decode-sized batches (M <= 8 per launch chunk):
// y[m, n] = sum_k x[m, k] * deq(W)[n, k] over GGUF Q4_K / Q6_K / Q8_0 rows.
//
// B200 design (HBM-bound):
//  * x prologue: each CTA turns its x rows into 15-bit fixed point per
//    32-value sub-block (x ~= sx * (128 * xh + xl), xh int8, xl in [0,127])
//    in shared memory, optionally applying RMSNorm on the way.
//  * Streamed kernel (qmv_tma_kernel): persistent CTAs; a producer warp
//    streams row blocks of the packed weight matrix HBM -> shared memory with
//    1-D bulk async copies (cp.async.bulk, completion on mbarriers) through a
//    ring of stages, while four consumer warps decode the staged blocks.  The
//    copies need no registers, so the bytes in flight per SM are set by the
//    ring depth, not by occupancy.
//  * Decode: integer nibble / 6-bit / int8 codes meet the int8 x planes in
//    dp4a (exact integer sub-block sums); the block scales d*sc and dmin*m
//    are applied once per sub-block in fp32.  Each lane keeps four rows'
//    partial sums so one x fragment serves four rows; partial sums are
//    reduced with warp shuffles.
//  * Epilogues: + residual (matvec_add), silu(gate) * up (SwiGLU pair), fp16
//    store.
//  * Direct kernel (qmv_direct_kernel): the same decode reading weights
//    straight from global memory; used when a layout cannot be bulk-copied
//    (16-byte alignment).
// Semantics follow the reference matvec shaders
// (src/models/quantized_qwen3/shaders/linear_nobias_q4_k_matvec_f32.py:107-197,
//  linear_nobias_q6_k_matvec_f32.py:116-193, linear_nobias_q8_0_matvec_f32.py:84-119):
// fp32 accumulation of x * (d*sc*q - dmin*m); only the rounding of x to
// 15 bits per 32-value sub-block differs (relative error <= 2^-15 of the
// sub-block maximum).
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
};

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

__device__ __forceinline__ void mma_s8_16832(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}

// Scales of sub-blocks 2t, 2t+1 of one Q4_K block header (d*sc, dmin*m).
__device__ __forceinline__ void q4k_pair_scales(const uint4 h, int t, float &ds0, float &ds1, float &dm0, float &dm1) {
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const int i0 = (2 * t) & 3;
    const bool low = t < 2;
    const uint32_t y = h.y >> (8 * i0), z = h.z >> (8 * i0), w = h.w >> (8 * i0);
    const uint32_t hs = ((y >> 6) & 0x3u) | (((y >> 14) & 0x3u) << 8);
    const uint32_t hm = ((z >> 6) & 0x3u) | (((z >> 14) & 0x3u) << 8);
    const uint32_t scp = low ? (y & 0x3F3Fu) : ((w & 0x0F0Fu) | (hs << 4));
    const uint32_t mnp = low ? (z & 0x3F3Fu) : (((w >> 4) & 0x0F0Fu) | (hm << 4));
    ds0 = d * small_u2f(scp & 0xffu);
    ds1 = d * small_u2f(scp >> 8);
    dm0 = dmin * small_u2f(mnp & 0xffu);
    dm1 = dmin * small_u2f(mnp >> 8);
}

// One 144-byte super-block of a 16-row group: acc[0] row g, acc[1] row g+8 (batch row t).
// rowg: shared address of the block in row g; xk: x offset (values) of the block.
__device__ __forceinline__ void mma_q4k_block(uint32_t rowg, uint32_t row_stride, int kabs, const XS &x, int lane,
                                              int M, float acc[2]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t rowg8 = rowg + 8u * row_stride;
    const uint4 hg = lds128(rowg), hg8 = lds128(rowg8);
    float ds[2][2], dm[2][2];
    q4k_pair_scales(hg, t, ds[0][0], ds[0][1], dm[0][0], dm[0][1]);
    q4k_pair_scales(hg8, t, ds[1][0], ds[1][1], dm[1][0], dm[1][1]);
    // B column g: batch row g/2, plane g%2 (zero for absent batch rows)
    const bool bcol = (g >> 1) < M;
    const uint32_t xplane = (g & 1) ? x.xl : x.xh;
    const int bm = bcol ? (g >> 1) : 0;
    const bool dcol = t < M;
    const int dmrow = dcol ? t : 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint2 wg = lds64(rowg + 16 + 32 * q + 8 * t);
        const uint2 wg8 = lds64(rowg8 + 16 + 32 * q + 8 * t);
        const int k0 = kabs + 64 * q + 8 * t;
        const uint2 b_lo = bcol ? lds64(xplane + x.off(bm, k0)) : make_uint2(0u, 0u);
        const uint2 b_hi = bcol ? lds64(xplane + x.off(bm, k0 + 32)) : make_uint2(0u, 0u);
        const uint4 mt = lds128(x.meta + 16u * static_cast<uint32_t>(dmrow * x.u64 + ((kabs >> 6) + q)));
        const uint32_t a_lo[4] = {wg.x & 0x0F0F0F0Fu, wg8.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu, wg8.y & 0x0F0F0F0Fu};
        const uint32_t a_hi[4] = {(wg.x >> 4) & 0x0F0F0F0Fu, (wg8.x >> 4) & 0x0F0F0F0Fu, (wg.y >> 4) & 0x0F0F0F0Fu,
                                  (wg8.y >> 4) & 0x0F0F0F0Fu};
        int d_lo[4], d_hi[4];
        mma_s8_16832(d_lo, a_lo, b_lo.x, b_lo.y);
        mma_s8_16832(d_hi, a_hi, b_hi.x, b_hi.y);
        // scales of sub-blocks 2q, 2q+1 live in lane (g, q)
        const int src = (lane & ~3) | q;
        const float s0g = __shfl_sync(0xffffffffu, ds[0][0], src), s1g = __shfl_sync(0xffffffffu, ds[0][1], src);
        const float m0g = __shfl_sync(0xffffffffu, dm[0][0], src), m1g = __shfl_sync(0xffffffffu, dm[0][1], src);
        const float s0h = __shfl_sync(0xffffffffu, ds[1][0], src), s1h = __shfl_sync(0xffffffffu, ds[1][1], src);
        const float m0h = __shfl_sync(0xffffffffu, dm[1][0], src), m1h = __shfl_sync(0xffffffffu, dm[1][1], src);
        const float sx0 = dcol ? __uint_as_float(mt.x) : 0.0f, sx1 = dcol ? __uint_as_float(mt.y) : 0.0f;
        const float xs0 = dcol ? __uint_as_float(mt.z) : 0.0f, xs1 = dcol ? __uint_as_float(mt.w) : 0.0f;
        acc[0] = fmaf(s0g * sx0, static_cast<float>(d_lo[0] * 128 + d_lo[1]), acc[0]);
        acc[1] = fmaf(s0h * sx0, static_cast<float>(d_lo[2] * 128 + d_lo[3]), acc[1]);
        acc[0] = fmaf(s1g * sx1, static_cast<float>(d_hi[0] * 128 + d_hi[1]), acc[0]);
        acc[1] = fmaf(s1h * sx1, static_cast<float>(d_hi[2] * 128 + d_hi[3]), acc[1]);
        acc[0] = fmaf(-m0g, xs0, fmaf(-m1g, xs1, acc[0]));
        acc[1] = fmaf(-m0h, xs0, fmaf(-m1h, xs1, acc[1]));
    }
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

// Split-K partials of a row block meet in a shared-memory slot: each warp of the
// block's group adds its rows, and the last to arrive applies the epilogue.
// Slot (iteration % kMmaSlots, group) is reused once the previous use is done
// (generation counter); the wait for that is bounded.
constexpr int kMmaSlots = 4;
struct MmaSlot {
    float v[2][kMmaRows][4];  // [gate/up or value][row][batch row]
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
    float4 *meta = reinterpret_cast<float4 *>(slots + kMmaSlots * kMmaWarps);
    int8_t *xh = reinterpret_cast<int8_t *>(meta + MT * (K >> 6));
    int8_t *xl = xh + MT * padded_k(K) + 32;  // +32: xh / xl fragments of one k on different banks
    float *sx = reinterpret_cast<float *>(xl + MT * padded_k(K));
    int *xq16 = reinterpret_cast<int *>(sx + MT * (K >> 5));
    float *pred = reinterpret_cast<float *>(xq16 + MT * (K >> 4));
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
    prepare_x<MT, kMmaThreads>(p, xh, xl, sx, xq16, meta, pred);  // ends with a CTA barrier
    const XS x{smem_u32(xh), smem_u32(xl), smem_u32(meta), smem_u32(sx), smem_u32(xq16), padded_k(K), K >> 6,
               K >> 5};
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
        MmaSlot *slot = slots + (it % kMmaSlots) * kMmaWarps + group;
        if (!slot_wait_gen(&slot->gen, static_cast<int>(it / kMmaSlots))) {
            report_device_error(T2C_ETIMEOUT);
            failed = true;
            continue;
        }
        if (t < p.M) {  // lane (g, t) holds rows g, g+8 of batch row t
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                atomicAdd(&slot->v[r][g][t], acc[r][0]);
                atomicAdd(&slot->v[r][g + 8][t], acc[r][1]);
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
        float v[2][2];
        const int tm = t < p.M ? t : 0;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            v[r][0] = *reinterpret_cast<volatile float *>(&slot->v[r][g][tm]);
            v[r][1] = *reinterpret_cast<volatile float *>(&slot->v[r][g + 8][tm]);
        }
        mma_finish_block<MT>(p, block, v, lane);
        __syncwarp();
        if (t < p.M) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                slot->v[r][g][t] = 0.0f;
                slot->v[r][g + 8][t] = 0.0f;
            }
        }
        __syncwarp();
        if (lane == 0) {
            slot->arrived = 0;
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&slot->gen) = slot->gen + 1;
        }
    }
}

// ------------------------------------------------ M = 1 kernel, per-warp x
// Same streaming and split-K as qmv_mma_kernel, but each warp quantizes only
// the x values of its own K-segments (after, when there is a fused RMSNorm,
// a warp-local sum of squares over the whole row), so the prologue has no
// CTA barrier and x costs ~1.2 KB of shared memory per segment: two CTAs fit
// on an SM.  Per segment: xh[512], 32-byte gap, xl[512], then (sx', xs) per
// 32-value sub-block, where sx' = sx / 16 for the odd (high-nibble) sub-blocks.
constexpr int kM1SegX = 512 + 32 + 512 + 32;      // plane bytes (+ gaps)
constexpr int kM1SegBytes = kM1SegX + 16 * 8;    // + meta
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

// Quantizes one segment of x (f, already scaled by the RMSNorm when there is
// one) into a segment area.
__device__ __forceinline__ void m1_prepare_segment(const float f[16], uint8_t *area, int lane) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) amax = fmaxf(amax, fabsf(f[e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));  // lanes 2i, 2i+1 = sub-block i
    const float inv = amax > 0.0f ? 16383.0f / amax : 0.0f;
    uint32_t hw[4] = {0u, 0u, 0u, 0u}, lw[4] = {0u, 0u, 0u, 0u};
    int sum = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        int q = __float2int_rn(f[e] * inv);
        q = max(-16383, min(16383, q));
        sum += q;
        hw[e >> 2] |= (static_cast<uint32_t>(q >> 7) & 0xffu) << (8 * (e & 3));
        lw[e >> 2] |= static_cast<uint32_t>(q & 127) << (8 * (e & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    *reinterpret_cast<uint4 *>(area + 16 * lane) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4 *>(area + 512 + 32 + 16 * lane) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    if ((lane & 1) == 0) {
        const float sx = amax / 16383.0f;
        // sub-block lane / 2: the odd ones are high nibbles, which enter the mma as 16 q
        const float f_sx = (lane & 2) ? sx * 0.0625f : sx;
        *reinterpret_cast<float2 *>(area + kM1SegX + 8 * (lane >> 1)) = make_float2(f_sx, sx * static_cast<float>(sum));
    }
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

// Fragment mapping of the M = 1 kernel (m16n8k32, A = 16 weight rows, B = x).
// In a group G of two quarters (sub-blocks 4G .. 4G+3), lane (g, t) loads 16
// bytes of rows g and g+8: quarter 2G + (t & 1), bytes 16 (t >> 1) .. +15.
// mma i takes word i of each: its low nibbles fill k-slots 4t .. 4t+3 and its
// high nibbles (unshifted, i.e. 16 q) k-slots 16+4t .. 16+4t+3.  So k-slots
// {0-3, 8-11} hold the low-nibble sub-block of quarter 2G (sub-block 4G),
// {4-7, 12-15} that of quarter 2G+1 (4G+2), {16-19, 24-27} sub-block 4G+1 and
// {20-23, 28-31} sub-block 4G+3.  B column pair c carries the two x planes of
// one of them (c = 0: 4G, 1: 4G+2, 2: 4G+1, 3: 4G+3), zero in the other
// k-slots, so D columns 2t, 2t+1 of lane (g, t) are sub-block 4G + cc(t),
// cc = {0, 2, 1, 3}[t]: every lane applies the scales of one sub-block per
// group, and the four lanes of a quad are summed per row block at the end.
struct M1Lane {
    uint32_t aoff;   // A words in a 144-byte block
    uint32_t xoff;   // x plane words of G = 0 in a segment area
    uint32_t moff;   // (sx', xs) of sub-block cc of G = 0 in a segment area
    uint32_t m0, m1; // B masks: k-slots < 16 / >= 16 carry this lane's x column
    uint32_t sel;    // byte_perm selector of header byte cc
};

__device__ __forceinline__ M1Lane m1_lane(int lane) {
    const int g = lane >> 2, t = lane & 3, c = g >> 1, plane = g & 1;
    const int cc = ((t & 1) << 1) | (t >> 1);
    const bool mine = (c & 1) == (t & 1);
    M1Lane L;
    L.aoff = static_cast<uint32_t>(16 + 32 * (t & 1) + 16 * (t >> 1));
    L.xoff = static_cast<uint32_t>((plane ? 512 + 32 : 0) + 32 * (2 * (t & 1) + (c >> 1)) + 16 * (t >> 1));
    L.moff = static_cast<uint32_t>(kM1SegX + 8 * cc);
    L.m0 = (mine && c < 2) ? 0xffffffffu : 0u;
    L.m1 = (mine && c >= 2) ? 0xffffffffu : 0u;
    L.sel = 0x4440u + static_cast<uint32_t>(cc);
    return L;
}

__device__ __forceinline__ void mma_u8s8_16832(int d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d * sc and dmin * m of sub-blocks cc and cc + 4 of one Q4_K header.
__device__ __forceinline__ void q4k_scales_sel(const uint4 h, uint32_t sel, float ds[2], float dm[2]) {
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    const uint32_t y = __byte_perm(h.y, 0u, sel), z = __byte_perm(h.z, 0u, sel), w = __byte_perm(h.w, 0u, sel);
    ds[0] = d * small_u2f(y & 63u);
    dm[0] = dmin * small_u2f(z & 63u);
    ds[1] = d * small_u2f((w & 15u) | ((y >> 6) << 4));
    dm[1] = dmin * small_u2f((w >> 4) | ((z >> 6) << 4));
}

// One 144-byte block (values voff .. voff+255 of the segment) of a 16-row
// group whose rows are kMmaSegBytes apart; acc = rows g, g + 8.
__device__ __forceinline__ void m1_block(const uint8_t *rowg, const uint8_t *xseg, int voff, const M1Lane &L,
                                         float acc[2]) {
    const uint8_t *rowg8 = rowg + 8 * kMmaSegBytes;
    const uint4 hg = *reinterpret_cast<const uint4 *>(rowg), hg8 = *reinterpret_cast<const uint4 *>(rowg8);
    float dsg[2], dmg[2], dsh[2], dmh[2];
    q4k_scales_sel(hg, L.sel, dsg, dmg);
    q4k_scales_sel(hg8, L.sel, dsh, dmh);
#pragma unroll
    for (int G = 0; G < 2; ++G) {
        const uint4 X = *reinterpret_cast<const uint4 *>(xseg + L.xoff + voff + 128 * G);
        const float2 mt = *reinterpret_cast<const float2 *>(xseg + L.moff + (voff >> 2) + 32 * G);
        const uint4 qa = *reinterpret_cast<const uint4 *>(rowg + L.aoff + 64 * G);
        const uint4 ra = *reinterpret_cast<const uint4 *>(rowg8 + L.aoff + 64 * G);
        const uint32_t wa[4] = {qa.x, qa.y, qa.z, qa.w}, va[4] = {ra.x, ra.y, ra.z, ra.w};
        const uint32_t xw[4] = {X.x, X.y, X.z, X.w};
        int d[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t a[4] = {wa[i] & 0x0F0F0F0Fu, va[i] & 0x0F0F0F0Fu, wa[i] & 0xF0F0F0F0u, va[i] & 0xF0F0F0F0u};
            mma_u8s8_16832(d, a, xw[i] & L.m0, xw[i] & L.m1);
        }
        acc[0] = fmaf(dsg[G] * mt.x, static_cast<float>(d[0] * 128 + d[1]), fmaf(-dmg[G], mt.y, acc[0]));
        acc[1] = fmaf(dsh[G] * mt.x, static_cast<float>(d[2] * 128 + d[3]), fmaf(-dmh[G], mt.y, acc[1]));
    }
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
                for (int sb = 0; sb < kMmaSegBlocks; ++sb) m1_block(stage + sb * 144, xseg, sb * 256, L, part);
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
        mma_finish_block<1>(p, blk, v, lane, rv);
        __syncwarp();
        if (lane == 0) {
            slot->arrived = 0;
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&slot->gen) = slot->gen + 1;
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
    return kStageHead + kMmaSlots * kMmaWarps * sizeof(MmaSlot) + static_cast<size_t>(MT) * (K / 64) * 16 +
           2 * static_cast<size_t>(MT) * padded_k(K) + 32 + static_cast<size_t>(MT) * (K / 32) * 4 +
           static_cast<size_t>(MT) * (K / 16) * 4 + static_cast<size_t>(kMmaWarps) * MT * 4;
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
    return launch_pdl(qmv_m1_kernel, static_cast<int>(blocks), kMmaThreads, smem, stream, p);
}

bool mma_disabled() {
    static const bool off = [] {
        const char *v = getenv("T2C_QMV_DP4A");
        return v != nullptr && v[0] == '1';
    }();
    return off;
}

// Tensor-core path when every stream is Q4_K, M <= 4 and K splits into 512-value segments.
int try_mma(QParams p, int64_t M, cudaStream_t stream, bool &used) {
    used = false;
    if (mma_disabled() || M > 4 || p.K % (kMmaSegBlocks * 256) != 0) return T2C_OK;
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

// M > 4, Q4_K / Q6_K / Q8_0 streams, no fused RMSNorm: tcgen05 GEMM (fused QKV in one launch when the
// formats agree, else one launch per weight).
int try_gemm(const QParams &p, int64_t M, cudaStream_t stream, bool &used) {
    used = false;
    if (mma_disabled() || M <= 4 || p.norm_w != nullptr) return T2C_OK;
    const int fmt = p.s[0].fmt;
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
            const bool ok_fmt = fi == T2C_Q4_K || fi == T2C_Q8_0 || (fi == T2C_Q6_K && p.K % 2048 == 0);
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

int run_linear(QParams p, int64_t M, cudaStream_t stream) {
    bool used = false;
    const int rc_gemm = try_gemm(p, M, stream, used);
    if (used) return rc_gemm;
    const int rc_mma = try_mma(p, M, stream, used);
    if (used) return rc_mma;
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
    if (!mma_disabled() && M > 4 && (wtype == T2C_Q4_K || wtype == T2C_Q8_0 || (wtype == T2C_Q6_K && K % 2048 == 0))) {
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

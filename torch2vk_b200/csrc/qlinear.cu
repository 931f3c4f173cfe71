// Quantized linear for decode-sized batches (M <= 8 per launch chunk):
// y[m, n] = sum_k x[m, k] * deq(W)[n, k] over GGUF Q4_K / Q6_K / Q8_0 rows.
//
// Design (B200, HBM-bound):
//  * Each CTA first turns its x rows into 15-bit fixed point per 32-value
//    sub-block (x ~= sx * (128 * xh + xl), xh int8, xl in [0,127]) in shared
//    memory, optionally applying RMSNorm on the way (fused prologue).
//  * Warps (or 16/8-lane sub-warps for short rows) then stream weight rows
//    straight from HBM with coalesced 16-byte (Q4_K) or 4-byte funnel-aligned
//    (Q6_K, Q8_0) loads, four rows at a time so every x fragment held in
//    registers serves four rows.  Integer nibble/6-bit codes meet the int8 x
//    planes in dp4a; the integer sub-block sums are exact, and the block scales
//    (d * sc, dmin * m) are applied once per sub-block in fp32.
//  * Partial row sums are reduced with warp shuffles; the epilogue adds the
//    residual (matvec_add), or forms silu(gate) * up (SwiGLU pair), and stores
//    fp16.
// Semantics follow the reference matvec shaders
// (src/models/quantized_qwen3/shaders/linear_nobias_q4_k_matvec_f32.py:107-197,
//  linear_nobias_q6_k_matvec_f32.py:116-193, linear_nobias_q8_0_matvec_f32.py:84-119):
// fp32 accumulation of x * (d*sc*q - dmin*m); only the rounding of x to
// 15 bits per 32-value sub-block differs (relative error <= 2^-15 of the
// sub-block maximum).
#include <stdio.h>

#include "common.cuh"

namespace t2c {
namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kRows = 4;  // rows per row-set (x fragments are reused across them)
constexpr int kMaxStreams = 3;

enum Mode : int { MODE_ROWS = 0, MODE_SWIGLU = 1 };

struct QStream {
    const uint8_t *w;
    __half *y;
    const __half *res;
    int64_t n;
    int64_t row_bytes;
    int64_t rs_begin;
    int fmt;
};

struct QParams {
    QStream s[kMaxStreams];
    int nstreams;
    int mode;
    const __half *x;
    const float *norm_w;
    float eps;
    int M;         // tokens in this launch chunk (<= MT)
    int K;
    int units;     // 64-value units per row
    int lpr;       // lanes per row-set (4, 8, 16 or 32)
    int64_t total_rowsets;
};

// Four weight rows: rows 0,1 start at base0 (+ r * row_bytes), rows 2,3 at base1.
struct RowSet {
    const uint8_t *base0;
    const uint8_t *base1;
    int64_t row_bytes;
    int valid;  // bit r set when row r exists
    __device__ __forceinline__ const uint8_t *row(int r) const {
        return ((valid >> r) & 1) ? ((r < 2 ? base0 : base1) + (r & 1) * row_bytes) : nullptr;
    }
};

struct XPlanes {
    const int8_t *xh;   // [MT][K]
    const int8_t *xl;   // [MT][K]
    const float *sx;    // [MT][K/32]
    const int *xq16;    // [MT][K/16] integer sums of (128 xh + xl) over 16 values
};

__device__ __forceinline__ uint32_t funnel16(uint32_t lo, uint32_t hi, uint32_t sh) {
    return __funnelshift_r(lo, hi, sh);
}

// Loads 16 bytes starting at a 2-byte aligned global address.
__device__ __forceinline__ uint4 load16_u2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *base = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t sh = static_cast<uint32_t>(a & 3) * 8u;
    uint32_t w0 = ldg_nc_u32(base + 0), w1 = ldg_nc_u32(base + 1), w2 = ldg_nc_u32(base + 2);
    uint32_t w3 = ldg_nc_u32(base + 3);
    uint32_t w4 = sh ? ldg_nc_u32(base + 4) : 0u;
    return make_uint4(funnel16(w0, w1, sh), funnel16(w1, w2, sh), funnel16(w2, w3, sh), funnel16(w3, w4, sh));
}

// ---------------------------------------------------------------- x prologue
// Chunks of 8 fp16 values (16 bytes).  Thread t owns chunks t, t + kThreads,
// ...; the four chunks of a 32-value sub-block sit on four consecutive lanes,
// so sub-block maxima and 16-value sums are two/one xor-shuffles away.  Loads
// are issued kRound chunks at a time so their latencies overlap.
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

template <int MT>
__device__ void prepare_x(const QParams &p, int8_t *xh, int8_t *xl, float *sx, int *xq16, float *red) {
    const int K = p.K;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
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
                const int c = base + i * kThreads + threadIdx.x;
                const int m = c / chunks_per_row;
                v[i] = (c < total && m < p.M) ? xv[c] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < kRound; ++i) {
                const int c = base + i * kThreads + threadIdx.x;
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
        __syncthreads();
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
            const int c = base + i * kThreads + threadIdx.x;
            const int m = c / chunks_per_row;
            v[i] = (c < total && m < p.M) ? xv[c] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < kRound; ++i) {
            const int c = base + i * kThreads + threadIdx.x;
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
                *reinterpret_cast<uint2 *>(xh + c * 8) = make_uint2(hw[0], hw[1]);
                *reinterpret_cast<uint2 *>(xl + c * 8) = make_uint2(lw[0], lw[1]);
                if ((lane & 1) == 0) xq16[c >> 1] = sum;
                if ((lane & 3) == 0) sx[c >> 2] = amax / 16383.0f;
            }
        }
    }
}

// ------------------------------------------------------------- Q4_K unit
// Unit u of a row = group G (32 bytes) of block b: low nibbles are sub-block
// 2G (k0 .. k0+31), high nibbles sub-block 2G+1 (k0+32 .. k0+63).
template <int MT>
__device__ __forceinline__ void unit_q4k(const RowSet &rows, int u, int K, const XPlanes &xp,
                                         float acc[kRows][MT]) {
    const int b = u >> 2, G = u & 3;
    const int k0 = b * 256 + G * 64;
    const int j0 = k0 >> 5;
    uint4 hdr[kRows], q0[kRows], q1[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        if ((rows.valid >> r) & 1) {
            const uint8_t *blk = rows.row(r) + b * 144;
            hdr[r] = ldg_nc_v4(blk);
            q0[r] = ldg_nc_v4(blk + 16 + G * 32);
            q1[r] = ldg_nc_v4(blk + 32 + G * 32);
        } else {
            hdr[r] = make_uint4(0, 0, 0, 0);
            q0[r] = hdr[r];
            q1[r] = hdr[r];
        }
    }
    // 6-bit scale/min codes for sub-blocks 2G and 2G+1 (quantize/vulkan.py:331-342 packing)
    float ds0[kRows], ds1[kRows], dm0[kRows], dm1[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        const float d = half_bits_to_float(hdr[r].x);
        const float dmin = half_bits_to_float(hdr[r].x >> 16);
        uint32_t sc0, sc1, mn0, mn1;
        const int j = 2 * G;
        if (G < 2) {
            sc0 = (hdr[r].y >> (8 * j)) & 63u;
            sc1 = (hdr[r].y >> (8 * j + 8)) & 63u;
            mn0 = (hdr[r].z >> (8 * j)) & 63u;
            mn1 = (hdr[r].z >> (8 * j + 8)) & 63u;
        } else {
            const int i0 = j - 4;
            const uint32_t lo0 = (hdr[r].w >> (8 * i0)) & 0xffu, lo1 = (hdr[r].w >> (8 * i0 + 8)) & 0xffu;
            const uint32_t s0 = (hdr[r].y >> (8 * i0)) & 0xffu, s1 = (hdr[r].y >> (8 * i0 + 8)) & 0xffu;
            const uint32_t m0 = (hdr[r].z >> (8 * i0)) & 0xffu, m1 = (hdr[r].z >> (8 * i0 + 8)) & 0xffu;
            sc0 = (lo0 & 15u) | ((s0 >> 6) << 4);
            sc1 = (lo1 & 15u) | ((s1 >> 6) << 4);
            mn0 = (lo0 >> 4) | ((m0 >> 6) << 4);
            mn1 = (lo1 >> 4) | ((m1 >> 6) << 4);
        }
        ds0[r] = d * static_cast<float>(sc0);
        ds1[r] = d * static_cast<float>(sc1) * 0.0625f;  // high nibbles enter dp4a as 16*q
        dm0[r] = dmin * static_cast<float>(mn0);
        dm1[r] = dmin * static_cast<float>(mn1);
    }
    const int sub_per_row = K >> 5;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int4 *xhv = reinterpret_cast<const int4 *>(xp.xh + m * K + k0);
        const int4 *xlv = reinterpret_cast<const int4 *>(xp.xl + m * K + k0);
        const int4 hA0 = xhv[0], hA1 = xhv[1], hB0 = xhv[2], hB1 = xhv[3];
        const int4 lA0 = xlv[0], lA1 = xlv[1], lB0 = xlv[2], lB1 = xlv[3];
        const float s0 = xp.sx[m * sub_per_row + j0];
        const float s1 = xp.sx[m * sub_per_row + j0 + 1];
        const int *q16 = xp.xq16 + (m * sub_per_row + j0) * 2;
        const float xs0 = s0 * static_cast<float>(q16[0] + q16[1]);
        const float xs1 = s1 * static_cast<float>(q16[2] + q16[3]);
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
            const uint32_t wA[8] = {q0[r].x, q0[r].y, q0[r].z, q0[r].w, q1[r].x, q1[r].y, q1[r].z, q1[r].w};
            const int xhA[8] = {hA0.x, hA0.y, hA0.z, hA0.w, hA1.x, hA1.y, hA1.z, hA1.w};
            const int xlA[8] = {lA0.x, lA0.y, lA0.z, lA0.w, lA1.x, lA1.y, lA1.z, lA1.w};
            const int xhB[8] = {hB0.x, hB0.y, hB0.z, hB0.w, hB1.x, hB1.y, hB1.z, hB1.w};
            const int xlB[8] = {lB0.x, lB0.y, lB0.z, lB0.w, lB1.x, lB1.y, lB1.z, lB1.w};
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
// Unit u = (block b, half s, l-half lh): values i = 128 s + 32 c + 16 lh + l,
// c = 0..3, l = 0..15 (quantize/vulkan.py:542-564 layout).
template <int MT>
__device__ __forceinline__ void unit_q6k(const RowSet &rows, int u, int K, const XPlanes &xp,
                                         float acc[kRows][MT]) {
    const int b = u >> 2, s = (u >> 1) & 1, lh = u & 1;
    const int kbase = b * 256 + s * 128 + lh * 16;
    uint4 qa[kRows], qb[kRows], qh[kRows];
    float dsc[kRows][4];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        if ((rows.valid >> r) & 1) {
            const uint8_t *blk = rows.row(r) + b * 210;
            qa[r] = load16_u2(blk + 64 * s + 16 * lh);
            qb[r] = load16_u2(blk + 64 * s + 32 + 16 * lh);
            qh[r] = load16_u2(blk + 128 + 32 * s + 16 * lh);
            const float d = half_bits_to_float(ldg_nc_u16(blk + 208));
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t pair = ldg_nc_u16(blk + 192 + 8 * s + 2 * c);
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
            const int k = kbase + 32 * c;
            const int4 xh4 = *reinterpret_cast<const int4 *>(xp.xh + m * K + k);
            const int4 xl4 = *reinterpret_cast<const int4 *>(xp.xl + m * K + k);
            const float sxv = xp.sx[m * sub_per_row + (k >> 5)];
            const int q16 = xp.xq16[m * sub_per_row * 2 + (k >> 4)];
            const int xhw[4] = {xh4.x, xh4.y, xh4.z, xh4.w};
            const int xlw[4] = {xl4.x, xl4.y, xl4.z, xl4.w};
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
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
// Unit u = blocks 2u and 2u+1 (68 bytes, 4-byte aligned when K % 64 == 0).
template <int MT>
__device__ __forceinline__ void unit_q8_0(const RowSet &rows, int u, int K, const XPlanes &xp,
                                          float acc[kRows][MT]) {
    uint32_t qa[kRows][8], qb[kRows][8];
    float da[kRows], db[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
        if ((rows.valid >> r) & 1) {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(rows.row(r) + u * 68);
            uint32_t w[17];
#pragma unroll
            for (int i = 0; i < 17; ++i) w[i] = ldg_nc_u32(p + i);
            da[r] = half_bits_to_float(w[0]);
            db[r] = half_bits_to_float(w[8] >> 16);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qa[r][i] = funnel16(w[i], w[i + 1], 16);
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
    const int sub_per_row = K >> 5;
    const int k0 = u * 64;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
        const int4 *xhv = reinterpret_cast<const int4 *>(xp.xh + m * K + k0);
        const int4 *xlv = reinterpret_cast<const int4 *>(xp.xl + m * K + k0);
        const int4 h0 = xhv[0], h1 = xhv[1], h2 = xhv[2], h3 = xhv[3];
        const int4 l0 = xlv[0], l1 = xlv[1], l2 = xlv[2], l3 = xlv[3];
        const int xhA[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const int xlA[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
        const int xhB[8] = {h2.x, h2.y, h2.z, h2.w, h3.x, h3.y, h3.z, h3.w};
        const int xlB[8] = {l2.x, l2.y, l2.z, l2.w, l3.x, l3.y, l3.z, l3.w};
        const float sA = xp.sx[m * sub_per_row + (k0 >> 5)];
        const float sB = xp.sx[m * sub_per_row + (k0 >> 5) + 1];
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
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

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

// FMT: the weight type of every stream, or 0 when streams mix types.
template <int MT, int FMT>
__global__ void __launch_bounds__(kThreads, (MT == 1 ? 2 : 1)) qmv_kernel(const QParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int K = p.K;
    int8_t *xh = reinterpret_cast<int8_t *>(smem);
    int8_t *xl = xh + MT * K;
    float *sx = reinterpret_cast<float *>(xl + MT * K);
    int *xq16 = reinterpret_cast<int *>(sx + MT * (K >> 5));
    float *red = reinterpret_cast<float *>(xq16 + MT * (K >> 4));

    pdl_wait();
    prepare_x<MT>(p, xh, xl, sx, xq16, red);
    __syncthreads();
    pdl_trigger();

    const XPlanes xp{xh, xl, sx, xq16};
    const int lane = threadIdx.x & 31;
    const int lpr = p.lpr;
    const int sub = lane / lpr;              // sub-warp index
    const int sub_lane = lane - sub * lpr;   // lane within the sub-warp
    const int subs_per_warp = 32 / lpr;
    const int64_t gsub = (static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5)) * subs_per_warp + sub;
    const int64_t gsub_stride = static_cast<int64_t>(gridDim.x) * kWarps * subs_per_warp;

    // Every sub-warp runs the same number of iterations so the shuffles below
    // always see full warps; row-sets past the end are masked out.
    const int64_t iters = (p.total_rowsets + gsub_stride - 1) / gsub_stride;
    for (int64_t it = 0; it < iters; ++it) {
        const int64_t rs = gsub + it * gsub_stride;
        RowSet rows{nullptr, nullptr, 0, 0};
        int fmt = T2C_Q4_K;
        int si = 0;
        int64_t n0 = 0;
        if (rs < p.total_rowsets) {
            if (p.mode == MODE_SWIGLU) {
                // rows 0,1: gate rows n0, n0+1; rows 2,3: up rows n0, n0+1
                fmt = p.s[0].fmt;
                n0 = rs * 2;
                const int64_t nv = p.s[0].n - n0;
                rows.base0 = p.s[0].w + n0 * p.s[0].row_bytes;
                rows.base1 = p.s[1].w + n0 * p.s[1].row_bytes;
                rows.row_bytes = p.s[0].row_bytes;
                rows.valid = nv >= 2 ? 0xF : 0x5;
            } else {
#pragma unroll
                for (int i = 1; i < kMaxStreams; ++i)
                    if (i < p.nstreams && rs >= p.s[i].rs_begin) si = i;
                const QStream &st = p.s[si];
                fmt = st.fmt;
                n0 = (rs - st.rs_begin) * kRows;
                const int64_t nv = st.n - n0;
                rows.base0 = st.w + n0 * st.row_bytes;
                rows.base1 = rows.base0 + 2 * st.row_bytes;
                rows.row_bytes = st.row_bytes;
                rows.valid = nv >= 4 ? 0xF : ((1 << nv) - 1);
            }
        }
        float acc[kRows][MT];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
        if (FMT != 0) fmt = FMT;
        if (rs < p.total_rowsets) {
            if (fmt == T2C_Q4_K) {
                for (int u = sub_lane; u < p.units; u += lpr) unit_q4k<MT>(rows, u, K, xp, acc);
            } else if (fmt == T2C_Q6_K) {
                for (int u = sub_lane; u < p.units; u += lpr) unit_q6k<MT>(rows, u, K, xp, acc);
            } else {
                for (int u = sub_lane; u < p.units; u += lpr) unit_q8_0<MT>(rows, u, K, xp, acc);
            }
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                float v = acc[r][m];
                for (int o = lpr >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                acc[r][m] = v;
            }
        if (sub_lane == 0 && rs < p.total_rowsets) {
            if (p.mode == MODE_SWIGLU) {
                __half *y = p.s[0].y;
                const int64_t N = p.s[0].n;
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    if ((rows.valid >> r) & 1) {
#pragma unroll
                        for (int m = 0; m < MT; ++m)
                            if (m < p.M) y[m * N + n0 + r] = __float2half_rn(silu(acc[r][m]) * acc[r + 2][m]);
                    }
                }
            } else {
                const QStream &st = p.s[si];
#pragma unroll
                for (int r = 0; r < kRows; ++r) {
                    if (!((rows.valid >> r) & 1)) continue;
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        if (m < p.M) {
                            const int64_t o = m * st.n + n0 + r;
                            float v = acc[r][m];
                            if (st.res) v += __half2float(st.res[o]);
                            st.y[o] = __float2half_rn(v);
                        }
                    }
                }
            }
        }
    }
}

size_t smem_bytes(int MT, int K) {
    return static_cast<size_t>(MT) * K * 2 + static_cast<size_t>(MT) * (K / 32) * 4 +
           static_cast<size_t>(MT) * (K / 16) * 4 + static_cast<size_t>(kWarps) * 8 * 4;
}

int pick_mt(int64_t M, int K) {
    const size_t budget = 160 * 1024;
    int mt = 8;
    while (mt > 1 && (mt / 2 >= M || smem_bytes(mt, K) > budget)) mt /= 2;
    return mt;
}

template <int MT, int FMT>
int launch_mt(QParams p, cudaStream_t stream) {
    const size_t smem = smem_bytes(MT, p.K);
    static bool configured[64] = {false};
    int device = 0;
    cudaGetDevice(&device);
    if (device < 0 || device >= 64) return set_error(T2C_EINVAL, "device index %d out of range", device);
    if (!configured[device]) {
        if (cudaFuncSetAttribute(qmv_kernel<MT, FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
            cudaSuccess) {
            return set_error(T2C_ECUDA, "qmv: cudaFuncSetAttribute failed");
        }
        configured[device] = true;
    }
    const int sms = sm_count();
    const int subs_per_block = kWarps * (32 / p.lpr);
    int64_t blocks = (p.total_rowsets + subs_per_block - 1) / subs_per_block;
    const int64_t max_blocks = static_cast<int64_t>(sms) * (smem > 100 * 1024 ? 1 : 2);
    if (blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(blocks));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, qmv_kernel<MT, FMT>, p);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "qmv launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

template <int FMT>
int launch_fmt_mt(const QParams &c, int mt, cudaStream_t stream) {
    switch (mt) {
        case 1: return launch_mt<1, FMT>(c, stream);
        case 2: return launch_mt<2, FMT>(c, stream);
        case 4: return launch_mt<4, FMT>(c, stream);
        default: return launch_mt<8, FMT>(c, stream);
    }
}

int launch_fmt(const QParams &c, int mt, cudaStream_t stream) {
    int fmt = c.s[0].fmt;
    for (int i = 1; i < c.nstreams; ++i)
        if (c.s[i].fmt != fmt) fmt = 0;
    switch (fmt) {
        case T2C_Q4_K: return launch_fmt_mt<T2C_Q4_K>(c, mt, stream);
        case T2C_Q6_K: return launch_fmt_mt<T2C_Q6_K>(c, mt, stream);
        case T2C_Q8_0: return launch_fmt_mt<T2C_Q8_0>(c, mt, stream);
        default: return launch_fmt_mt<0>(c, mt, stream);
    }
}

int launch_chunked(QParams p, int64_t M, cudaStream_t stream) {
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
        int rc = launch_fmt(c, mt, stream);
        if (rc != T2C_OK) return rc;
    }
    return T2C_OK;
}

int validate_common(int64_t M, int64_t K, const void *x) {
    if (x == nullptr) return set_error(T2C_EINVAL, "x is NULL");
    if (M <= 0 || K <= 0) return set_error(T2C_EINVAL, "M=%lld K=%lld must be positive", (long long)M, (long long)K);
    if (K % 256 != 0 && K % 64 != 0) return set_error(T2C_EINVAL, "K=%lld must be a multiple of 64", (long long)K);
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

int lanes_per_row(int units) {
    int lpr = 32;
    while (lpr > 4 && lpr > units) lpr >>= 1;
    return lpr;
}

}  // namespace
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
    p.units = static_cast<int>(K / 64);
    p.lpr = lanes_per_row(p.units);
    int64_t rs = 0;
    for (int i = 0; i < count; ++i) {
        if ((rc = validate_weight(wtypes[i], ws[i], K))) return rc;
        if (ys[i] == nullptr || Ns[i] <= 0) return set_error(T2C_EINVAL, "stream %d: bad output or N", i);
        p.s[i].w = static_cast<const uint8_t *>(ws[i]);
        p.s[i].y = static_cast<__half *>(ys[i]);
        p.s[i].res = residuals ? static_cast<const __half *>(residuals[i]) : nullptr;
        p.s[i].n = Ns[i];
        p.s[i].row_bytes = row_bytes(wtypes[i], K);
        p.s[i].fmt = wtypes[i];
        p.s[i].rs_begin = rs;
        rs += (Ns[i] + kRows - 1) / kRows;
    }
    p.total_rowsets = rs;
    return launch_chunked(p, M, as_stream(stream));
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
    p.units = static_cast<int>(K / 64);
    p.lpr = lanes_per_row(p.units);
    const int64_t rb = row_bytes(wtype, K);
    p.s[0] = QStream{static_cast<const uint8_t *>(w_gate), static_cast<__half *>(y), nullptr, N, rb, 0, wtype};
    p.s[1] = QStream{static_cast<const uint8_t *>(w_up), nullptr, nullptr, N, rb, 0, wtype};
    p.total_rowsets = (N + 1) / 2;
    return launch_chunked(p, M, as_stream(stream));
}

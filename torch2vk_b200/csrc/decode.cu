// Decode-step kernels around the quantized linears: RMSNorm, fused q/k-norm +
// RoPE + KV-cache write, split-K decode attention, causal prefill attention,
// embedding gather, elementwise add / SwiGLU, and the greedy token select /
// store pair.  fp16 storage, fp32 arithmetic throughout.
#include <float.h>

#include <mutex>

#include "common.cuh"

namespace t2c {
int attn_prefill_umma(const void *q, const void *k_cache, const void *v_cache, void *out, const int32_t *positions,
                      int64_t B, int64_t T, int64_t NH, int64_t NK, int64_t cb, int64_t cs, int64_t ch, int64_t qb,
                      int64_t qt, int64_t qh, int64_t ob, int64_t ot, int64_t oh, float scale, cudaStream_t stream,
                      const void *mask, int64_t m_sb, int64_t m_st, int64_t S, bool f32io);
}  // namespace t2c

namespace t2c {
namespace {

__device__ __forceinline__ float4 h4_to_f4(uint2 v) {
    const __half2 a = *reinterpret_cast<const __half2 *>(&v.x);
    const __half2 b = *reinterpret_cast<const __half2 *>(&v.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    return make_float4(fa.x, fa.y, fb.x, fb.y);
}
__device__ __forceinline__ uint2 f4_to_h4(float4 f) {
    const __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
    return make_uint2(*reinterpret_cast<const uint32_t *>(&a), *reinterpret_cast<const uint32_t *>(&b));
}

// ------------------------------------------------------------------ RMSNorm
// One warp per row; lanes stride the row in 8-value chunks.
__global__ void rms_norm_kernel(const __half *__restrict__ x, const float *__restrict__ w, __half *__restrict__ y,
                                int64_t rows, int cols, float eps) {
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    pdl_wait();
    pdl_trigger();
    const __half *xr = x + row * cols;
    float ss = 0.0f;
    for (int c = lane * 4; c < cols; c += 128) {
        const float4 v = h4_to_f4(*reinterpret_cast<const uint2 *>(xr + c));
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / static_cast<float>(cols) + eps);
    __half *yr = y + row * cols;
    for (int c = lane * 4; c < cols; c += 128) {
        float4 v = h4_to_f4(*reinterpret_cast<const uint2 *>(xr + c));
        const float4 g = *reinterpret_cast<const float4 *>(w + c);
        v = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
        *reinterpret_cast<uint2 *>(yr + c) = f4_to_h4(v);
    }
}

// One CTA per row (rows of up to 32 x 256 values): every thread issues its
// 16-byte loads at once, so a row costs one load latency instead of a chain of
// them; the sum of squares meets in shared memory.
constexpr int kRnThreads = 256;
constexpr int kRnVec = 4;  // 16-byte vectors per thread
__global__ void __launch_bounds__(kRnThreads) rms_norm_row_kernel(const __half *__restrict__ x, const float *__restrict__ w,
                                                                  __half *__restrict__ y, int cols, float eps) {
    __shared__ float part[kRnThreads / 32];
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x;
    const int nv = cols / 8;
    pdl_wait();
    pdl_trigger();
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * cols);
    uint4 v[kRnVec];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kRnVec; ++i) {
        const int c = tid + i * kRnThreads;
        v[i] = c < nv ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < kRnVec; ++i) {
        const float4 a = h4_to_f4(make_uint2(v[i].x, v[i].y)), b = h4_to_f4(make_uint2(v[i].z, v[i].w));
        ss += a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) part[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < kRnThreads / 32; ++i) tot += part[i];
    const float inv = rsqrtf(tot / static_cast<float>(cols) + eps);
    uint4 *yr = reinterpret_cast<uint4 *>(y + row * cols);
#pragma unroll
    for (int i = 0; i < kRnVec; ++i) {
        const int c = tid + i * kRnThreads;
        if (c >= nv) continue;
        const float4 g0 = *reinterpret_cast<const float4 *>(w + 8 * c), g1 = *reinterpret_cast<const float4 *>(w + 8 * c + 4);
        float4 a = h4_to_f4(make_uint2(v[i].x, v[i].y)), b = h4_to_f4(make_uint2(v[i].z, v[i].w));
        a = make_float4(a.x * inv * g0.x, a.y * inv * g0.y, a.z * inv * g0.z, a.w * inv * g0.w);
        b = make_float4(b.x * inv * g1.x, b.y * inv * g1.y, b.z * inv * g1.z, b.w * inv * g1.w);
        const uint2 ha = f4_to_h4(a), hb = f4_to_h4(b);
        yr[c] = make_uint4(ha.x, ha.y, hb.x, hb.y);
    }
}

// ------------------------------------------------ q/k norm + RoPE + cache
// One warp per (token, head) vector of D values (D/32 per lane, D <= 256).
// Heads [0, NH): q; [NH, NH+NK): k (norm + rope -> k cache); [NH+NK, NH+2NK): v copy.
// Rotate-half partners d and d +- D/2 sit on lanes l and l ^ 16.
template <int E>
__global__ void qk_norm_rope_cache_kernel(const __half *__restrict__ q_in, const __half *__restrict__ k_in,
                                          const __half *__restrict__ v_in, const float *__restrict__ q_w,
                                          const float *__restrict__ k_w, __half *q_out, __half *__restrict__ k_cache,
                                          __half *__restrict__ v_cache, const int32_t *__restrict__ positions,
                                          int B, int T, int NH, int NK, int64_t cb, int64_t cs, int64_t ch,
                                          const float *__restrict__ inv_freq, float eps) {
    constexpr int D = E * 32;
    const int64_t vec = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int heads = NH + 2 * NK;
    const int64_t total = static_cast<int64_t>(B) * T * heads;
    if (vec >= total) return;
    pdl_wait();
    pdl_trigger();
    const int64_t m = vec / heads;
    const int h = static_cast<int>(vec - m * heads);
    const int b = static_cast<int>(m / T), t = static_cast<int>(m - static_cast<int64_t>(b) * T);
    const int pos = positions[b] + t;
    const int d0 = lane * E;
    float v[E];
    const __half *src;
    if (h < NH) {
        src = q_in + (m * NH + h) * D;
    } else if (h < NH + NK) {
        src = k_in + (m * NK + (h - NH)) * D;
    } else {
        src = v_in + (m * NK + (h - NH - NK)) * D;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = __half2float(src[d0 + e]);
    if (h >= NH + NK) {
        __half *dst = v_cache + b * cb + static_cast<int64_t>(pos) * cs + (h - NH - NK) * ch;
#pragma unroll
        for (int e = 0; e < E; ++e) dst[d0 + e] = __float2half_rn(v[e]);
        return;
    }
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss += v[e] * v[e];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
    const float *w = h < NH ? q_w : k_w;
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = v[e] * inv * w[d0 + e];
    float out[E];
    const bool first_half = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const int i = (d0 + e) & (D / 2 - 1);
        float sn, cs_;
        sincosf(static_cast<float>(pos) * inv_freq[i], &sn, &cs_);
        out[e] = first_half ? v[e] * cs_ - partner * sn : v[e] * cs_ + partner * sn;
    }
    __half *dst;
    if (h < NH) {
        dst = q_out + (m * NH + h) * D;
    } else {
        dst = k_cache + b * cb + static_cast<int64_t>(pos) * cs + (h - NH) * ch;
    }
#pragma unroll
    for (int e = 0; e < E; ++e) dst[d0 + e] = __float2half_rn(out[e]);
}

// ------------------------------------------------------- decode attention
// CTA = 4 warps on (batch b, kv head kh, split sp): cache positions
// [sp * chunk, min((sp+1) * chunk, len_b)).  The G = NH / NK query heads of
// the group share every K/V load.  Scores: lane j of a warp owns position j
// of a 32-position tile (full D-length dot products, q from shared memory);
// values: lanes split D.  Each warp keeps an online softmax (max, sum, acc);
// the four warps merge in shared memory and write either the final output
// (one split) or the split's partial (max, sum, acc) to the workspace.
constexpr int kAttnWarps = 4;
constexpr int kMaxGroup = 8;
constexpr int kMaxSplits = 64;

// Paged caches (PAGED): position p of sequence b lives in physical page
// bt[b * bt_stride + (p >> page_log2)], row (p & (page size - 1)) of it; cb is
// then the page stride (elements) and cs the row stride inside a page.  A
// block-table entry outside [0, num_pages) is reported and read as page 0, so
// every access stays inside the pool.
template <int E, int G, bool PAGED>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(
    const __half *__restrict__ q, const __half *__restrict__ kc, const __half *__restrict__ vc,
    __half *__restrict__ out, const int32_t *__restrict__ positions, int NH, int NK, int64_t cb, int64_t cs,
    int64_t ch, int max_len, int chunk, int splits, float *__restrict__ ws, float scale,
    const int32_t *__restrict__ bt, int64_t bt_stride, int page_log2, int num_pages) {
    constexpr int D = E * 32;
    __shared__ float qs[G][D];
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ float wacc[kAttnWarps][G][D];
    const int sp = blockIdx.x % splits;
    const int kh = (blockIdx.x / splits) % NK;
    const int b = blockIdx.x / (splits * NK);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    // A position outside the cache has no rows to attend to: report it and
    // attend to nothing (every split still writes its record, so the combine
    // never reads stale workspace).
    const int pos_b = positions[b];
    const bool bad_pos = pos_b < 0 || pos_b >= max_len;
    if (bad_pos && sp == 0 && kh == 0 && threadIdx.x == 0) report_device_error(T2C_EINVAL);
    const int len = bad_pos ? 0 : pos_b + 1;
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i - g * D;
        qs[g][d] = __half2float(q[(static_cast<int64_t>(b) * NH + kh * G + g) * D + d]) * scale;
    }
    __syncthreads();
    const int p0 = sp * chunk;
    const int p1 = min(len, p0 + chunk);
    float m_run[G], l_run[G], acc[G][E];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m_run[g] = -FLT_MAX;
        l_run[g] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[g][e] = 0.0f;
    }
    for (int t0 = p0 + warp * 32; t0 < p1; t0 += kAttnWarps * 32) {
        const int pos = t0 + lane;
        const bool valid = pos < p1;
        // element offset of this lane's position row (K and V share it)
        int64_t roff = kh * ch;
        if constexpr (PAGED) {
            if (valid) {
                int page = bt[b * bt_stride + (pos >> page_log2)];
                if (page < 0 || page >= num_pages) {
                    report_device_error(T2C_EINVAL);
                    page = 0;
                }
                roff += static_cast<int64_t>(page) * cb + static_cast<int64_t>(pos & ((1 << page_log2) - 1)) * cs;
            }
        } else {
            roff += b * cb + static_cast<int64_t>(pos) * cs;
        }
        // scores: lane = position; the whole K row is requested at once
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.0f;
        if (valid) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(kc + roff);
            uint4 kraw[D / 8];
#pragma unroll
            for (int c = 0; c < D / 8; ++c) kraw[c] = kr[c];
#pragma unroll
            for (int c = 0; c < D / 8; ++c) {
                const float4 lo = h4_to_f4(make_uint2(kraw[c].x, kraw[c].y));
                const float4 hi = h4_to_f4(make_uint2(kraw[c].z, kraw[c].w));
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][c * 8]);
                    const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][c * 8 + 4]);
                    s[g] += lo.x * qa.x + lo.y * qa.y + lo.z * qa.z + lo.w * qa.w + hi.x * qb.x + hi.y * qb.y +
                            hi.z * qb.z + hi.w * qb.w;
                }
            }
        }
        // values: lane = E dims; the 32 V fragments of the tile are requested at once
        const int n_valid = min(32, p1 - t0);
        float vf[32][E];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const int64_t rj = __shfl_sync(0xffffffffu, roff, j);
            if (j < n_valid) {
                const __half *vr = vc + rj + lane * E;
                if constexpr (E == 4) {
                    const float4 f = h4_to_f4(*reinterpret_cast<const uint2 *>(vr));
                    vf[j][0] = f.x;
                    vf[j][1] = f.y;
                    vf[j][2] = f.z;
                    vf[j][3] = f.w;
                } else {
#pragma unroll
                    for (int e = 0; e < E; ++e) vf[j][e] = __half2float(vr[e]);
                }
            } else {
#pragma unroll
                for (int e = 0; e < E; ++e) vf[j][e] = 0.0f;
            }
        }
        float p[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float sv = valid ? s[g] : -FLT_MAX;
            const float tile_max = warp_max(sv);
            const float m_new = fmaxf(m_run[g], tile_max);
            const float corr = __expf(m_run[g] - m_new);
            p[g] = valid ? __expf(sv - m_new) : 0.0f;
            l_run[g] = l_run[g] * corr + warp_sum(p[g]);
            m_run[g] = m_new;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[g][e] *= corr;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pj = __shfl_sync(0xffffffffu, p[g], j);
#pragma unroll
                for (int e = 0; e < E; ++e) acc[g][e] = fmaf(pj, vf[j][e], acc[g][e]);
            }
        }
    }
    // merge the warps
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp][g] = m_run[g];
            wl[warp][g] = l_run[g];
        }
#pragma unroll
        for (int e = 0; e < E; ++e) wacc[warp][g][lane * E + e] = acc[g][e];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
        const int g = i / D, d = i - g * D;
        float mx = -FLT_MAX;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w][g]);
        float l = 0.0f, a = 0.0f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = wm[w][g] == -FLT_MAX ? 0.0f : __expf(wm[w][g] - mx);
            l += wl[w][g] * f;
            a += wacc[w][g][d] * f;
        }
        const int h = kh * G + g;
        if (splits == 1) {
            out[(static_cast<int64_t>(b) * NH + h) * D + d] = __float2half_rn(l > 0.0f ? a / l : 0.0f);
        } else {
            float *rec = ws + ((static_cast<int64_t>(b) * NH + h) * splits + sp) * (D + 2);
            rec[2 + d] = a;
            if (d == 0) {
                rec[0] = mx;
                rec[1] = l;
            }
        }
    }
}

template <int E>
__global__ void attn_combine_kernel(const float *__restrict__ ws, __half *__restrict__ out, int B, int NH, int splits) {
    constexpr int D = E * 32;
    __shared__ float wts[kMaxSplits];
    __shared__ float total;
    const int64_t bh = blockIdx.x;  // b * NH + h
    if (bh >= static_cast<int64_t>(B) * NH) return;
    pdl_wait();
    pdl_trigger();
    const float *rec = ws + bh * splits * (D + 2);
    if (threadIdx.x < 32) {
        // split weights exp(m_s - max) and the combined softmax sum
        float m[kMaxSplits / 32], l[kMaxSplits / 32];
        float mx = -FLT_MAX;
#pragma unroll
        for (int i = 0; i < kMaxSplits / 32; ++i) {
            const int sp = threadIdx.x + 32 * i;
            m[i] = sp < splits ? rec[sp * (D + 2)] : -FLT_MAX;
            l[i] = sp < splits ? rec[sp * (D + 2) + 1] : 0.0f;
            mx = fmaxf(mx, m[i]);
        }
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxSplits / 32; ++i) {
            const int sp = threadIdx.x + 32 * i;
            const float w = m[i] == -FLT_MAX ? 0.0f : __expf(m[i] - mx);
            if (sp < splits) wts[sp] = w;
            sum += w * l[i];
        }
        sum = warp_sum(sum);
        if (threadIdx.x == 0) total = sum;
    }
    __syncthreads();
    const float inv = total > 0.0f ? 1.0f / total : 0.0f;
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        int sp = 0;
        for (; sp + 4 <= splits; sp += 4) {
            a0 = fmaf(wts[sp], rec[sp * (D + 2) + 2 + d], a0);
            a1 = fmaf(wts[sp + 1], rec[(sp + 1) * (D + 2) + 2 + d], a1);
            a2 = fmaf(wts[sp + 2], rec[(sp + 2) * (D + 2) + 2 + d], a2);
            a3 = fmaf(wts[sp + 3], rec[(sp + 3) * (D + 2) + 2 + d], a3);
        }
        for (; sp < splits; ++sp) a0 = fmaf(wts[sp], rec[sp * (D + 2) + 2 + d], a0);
        out[bh * D + d] = __float2half_rn((a0 + a1 + a2 + a3) * inv);
    }
}

// Paged KV write: rows src[b * src_sb + t * src_st + h * D ..] (T new tokens per
// sequence, NK heads) go to position positions[b] + t of sequence b: page
// bt[b * bt_stride + (pos >> page_log2)], row pos & (P - 1).  One thread per
// 16-byte piece of a row.
__global__ void kv_write_paged_kernel(__half *__restrict__ pages, const __half *__restrict__ src, int64_t src_sb,
                                      int64_t src_st, const int32_t *__restrict__ positions,
                                      const int32_t *__restrict__ bt, int64_t bt_stride, int page_log2,
                                      int64_t pstride, int64_t rstride, int64_t hstride, int B, int T, int NK, int D,
                                      int max_len, int num_pages) {
    pdl_wait();
    pdl_trigger();
    const int pieces = D / 8;
    const int64_t total = static_cast<int64_t>(B) * T * NK * pieces;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int piece = static_cast<int>(i % pieces);
        const int h = static_cast<int>((i / pieces) % NK);
        const int t = static_cast<int>((i / (static_cast<int64_t>(pieces) * NK)) % T);
        const int b = static_cast<int>(i / (static_cast<int64_t>(pieces) * NK * T));
        const int pos = positions[b] + t;
        if (pos < 0 || pos >= max_len) {  // no page row for it: report, write nothing
            if (piece == 0 && h == 0) report_device_error(T2C_EINVAL);
            continue;
        }
        const int64_t page = bt[b * bt_stride + (pos >> page_log2)];
        if (page < 0 || page >= num_pages) {  // not a page of the pool: report, write nothing
            report_device_error(T2C_EINVAL);
            continue;
        }
        const uint4 v = *reinterpret_cast<const uint4 *>(src + b * src_sb + t * src_st + h * D + 8 * piece);
        *reinterpret_cast<uint4 *>(pages + page * pstride + static_cast<int64_t>(pos & ((1 << page_log2) - 1)) * rstride +
                                   h * hstride + 8 * piece) = v;
    }
}

// ------------------------------------------- fused decode attention (T = 1)
// One launch per layer for a decode step: q/k RMSNorm + RoPE, KV-cache write
// of the new position, split-K attention and the split combine.
// CTA = G warps on (batch b, kv head kh, split sp); warp g owns query head
// kh*G + g over the CTA's cache positions [sp * chunk, min((sp+1) * chunk, len)),
// chunk = ceil(len / splits) from the device-side length.  The G warps read
// the same K / V rows (L1 shares them) and never wait for each other: no
// CTA barrier anywhere.  Cache rows of earlier steps do not depend on the
// preceding kernel, so the first K / V tile is requested before
// griddepcontrol.wait; the raw q / k / v of this step (from the preceding QKV
// matvec) are read after it.  In the CTA whose range holds the new position,
// every warp computes the new k (normed, rotated) itself and warp 0 writes
// k / v into the cache.  Splits leave (max, sum, acc) partials per head; the
// last warp to arrive for a head (arrival counter) combines them and resets
// the counter to zero.  Scores use base-2 exponentials with q pre-scaled by
// log2(e) / sqrt(D).  Lane j scores position j of a 32-position tile (whole
// K row per lane, q broadcast from shared memory); lanes split D for P V.
__device__ __forceinline__ void norm_rope_lane(const uint2 raw, const float *__restrict__ w,
                                               const float *__restrict__ inv_freq, int pos, float eps, int lane,
                                               float r[4]) {
    constexpr int D = 128;
    const float4 f = h4_to_f4(raw);
    float v[4] = {f.x, f.y, f.z, f.w};
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = v[e] * inv * w[lane * 4 + e];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        float sn, cs_;
        sincosf(static_cast<float>(pos) * inv_freq[(lane * 4 + e) & (D / 2 - 1)], &sn, &cs_);
        r[e] = lane < 16 ? v[e] * cs_ - partner * sn : v[e] * cs_ + partner * sn;
    }
}

template <int G>
__global__ void __launch_bounds__(G * 32) attn_decode_fused_kernel(
    const __half *__restrict__ q_in, const __half *__restrict__ k_in, const __half *__restrict__ v_in, int64_t q_sb,
    int64_t k_sb, int64_t v_sb, const float *__restrict__ q_w, const float *__restrict__ k_w,
    const float *__restrict__ inv_freq, float eps, __half *kc, __half *vc, int64_t cb, int64_t cs, int64_t ch,
    __half *__restrict__ out, int64_t o_sb, const int32_t *__restrict__ positions, int NK, int max_len, int splits,
    float *__restrict__ ws, int *__restrict__ counters, float qscale) {
    constexpr int D = 128, E = 4;
    __shared__ __align__(16) float qs[G][D];
    __shared__ __align__(16) float ps[G][32];
    __shared__ __align__(16) __half knew[G][D];
    __shared__ float cw[G][kMaxSplits];
    const int sp = blockIdx.x % splits;
    const int kh = (blockIdx.x / splits) % NK;
    const int b = blockIdx.x / (splits * NK);
    const int g = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int NH = NK * G;
    const int h = kh * G + g;
    const int pos = positions[b];
    if (pos < 0 || pos >= max_len) {  // no cache row to write: report, touch nothing
        pdl_wait();
        pdl_trigger();
        if (threadIdx.x == 0) report_device_error(T2C_EINVAL);
        return;
    }
    const int len = pos + 1;
    const int chunk = (len + splits - 1) / splits;
    const int p0 = sp * chunk, p1 = min(len, p0 + chunk);
    const bool owner = p0 <= pos && pos < p1;
    const __half *kbase = kc + b * cb + kh * ch;
    const __half *vbase = vc + b * cb + kh * ch;

    int t0 = p0;
    uint4 kraw[D / 8];
    uint2 vraw[32];
    auto load_tile = [&](int base) {
        const int pk = base + lane;
        if (pk < p1) {
            const uint4 *kr = reinterpret_cast<const uint4 *>(kbase + static_cast<int64_t>(pk) * cs);
#pragma unroll
            for (int c = 0; c < D / 8; ++c) kraw[c] = kr[c];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (base + j < p1)
                vraw[j] = *reinterpret_cast<const uint2 *>(vbase + static_cast<int64_t>(base + j) * cs + lane * E);
    };
    if (t0 < p1) load_tile(t0);

    pdl_wait();
    pdl_trigger();
    {
        float r[4];
        norm_rope_lane(*reinterpret_cast<const uint2 *>(q_in + b * q_sb + static_cast<int64_t>(h) * D + lane * E), q_w,
                       inv_freq, pos, eps, lane, r);
#pragma unroll
        for (int e = 0; e < E; ++e) qs[g][lane * E + e] = __half2float(__float2half_rn(r[e])) * qscale;
    }
    uint2 vnew = make_uint2(0u, 0u);
    if (owner) {
        float r[4];
        norm_rope_lane(*reinterpret_cast<const uint2 *>(k_in + b * k_sb + static_cast<int64_t>(kh) * D + lane * E), k_w,
                       inv_freq, pos, eps, lane, r);
        const uint2 kh4 = f4_to_h4(make_float4(r[0], r[1], r[2], r[3]));
        vnew = *reinterpret_cast<const uint2 *>(v_in + b * v_sb + static_cast<int64_t>(kh) * D + lane * E);
        *reinterpret_cast<uint2 *>(&knew[g][lane * E]) = kh4;
        if (g == 0) {
            *reinterpret_cast<uint2 *>(kc + b * cb + static_cast<int64_t>(pos) * cs + kh * ch + lane * E) = kh4;
            *reinterpret_cast<uint2 *>(vc + b * cb + static_cast<int64_t>(pos) * cs + kh * ch + lane * E) = vnew;
        }
    }
    __syncwarp();

    float m_run = -FLT_MAX, l_run = 0.0f;
    float acc[E] = {0.0f, 0.0f, 0.0f, 0.0f};
    while (t0 < p1) {
        const int pk = t0 + lane;
        const bool valid = pk < p1;
        if (owner && pk == pos) {
#pragma unroll
            for (int c = 0; c < D / 8; ++c) kraw[c] = reinterpret_cast<const uint4 *>(knew[g])[c];
        }
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
            const float4 lo = h4_to_f4(make_uint2(kraw[c].x, kraw[c].y));
            const float4 hi = h4_to_f4(make_uint2(kraw[c].z, kraw[c].w));
            const float4 qa = *reinterpret_cast<const float4 *>(&qs[g][c * 8]);
            const float4 qb = *reinterpret_cast<const float4 *>(&qs[g][c * 8 + 4]);
            s0 = fmaf(lo.x, qa.x, s0);
            s1 = fmaf(lo.y, qa.y, s1);
            s0 = fmaf(lo.z, qa.z, s0);
            s1 = fmaf(lo.w, qa.w, s1);
            s0 = fmaf(hi.x, qb.x, s0);
            s1 = fmaf(hi.y, qb.y, s1);
            s0 = fmaf(hi.z, qb.z, s0);
            s1 = fmaf(hi.w, qb.w, s1);
        }
        const float sv = valid ? s0 + s1 : -FLT_MAX;
        const float m_new = fmaxf(m_run, warp_max(sv));
        const float corr = exp2f(m_run - m_new);
        const float p = valid ? exp2f(sv - m_new) : 0.0f;
        l_run = l_run * corr + p;  // per-lane partial sums, reduced once at the end
        m_run = m_new;
        ps[g][lane] = p;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] *= corr;
        __syncwarp();
        const int n_valid = min(32, p1 - t0);
#pragma unroll
        for (int j4 = 0; j4 < 32; j4 += 4) {
            const float4 pj = *reinterpret_cast<const float4 *>(&ps[g][j4]);
            const float pv[4] = {pj.x, pj.y, pj.z, pj.w};
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int j = j4 + jj;
                if (j < n_valid) {
                    const uint2 raw = owner && t0 + j == pos ? vnew : vraw[j];
                    const float4 vf = h4_to_f4(raw);
                    acc[0] = fmaf(pv[jj], vf.x, acc[0]);
                    acc[1] = fmaf(pv[jj], vf.y, acc[1]);
                    acc[2] = fmaf(pv[jj], vf.z, acc[2]);
                    acc[3] = fmaf(pv[jj], vf.w, acc[3]);
                }
            }
        }
        __syncwarp();
        t0 += 32;
        if (t0 < p1) load_tile(t0);
    }
    const float l_tot = warp_sum(l_run);
    __half *orow = out + b * o_sb + static_cast<int64_t>(h) * D + lane * E;
    if (splits == 1) {
        const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
        *reinterpret_cast<uint2 *>(orow) = f4_to_h4(make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv));
        return;
    }
    // partial of this split for head h; the last warp to arrive combines
    float *head_base = ws + (static_cast<int64_t>(b) * NH + h) * splits * (D + 4);
    float *rec = head_base + static_cast<int64_t>(sp) * (D + 4);
    *reinterpret_cast<float4 *>(rec + 4 + lane * E) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (lane == 0) *reinterpret_cast<float2 *>(rec) = make_float2(m_run, l_tot);
    __threadfence();
    __syncwarp();
    int ticket = 0;
    if (lane == 0) ticket = atomicAdd(&counters[b * NH + h], 1);
    ticket = __shfl_sync(0xffffffffu, ticket, 0);
    if (ticket != splits - 1) return;
    __threadfence();
    float mx = -FLT_MAX;
    for (int s2 = lane; s2 < splits; s2 += 32) mx = fmaxf(mx, __ldcg(head_base + static_cast<int64_t>(s2) * (D + 4)));
    mx = warp_max(mx);
    float lsum = 0.0f;
    for (int s2 = lane; s2 < splits; s2 += 32) {
        const float2 ml = __ldcg(reinterpret_cast<const float2 *>(head_base + static_cast<int64_t>(s2) * (D + 4)));
        const float w = ml.x == -FLT_MAX ? 0.0f : exp2f(ml.x - mx);
        cw[g][s2] = w;
        lsum = fmaf(w, ml.y, lsum);
    }
    lsum = warp_sum(lsum);
    __syncwarp();
    float4 a = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float *col = head_base + 4 + lane * E;
    int s2 = 0;
    for (; s2 + 8 <= splits; s2 += 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] = __ldcg(reinterpret_cast<const float4 *>(col + static_cast<int64_t>(s2 + u) * (D + 4)));
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const float w = cw[g][s2 + u];
            a.x = fmaf(w, v[u].x, a.x);
            a.y = fmaf(w, v[u].y, a.y);
            a.z = fmaf(w, v[u].z, a.z);
            a.w = fmaf(w, v[u].w, a.w);
        }
    }
    for (; s2 < splits; ++s2) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(col + static_cast<int64_t>(s2) * (D + 4)));
        const float w = cw[g][s2];
        a.x = fmaf(w, v.x, a.x);
        a.y = fmaf(w, v.y, a.y);
        a.z = fmaf(w, v.z, a.z);
        a.w = fmaf(w, v.w, a.w);
    }
    const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
    *reinterpret_cast<uint2 *>(orow) = f4_to_h4(make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv));
    if (lane == 0) counters[b * NH + h] = 0;
}

// ------------------------------------------ cluster decode attention (T = 1)
// The same work as attn_decode_fused_kernel for splits <= 8, on tensor cores:
// the `splits` CTAs of one (batch b, kv head kh) form a thread-block cluster.
// A CTA owns the cache positions [p0, p1) of its split and streams them as
// 32-position tiles, one shared-memory stage per warp: warp w takes tiles
// w, w + 8, ... and loads them itself (cp.async; its first tile, the RoPE
// angles and the norm weights are requested before griddepcontrol.wait), so
// the tile loop has no CTA barrier and up to 256 positions per CTA (2048 per
// cluster) take one pass.  For its tile a warp computes the scores of all G query heads of the KV head with
// mma.m16n8k16 (positions as rows, heads as the 8 columns: S^T = K Q^T), runs
// an online softmax per head, and accumulates O^T += V^T P^T (dims as rows;
// P split into fp16 high and low parts so the product keeps fp32 accuracy).
// The warps' states merge through shared memory into the CTA's partial
// (max, sum, acc) per head, which goes by distributed-shared-memory stores to
// the CTA that combines that head (head hh -> cluster rank hh % splits); one
// cluster barrier (release / acquire) then lets the combining CTAs finish.
// No workspace, no atomics, no global round trip for the combine.
constexpr int kCaTile = 32;
constexpr int kCaWarps = 8;
constexpr int kCaStages = kCaWarps;  // one stage per warp
constexpr int kCaMaxSplits = 8;
constexpr int kCaRow = 136;  // halves per K / V row in shared memory (272 B: conflict-free ldmatrix rows)
constexpr int kCaStageBytes = 2 * kCaTile * kCaRow * 2;
static_assert(kCaStageBytes % 16 == 0 && kCaStageBytes >= 8 * 128 * 4, "a stage holds a warp's [8 heads][128] fp32 partial");
constexpr int kCaSmem = kCaStages * kCaStageBytes;
constexpr int kCaRecv = 132;  // floats per received partial: acc[128], max, sum

__device__ __forceinline__ void ca_cp16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void ca_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ca_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t ca_cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void ca_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }
__device__ __forceinline__ void ca_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void ca_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void ca_st_remote(float *local, uint32_t rank, float v) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(remote), "f"(v) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t r[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
// not volatile: a pure register operation, so the compiler may interleave independent accumulator chains
__device__ __forceinline__ void mma_f16_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// RMSNorm (weights w) + RoPE (cos / sin of this lane's 4 dims) of one 128-value head row.
__device__ __forceinline__ void norm_rope_pre(const uint2 raw, const float w[4], const float c[4], const float sn[4],
                                              float eps, int lane, float r[4]) {
    const float4 f = h4_to_f4(raw);
    float v[4] = {f.x, f.y, f.z, f.w};
    const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
    const float inv = rsqrtf(ss / 128.0f + eps);
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = v[e] * inv * w[e];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        r[e] = lane < 16 ? v[e] * c[e] - partner * sn[e] : v[e] * c[e] + partner * sn[e];
    }
}

template <int G>
__global__ void __launch_bounds__(kCaWarps * 32) attn_decode_cluster_kernel(
    const __half *__restrict__ q_in, const __half *__restrict__ k_in, const __half *__restrict__ v_in, int64_t q_sb,
    int64_t k_sb, int64_t v_sb, const float *__restrict__ q_w, const float *__restrict__ k_w,
    const float *__restrict__ inv_freq, float eps, __half *kc, __half *vc, int64_t cb, int64_t cs, int64_t ch,
    __half *__restrict__ out, int64_t o_sb, const int32_t *__restrict__ positions, int NK, int max_len, int splits,
    float qscale) {
    static_assert(G <= 8, "at most 8 query heads per KV head (the mma N dimension)");
    constexpr int D = 128, E = 4, NT = kCaWarps * 32;
    extern __shared__ __align__(128) uint8_t ca_smem[];
    __shared__ __align__(16) __half qs[8][D];                 // fp16 q rows (heads >= G stay zero)
    __shared__ __align__(16) __half pst[kCaWarps][2][8][40];  // P^T (hi, lo) per warp: [head][position], padded rows
    __shared__ float wml[kCaWarps][8][2];                     // per-warp (max, sum)
    __shared__ __align__(16) __half kvnew[2][D];              // the new position's k / v row (owner CTA)
    __shared__ __align__(16) float recv[16][kCaRecv];         // partials received for the heads this CTA combines
    const int sp = static_cast<int>(ca_cluster_rank());
    const int kh = (blockIdx.x / splits) % NK;
    const int b = blockIdx.x / (splits * NK);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int pos = positions[b];
    if (pos < 0 || pos >= max_len) {  // no cache row to write: report, touch nothing (uniform over the cluster)
        pdl_wait();
        pdl_trigger();
        if (threadIdx.x == 0) report_device_error(T2C_EINVAL);
        return;
    }
    if (splits > 1) ca_arrive_relaxed();  // every CTA of the cluster has started before any remote store
    const int len = pos + 1;
    const int chunk = (len + splits - 1) / splits;
    const int p0 = min(len, sp * chunk), p1 = min(len, p0 + chunk);
    const int ntiles = (p1 - p0 + kCaTile - 1) / kCaTile;
    const bool owner = p0 <= pos && pos < p1;
    const __half *kbase = kc + b * cb + kh * ch;
    const __half *vbase = vc + b * cb + kh * ch;
    // this warp's tile `tile` into its own stage (rows past p1 zero-filled), by its own 32 lanes
    __half *const kst = reinterpret_cast<__half *>(ca_smem + w * kCaStageBytes);
    __half *const vst = kst + kCaTile * kCaRow;
    auto issue = [&](int tile) {
        const int t0 = p0 + tile * kCaTile;
#pragma unroll 4
        for (int i = lane; i < kCaTile * 16; i += 32) {
            const int r = i >> 4, c = i & 15;
            const bool in = t0 + r < p1;
            const int64_t src = (in ? static_cast<int64_t>(t0 + r) * cs : 0) + c * 8;
            ca_cp16(kst + r * kCaRow + c * 8, kbase + src, in ? 16u : 0u);
            ca_cp16(vst + r * kCaRow + c * 8, vbase + src, in ? 16u : 0u);
        }
        ca_commit();
    };
    // norm weights and RoPE frequencies are requested first but used only after the wait: the
    // (possibly long, HBM-queued) latency of these loads does not delay reaching the wait
    float fr[E], qw[E], kw[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        fr[e] = inv_freq[(lane * E + e) & (D / 2 - 1)];
        qw[e] = q_w[lane * E + e];
        kw[e] = k_w[lane * E + e];
    }
    if (w < ntiles) issue(w);
    for (int i = threadIdx.x; i < 8 * D / 2; i += NT) reinterpret_cast<uint32_t *>(qs)[i] = 0u;
    __syncthreads();

    pdl_wait();
    pdl_trigger();
    float cw[E], sw[E];
#pragma unroll
    for (int e = 0; e < E; ++e) sincosf(static_cast<float>(pos) * fr[e], &sw[e], &cw[e]);
    for (int hh = w; hh < G; hh += kCaWarps) {
        float r[4];
        norm_rope_pre(*reinterpret_cast<const uint2 *>(q_in + b * q_sb + static_cast<int64_t>(kh * G + hh) * D + lane * E),
                      qw, cw, sw, eps, lane, r);
        *reinterpret_cast<uint2 *>(&qs[hh][lane * E]) = f4_to_h4(make_float4(r[0], r[1], r[2], r[3]));
    }
    if (owner && w == kCaWarps - 1) {  // the last warp: G <= 4 leaves it free of query rows
        float r[4];
        norm_rope_pre(*reinterpret_cast<const uint2 *>(k_in + b * k_sb + static_cast<int64_t>(kh) * D + lane * E), kw, cw,
                      sw, eps, lane, r);
        const uint2 knew = f4_to_h4(make_float4(r[0], r[1], r[2], r[3]));
        const uint2 vnew = *reinterpret_cast<const uint2 *>(v_in + b * v_sb + static_cast<int64_t>(kh) * D + lane * E);
        *reinterpret_cast<uint2 *>(kc + b * cb + static_cast<int64_t>(pos) * cs + kh * ch + lane * E) = knew;
        *reinterpret_cast<uint2 *>(vc + b * cb + static_cast<int64_t>(pos) * cs + kh * ch + lane * E) = vnew;
        *reinterpret_cast<uint2 *>(&kvnew[0][lane * E]) = knew;
        *reinterpret_cast<uint2 *>(&kvnew[1][lane * E]) = vnew;
    }
    __syncthreads();  // q rows (and the new k / v row) complete
    // B fragments of Q^T (k = dim, n = head) for the 8 k-steps of 16 dims
    uint32_t qb[8][2];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
        qb[ks][0] = *reinterpret_cast<const uint32_t *>(&qs[g][16 * ks + 2 * t]);
        qb[ks][1] = *reinterpret_cast<const uint32_t *>(&qs[g][16 * ks + 2 * t + 8]);
    }

    // per lane: heads 2t, 2t+1; acc rows dims 16m + g, 16m + g + 8
    float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.0f, 0.0f};
    float o[8][4];
#pragma unroll
    for (int m = 0; m < 8; ++m) o[m][0] = o[m][1] = o[m][2] = o[m][3] = 0.0f;
    const int new_tile = owner ? (pos - p0) / kCaTile : -1;
#pragma unroll 1
    for (int tile = w; tile < ntiles; tile += kCaWarps) {
        ca_wait<0>();
        __syncwarp();  // every lane's copies of this tile have landed
        if (tile == new_tile) {
            // the new position's row may have been read before this kernel wrote it
            const int r = pos - p0 - new_tile * kCaTile;
            *reinterpret_cast<uint2 *>(kst + r * kCaRow + lane * E) = *reinterpret_cast<const uint2 *>(&kvnew[0][lane * E]);
            *reinterpret_cast<uint2 *>(vst + r * kCaRow + lane * E) = *reinterpret_cast<const uint2 *>(&kvnew[1][lane * E]);
            __syncwarp();
        }
        {
            const __half *ks = kst;
            const __half *vs = vst;
            const int t0 = p0 + tile * kCaTile;
            // S^T = K Q^T: rows = 32 positions (2 m-tiles), columns = 8 heads; four independent
            // accumulator chains (m-tile x even / odd k-step), summed at the end
            float s[2][4], s2[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[mt][e] = s2[mt][e] = 0.0f;
#pragma unroll
            for (int ks8 = 0; ks8 < 8; ++ks8) {
                uint32_t a[2][4];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
                    ldsm_x4(a[mt], ks + (16 * mt + (lane & 15)) * kCaRow + 16 * ks8 + 8 * (lane >> 4));
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) mma_f16_16816((ks8 & 1) ? s2[mt] : s[mt], a[mt], qb[ks8][0], qb[ks8][1]);
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) s[mt][e] += s2[mt][e];
            // online softmax per head (columns 2t, 2t+1); rows g, g+8 of each m-tile
            float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int p = t0 + 16 * mt + g + 8 * (e >> 1);
                    s[mt][e] = p < p1 ? s[mt][e] * qscale : -FLT_MAX;
                    mx[e & 1] = fmaxf(mx[e & 1], s[mt][e]);
                }
            float corr[2];
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 4));
                mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 8));
                mx[c] = fmaxf(mx[c], __shfl_xor_sync(0xffffffffu, mx[c], 16));
                const float m_new = fmaxf(m_run[c], mx[c]);
                corr[c] = exp2f(m_run[c] - m_new);
                m_run[c] = m_new;
                l_run[c] *= corr[c];
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int c = e & 1;
                    const float p = s[mt][e] == -FLT_MAX ? 0.0f : exp2f(s[mt][e] - m_run[c]);
                    l_run[c] += p;
                    const __half ph = __float2half_rn(p);
                    const __half pl = __float2half_rn(p - __half2float(ph));
                    const int col = 16 * mt + g + 8 * (e >> 1);
                    pst[w][0][2 * t + c][col] = ph;
                    pst[w][1][2 * t + c][col] = pl;
                }
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                o[m][0] *= corr[0];
                o[m][1] *= corr[1];
                o[m][2] *= corr[0];
                o[m][3] *= corr[1];
            }
            __syncwarp();
            // O^T += V^T P^T: rows = 128 dims (8 m-tiles), k = 32 positions (2 k-steps), columns = heads
#pragma unroll
            for (int kk = 0; kk < 2; ++kk) {
                const uint32_t bh0 = *reinterpret_cast<const uint32_t *>(&pst[w][0][g][16 * kk + 2 * t]);
                const uint32_t bh1 = *reinterpret_cast<const uint32_t *>(&pst[w][0][g][16 * kk + 2 * t + 8]);
                const uint32_t bl0 = *reinterpret_cast<const uint32_t *>(&pst[w][1][g][16 * kk + 2 * t]);
                const uint32_t bl1 = *reinterpret_cast<const uint32_t *>(&pst[w][1][g][16 * kk + 2 * t + 8]);
                const __half *vrow = vs + (16 * kk + (lane & 7) + 8 * (lane >> 4)) * kCaRow + 8 * ((lane >> 3) & 1);
                // high parts over the 8 m-tiles, then the low parts: no back-to-back dependent pair
                uint32_t a[8][4];
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    ldsm_x4_t(a[m], vrow + 16 * m);
                    mma_f16_16816(o[m], a[m], bh0, bh1);
                }
#pragma unroll
                for (int m = 0; m < 8; ++m) mma_f16_16816(o[m], a[m], bl0, bl1);
            }
            __syncwarp();  // the stage is consumed before it is refilled
        }
        if (tile + kCaWarps < ntiles) issue(tile + kCaWarps);
    }
    // merge the warps' states per head: (max, sum, acc)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 4);
        l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 8);
        l_run[c] += __shfl_xor_sync(0xffffffffu, l_run[c], 16);
    }
    if (g == 0) {
        wml[w][2 * t][0] = m_run[0];
        wml[w][2 * t][1] = l_run[0];
        wml[w][2 * t + 1][0] = m_run[1];
        wml[w][2 * t + 1][1] = l_run[1];
    }
    // per-warp acc [8 heads][D] in the warp's own (consumed) stage
    auto wo = [&](int v) { return reinterpret_cast<float(*)[D]>(ca_smem + v * kCaStageBytes); };
    float(*const mine)[D] = wo(w);
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        mine[2 * t][16 * m + g] = o[m][0];
        mine[2 * t + 1][16 * m + g] = o[m][1];
        mine[2 * t][16 * m + g + 8] = o[m][2];
        mine[2 * t + 1][16 * m + g + 8] = o[m][3];
    }
    __syncthreads();
    if (splits > 1) ca_wait_acquire();  // (start barrier) every CTA of the cluster runs
    static_assert(NT == 2 * D, "two threads per dim: the halves take alternate heads");
    const int d = threadIdx.x & (D - 1), half = threadIdx.x >> 7;
    constexpr int GH = (G + 1) / 2;  // heads per half
    // every head's CTA partial from local shared memory first, then the remote stores in one burst
    // (no local load waits behind a remote store)
    float hmx[GH], hls[GH], ha[GH];
#pragma unroll
    for (int j = 0; j < GH; ++j) {
        const int hh = 2 * j + half;
        hmx[j] = -FLT_MAX;
        hls[j] = ha[j] = 0.0f;
        if (hh < G) {
            float mx = -FLT_MAX;
#pragma unroll
            for (int v = 0; v < kCaWarps; ++v) mx = fmaxf(mx, wml[v][hh][0]);
            float lsum = 0.0f, a = 0.0f;
#pragma unroll
            for (int v = 0; v < kCaWarps; ++v) {
                const float f = wml[v][hh][0] == -FLT_MAX ? 0.0f : exp2f(wml[v][hh][0] - mx);
                lsum = fmaf(f, wml[v][hh][1], lsum);
                a = fmaf(f, wo(v)[hh][d], a);
            }
            hmx[j] = mx;
            hls[j] = lsum;
            ha[j] = a;
        }
    }
    if (splits == 1) {
#pragma unroll
        for (int j = 0; j < GH; ++j) {
            const int hh = 2 * j + half;
            if (hh < G) {
                const float inv = hls[j] > 0.0f ? 1.0f / hls[j] : 0.0f;
                out[b * o_sb + static_cast<int64_t>(kh * G + hh) * D + d] = __float2half_rn(ha[j] * inv);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < GH; ++j) {
        const int hh = 2 * j + half;
        if (hh < G) {
            // partial of head hh -> CTA hh % splits, slot (hh / splits) * splits + sp
            float *dst = &recv[(hh / splits) * splits + sp][0];
            const uint32_t rank = static_cast<uint32_t>(hh % splits);
            ca_st_remote(dst + d, rank, ha[j]);
            if (d == 0) {
                ca_st_remote(dst + 128, rank, hmx[j]);
                ca_st_remote(dst + 129, rank, hls[j]);
            }
        }
    }
    ca_arrive_release();
    ca_wait_acquire();  // every partial has arrived
    for (int hh = sp + half * splits; hh < G; hh += 2 * splits) {
        const float *src = &recv[(hh / splits) * splits][0];
        float mx = -FLT_MAX;
        for (int q = 0; q < splits; ++q) mx = fmaxf(mx, src[q * kCaRecv + 128]);
        float lsum = 0.0f, a = 0.0f;
        for (int q = 0; q < splits; ++q) {
            const float m = src[q * kCaRecv + 128];
            const float f = m == -FLT_MAX ? 0.0f : exp2f(m - mx);
            lsum = fmaf(f, src[q * kCaRecv + 129], lsum);
            a = fmaf(f, src[q * kCaRecv + d], a);
        }
        const float inv = lsum > 0.0f ? 1.0f / lsum : 0.0f;
        out[b * o_sb + static_cast<int64_t>(kh * G + hh) * D + d] = __float2half_rn(a * inv);
    }
}

// ------------------------------------------------------ prefill attention
// CTA = 4 warps on (b, head h, 16-query tile).  Keys are processed in tiles
// of 32: warp w owns queries 4w..4w+3 of the tile; lane j scores key j of the
// key tile against those queries (q from shared memory), then lanes split D
// to accumulate P V with the probabilities broadcast by shuffles.
constexpr int kPfQ = 16;

template <int E>
__global__ void __launch_bounds__(128) attn_prefill_kernel(const __half *__restrict__ q, const __half *__restrict__ kc,
                                                           const __half *__restrict__ vc, __half *__restrict__ out,
                                                           const int32_t *__restrict__ positions, int T, int NH,
                                                           int NK, int64_t cb, int64_t cs, int64_t ch, int64_t q_sb,
                                                           int64_t q_st, int64_t q_sh, int64_t o_sb, int64_t o_st,
                                                           int64_t o_sh, float scale) {
    constexpr int D = E * 32;
    constexpr int QW = kPfQ / 4;  // queries per warp
    __shared__ float qs[kPfQ][D];
    const int qtiles = (T + kPfQ - 1) / kPfQ;
    const int qt = blockIdx.x % qtiles;
    const int h = (blockIdx.x / qtiles) % NH;
    const int b = blockIdx.x / (qtiles * NH);
    const int kh = h / (NH / NK);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_trigger();
    const int base = positions[b];
    for (int i = threadIdx.x; i < kPfQ * D; i += blockDim.x) {
        const int qi = i / D, d = i - qi * D;
        const int t = qt * kPfQ + qi;
        qs[qi][d] = t < T ? __half2float(q[b * q_sb + t * q_st + h * q_sh + d]) * scale : 0.0f;
    }
    __syncthreads();
    float m_run[QW], l_run[QW], acc[QW][E];
#pragma unroll
    for (int i = 0; i < QW; ++i) {
        m_run[i] = -FLT_MAX;
        l_run[i] = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[i][e] = 0.0f;
    }
    const int q_first = qt * kPfQ + warp * QW;           // chunk-local index of this warp's first query
    const int last_key = base + min(T - 1, q_first + QW - 1);  // keys 0..last_key are visible to some query
    const __half *kbase = kc + b * cb + kh * ch;
    const __half *vbase = vc + b * cb + kh * ch;
    if (q_first < T) {
        for (int k0 = 0; k0 <= last_key; k0 += 32) {
            const int key = k0 + lane;
            float s[QW];
#pragma unroll
            for (int i = 0; i < QW; ++i) s[i] = 0.0f;
            if (key <= last_key) {
                const uint4 *kr = reinterpret_cast<const uint4 *>(kbase + static_cast<int64_t>(key) * cs);
#pragma unroll 4
                for (int c = 0; c < D / 8; ++c) {
                    const uint4 raw = kr[c];
                    const float4 lo = h4_to_f4(make_uint2(raw.x, raw.y));
                    const float4 hi = h4_to_f4(make_uint2(raw.z, raw.w));
#pragma unroll
                    for (int i = 0; i < QW; ++i) {
                        const float *qq = &qs[warp * QW + i][c * 8];
                        s[i] += lo.x * qq[0] + lo.y * qq[1] + lo.z * qq[2] + lo.w * qq[3] + hi.x * qq[4] +
                                hi.y * qq[5] + hi.z * qq[6] + hi.w * qq[7];
                    }
                }
            }
            float p[QW];
#pragma unroll
            for (int i = 0; i < QW; ++i) {
                const bool vis = key <= base + q_first + i && q_first + i < T;
                const float sv = vis ? s[i] : -FLT_MAX;
                const float tmax = warp_max(sv);
                const float m_new = fmaxf(m_run[i], tmax);
                const float corr = m_run[i] == -FLT_MAX ? 0.0f : __expf(m_run[i] - m_new);
                p[i] = vis ? __expf(sv - m_new) : 0.0f;
                l_run[i] = l_run[i] * corr + warp_sum(p[i]);
                m_run[i] = m_new;
#pragma unroll
                for (int e = 0; e < E; ++e) acc[i][e] *= corr;
            }
            const int n_keys = min(32, last_key - k0 + 1);
            for (int j = 0; j < n_keys; ++j) {
                const __half *vr = vbase + static_cast<int64_t>(k0 + j) * cs + lane * E;
                float vv[E];
#pragma unroll
                for (int e = 0; e < E; ++e) vv[e] = __half2float(vr[e]);
#pragma unroll
                for (int i = 0; i < QW; ++i) {
                    const float pj = __shfl_sync(0xffffffffu, p[i], j);
#pragma unroll
                    for (int e = 0; e < E; ++e) acc[i][e] = fmaf(pj, vv[e], acc[i][e]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < QW; ++i) {
            const int t = q_first + i;
            if (t >= T) continue;
            __half *o = out + b * o_sb + t * o_st + h * o_sh + lane * E;
            const float invl = l_run[i] > 0.0f ? 1.0f / l_run[i] : 0.0f;
#pragma unroll
            for (int e = 0; e < E; ++e) o[e] = __float2half_rn(acc[i][e] * invl);
        }
    }
}

// ------------------------------------------- prefill attention, tensor cores
// Flash attention for a chunk of T queries (absolute positions positions[b] +
// t) against the cache rows 0 .. positions[b] + t, D = 128.  CTA = 4 warps on
// (b, head h, 64-query tile); warp w owns queries 16 w .. 16 w + 15 of the
// tile as the 16 rows of mma.m16n8k16.  Key / value tiles of 64 rows stream
// through a 3-stage shared-memory ring (cp.async, rows padded to 272 bytes so
// ldmatrix reads are conflict-free).  Per key tile a warp computes S = Q K^T
// (8 n-tiles x 8 k-steps), an online softmax per row in the log2 domain, and
// O += P V with P taken straight from the S accumulators as A fragments, split
// into fp16 high and low parts so the product keeps fp32 accuracy.  Query
// tiles are visited heaviest first (most keys under the causal mask).
constexpr int kPtQ = 64;
constexpr int kPtK = 64;
constexpr int kPtStages = 2;
constexpr int kPtRow = 136;  // halves per shared-memory row (272 B)
constexpr int kPtStageBytes = 2 * kPtK * kPtRow * 2;
constexpr int kPtSmem = kPtQ * kPtRow * 2 + kPtStages * kPtStageBytes;

// EXT = the llama.cpp-style program (llama_flash_attn_f32_f16_f16): keys [0, S) of the cache with
// an explicit additive fp16 mask [T, S] (sequence b's at mask + b * m_sb) instead of the causal
// rule, and the mask classifier's 2-bit codes per (16-row block, 64-key tile): 1 = all masked (the
// warp skips the tile), 2 = all zero (no mask values read).  F32IO: fp32 q and output (that
// program's), else fp16.
template <bool EXT, bool F32IO = EXT>
__global__ void __launch_bounds__(128) attn_prefill_tc_kernel(
    const void *__restrict__ qv, const __half *__restrict__ kc, const __half *__restrict__ vc,
    void *__restrict__ outv, const int32_t *__restrict__ positions, int T, int NH, int NK, int64_t cb, int64_t cs,
    int64_t ch, int64_t q_sb, int64_t q_st, int64_t q_sh, int64_t o_sb, int64_t o_st, int64_t o_sh, float scale_log2,
    const __half *__restrict__ mask, int64_t m_st, const uint32_t *__restrict__ mopt, int64_t mo_st, int S,
    int64_t m_sb) {
    extern __shared__ __align__(128) uint8_t pt_smem[];
    __shared__ int s_nkt;
    __half *qs = reinterpret_cast<__half *>(pt_smem);
    const int qtiles = (T + kPtQ - 1) / kPtQ;
    const int qt = qtiles - 1 - static_cast<int>(blockIdx.x % qtiles);
    const int h = (blockIdx.x / qtiles) % NH;
    const int b = blockIdx.x / (qtiles * NH);
    const int kh = h / (NH / NK);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3;
    pdl_wait();
    pdl_trigger();
    const int base = EXT ? 0 : positions[b];
    const int q0 = qt * kPtQ;
    const int last_key = EXT ? S - 1 : base + min(T - 1, q0 + kPtQ - 1);
    const int rb = (q0 >> 4) + w;  // this warp's 16-row block (mask classifier rows)
    auto code_of = [&](int kt) -> uint32_t {
        return (mopt[rb * mo_st + (kt >> 4)] >> (2 * (kt & 15))) & 3u;
    };
    int nkt = last_key / kPtK + 1;
    if (EXT && mopt != nullptr) {
        // the CTA stops after the last key tile that some warp's rows do not mask entirely
        if (threadIdx.x == 0) s_nkt = 0;
        __syncthreads();
        int last = -1;
        if (rb * 16 < T)
            for (int kt = lane; kt < nkt; kt += 32)
                if (code_of(kt) != 1u) last = kt;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
        if (lane == 0) atomicMax(&s_nkt, last + 1);
        __syncthreads();
        nkt = s_nkt;
    }
    const __half *kbase = kc + b * cb + kh * ch;
    const __half *vbase = vc + b * cb + kh * ch;
    auto issue = [&](int kt) {
        if (kt < nkt) {
            __half *ks = reinterpret_cast<__half *>(pt_smem + kPtQ * kPtRow * 2 + (kt % kPtStages) * kPtStageBytes);
            __half *vs = ks + kPtK * kPtRow;
            for (int i = threadIdx.x; i < kPtK * 16; i += 128) {
                const int r = i >> 4, c = i & 15;
                const int key = kt * kPtK + r;
                const bool in = key <= last_key;
                const int64_t src = (in ? static_cast<int64_t>(key) * cs : 0) + c * 8;
                ca_cp16(ks + r * kPtRow + c * 8, kbase + src, in ? 16u : 0u);
                ca_cp16(vs + r * kPtRow + c * 8, vbase + src, in ? 16u : 0u);
            }
        }
        ca_commit();
    };
    issue(0);
    issue(1);
    // q tile -> shared memory (rows past T zero; fp32 q rounded to fp16)
    for (int i = threadIdx.x; i < kPtQ * 16; i += 128) {
        const int r = i >> 4, c = i & 15;
        const int tq = q0 + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tq < T) {
            const int64_t off = b * q_sb + tq * q_st + h * q_sh + c * 8;
            if (F32IO) {
                const float4 a = *reinterpret_cast<const float4 *>(static_cast<const float *>(qv) + off);
                const float4 c4 = *reinterpret_cast<const float4 *>(static_cast<const float *>(qv) + off + 4);
                const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
                const __half2 h2 = __floats2half2_rn(c4.x, c4.y), h3 = __floats2half2_rn(c4.z, c4.w);
                v = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                               *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            } else {
                v = *reinterpret_cast<const uint4 *>(static_cast<const __half *>(qv) + off);
            }
        }
        *reinterpret_cast<uint4 *>(qs + r * kPtRow + c * 8) = v;
    }
    __syncthreads();
    uint32_t qa[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) ldsm_x4(qa[ks], qs + (16 * w + (lane & 15)) * kPtRow + 16 * ks + 8 * (lane >> 4));

    // rows g and g + 8 of this warp: chunk-local query indices
    const int tq0 = q0 + 16 * w + g, tq1 = tq0 + 8;
    const int qp0 = base + tq0, qp1 = base + tq1;  // absolute positions (keys <= qp visible)
    const int warp_first = base + q0 + 16 * w;      // smallest query position of the warp
    float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.0f, 0.0f};
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    for (int kt = 0; kt < nkt; ++kt) {
        ca_wait<1>();
        __syncthreads();
        const __half *ks = reinterpret_cast<const __half *>(pt_smem + kPtQ * kPtRow * 2 + (kt % kPtStages) * kPtStageBytes);
        const __half *vs = ks + kPtK * kPtRow;
        const int k0 = kt * kPtK;
        const uint32_t code = (EXT && mopt != nullptr && rb * 16 < T) ? code_of(kt) : 0u;
        // some key of the tile is visible to some row of the warp
        if (EXT ? (code != 1u && rb * 16 < T) : (k0 <= base + q0 + 16 * w + 15)) {
            float s[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
#pragma unroll
            for (int ks8 = 0; ks8 < 8; ++ks8) {
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t kb[4];
                    ldsm_x4(kb, ks + (16 * np + (lane & 7) + 8 * (lane >> 4)) * kPtRow + 16 * ks8 + 8 * ((lane >> 3) & 1));
                    mma_f16_16816(s[2 * np], qa[ks8], kb[0], kb[1]);
                    mma_f16_16816(s[2 * np + 1], qa[ks8], kb[2], kb[3]);
                }
            }
            const bool masked = k0 + kPtK - 1 > warp_first;
            float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = k0 + 8 * n + 2 * t4 + (e & 1);
                    const int r = e >> 1;
                    float v = s[n][e] * scale_log2;
                    if (EXT) {
                        if (key >= S) {
                            v = -FLT_MAX;
                        } else if (code != 2u) {
                            const int tq = min(r ? tq1 : tq0, T - 1);
                            const float mv = __half2float(mask[b * m_sb + tq * m_st + key]);
                            v = mv <= -1.7014117e38f ? -FLT_MAX : fmaf(mv, 1.4426950408889634f, v);
                        }
                    } else if (masked && key > (r ? qp1 : qp0)) {
                        v = -FLT_MAX;
                    }
                    s[n][e] = v;
                    mx[r] = fmaxf(mx[r], v);
                }
            float corr[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                const float m_new = fmaxf(m_run[r], mx[r]);
                corr[r] = exp2f(m_run[r] - m_new);
                m_run[r] = m_new;
                l_run[r] *= corr[r];
            }
#pragma unroll
            for (int n = 0; n < 16; ++n) {
                o[n][0] *= corr[0];
                o[n][1] *= corr[0];
                o[n][2] *= corr[1];
                o[n][3] *= corr[1];
            }
            // P as A fragments: k-step j covers keys 16 j .. 16 j + 15 = n-tiles 2 j, 2 j + 1
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float p[2][4];
#pragma unroll
                for (int hn = 0; hn < 2; ++hn)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float v = s[2 * j + hn][e];
                        const float pv = v == -FLT_MAX ? 0.0f : exp2f(v - m_run[e >> 1]);
                        l_run[e >> 1] += pv;
                        p[hn][e] = pv;
                    }
                uint32_t ah[4], al[4];
#pragma unroll
                for (int hn = 0; hn < 2; ++hn)
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        const __half2 hi = __floats2half2_rn(p[hn][2 * r], p[hn][2 * r + 1]);
                        const float2 hf = __half22float2(hi);
                        const __half2 lo = __floats2half2_rn(p[hn][2 * r] - hf.x, p[hn][2 * r + 1] - hf.y);
                        ah[2 * hn + r] = *reinterpret_cast<const uint32_t *>(&hi);
                        al[2 * hn + r] = *reinterpret_cast<const uint32_t *>(&lo);
                    }
#pragma unroll
                for (int dp = 0; dp < 8; ++dp) {
                    uint32_t vb[4];
                    ldsm_x4_t(vb, vs + (16 * j + (lane & 7) + 8 * ((lane >> 3) & 1)) * kPtRow + 16 * dp + 8 * (lane >> 4));
                    mma_f16_16816(o[2 * dp], ah, vb[0], vb[1]);
                    mma_f16_16816(o[2 * dp], al, vb[0], vb[1]);
                    mma_f16_16816(o[2 * dp + 1], ah, vb[2], vb[3]);
                    mma_f16_16816(o[2 * dp + 1], al, vb[2], vb[3]);
                }
            }
        }
        __syncthreads();  // the stage is consumed before it is refilled
        issue(kt + 2);
    }
    ca_wait<0>();
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
    const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
        const int d = 8 * n + 2 * t4;
        const int64_t o0 = b * o_sb + tq0 * o_st + h * o_sh + d, o1 = b * o_sb + tq1 * o_st + h * o_sh + d;
        if (F32IO) {
            float *out = static_cast<float *>(outv);
            if (tq0 < T) *reinterpret_cast<float2 *>(out + o0) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
            if (tq1 < T) *reinterpret_cast<float2 *>(out + o1) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
        } else {
            __half *out = static_cast<__half *>(outv);
            if (tq0 < T) *reinterpret_cast<__half2 *>(out + o0) = __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
            if (tq1 < T) *reinterpret_cast<__half2 *>(out + o1) = __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
        }
    }
}

// ---------------------------------------------------------------- misc
__global__ void embedding_f16_kernel(const __half *__restrict__ w, const int64_t *__restrict__ ids,
                                     __half *__restrict__ out, int64_t n_ids, int64_t vocab, int H) {
    const int64_t row = blockIdx.x;
    if (row >= n_ids) return;
    pdl_wait();
    pdl_trigger();
    int64_t id = ids[row];
    if (id < 0 || id >= vocab) {
        report_device_error(T2C_EINVAL);
        id = 0;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(w + id * H);
    uint4 *dst = reinterpret_cast<uint4 *>(out + row * H);
    for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = src[c];
}

// Q4_K row decode (embedding_q4_k_f32.py:96-110): w = (d * sc) * q - dmin * m.
template <typename OT>
__global__ void embedding_q4k_kernel(const uint8_t *__restrict__ w, const int64_t *__restrict__ ids,
                                     OT *__restrict__ out, int64_t n_ids, int64_t vocab, int H) {
    const int64_t row = blockIdx.x;
    if (row >= n_ids) return;
    pdl_wait();
    pdl_trigger();
    int64_t id = ids[row];
    if (id < 0 || id >= vocab) {
        report_device_error(T2C_EINVAL);
        id = 0;
    }
    const uint8_t *src = w + id * (H / 256) * 144;
    for (int k = threadIdx.x; k < H; k += blockDim.x) {
        const uint8_t *blk = src + (k >> 8) * 144;
        const int i = k & 255, j = i >> 5;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
        const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[2] | (blk[3] << 8))));
        uint32_t sc, m;
        if (j < 4) {
            sc = blk[4 + j] & 63u;
            m = blk[8 + j] & 63u;
        } else {
            sc = (blk[8 + j] & 15u) | ((blk[j] >> 6) << 4);
            m = (blk[8 + j] >> 4) | ((blk[4 + j] >> 6) << 4);
        }
        const uint8_t byte = blk[16 + (i >> 6) * 32 + (i & 31)];
        const uint32_t qv = (i & 32) ? (byte >> 4) : (byte & 15u);
        out[row * H + k] = static_cast<OT>((d * static_cast<float>(sc)) * static_cast<float>(qv) - dmin * static_cast<float>(m));
    }
}

__global__ void add_kernel(const __half *__restrict__ x, const __half *__restrict__ r, __half *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 a = h4_to_f4(*reinterpret_cast<const uint2 *>(x + i));
        const float4 c = h4_to_f4(*reinterpret_cast<const uint2 *>(r + i));
        *reinterpret_cast<uint2 *>(y + i) = f4_to_h4(make_float4(a.x + c.x, a.y + c.y, a.z + c.z, a.w + c.w));
    } else {
        for (int64_t j = i; j < n; ++j) y[j] = __float2half_rn(__half2float(x[j]) + __half2float(r[j]));
    }
}

__device__ __forceinline__ float silu_h(float g) { return __half2float(__float2half_rn(g / (1.0f + __expf(-g)))); }

__global__ void swiglu_kernel(const __half *__restrict__ g, const __half *__restrict__ u, __half *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
    if (i + 3 < n) {
        const float4 a = h4_to_f4(*reinterpret_cast<const uint2 *>(g + i));
        const float4 c = h4_to_f4(*reinterpret_cast<const uint2 *>(u + i));
        *reinterpret_cast<uint2 *>(y + i) =
            f4_to_h4(make_float4(silu_h(a.x) * c.x, silu_h(a.y) * c.y, silu_h(a.z) * c.z, silu_h(a.w) * c.w));
    } else {
        for (int64_t j = i; j < n; ++j) y[j] = __float2half_rn(silu_h(__half2float(g[j])) * __half2float(u[j]));
    }
}

// ------------------------------------------------------------ greedy select
__device__ __forceinline__ bool better(float s, uint32_t t, float bs, uint32_t bt) {
    return s > bs || (s == bs && t < bt);
}

__global__ void __launch_bounds__(1024) token_select_kernel(const float *__restrict__ ps, const uint32_t *__restrict__ pt,
                                                            int64_t G, const int64_t *__restrict__ eos, int64_t E,
                                                            int64_t *__restrict__ next_token, uint32_t *__restrict__ done) {
    __shared__ float ss[32];
    __shared__ uint32_t st[32];
    const int64_t m = blockIdx.x;
    pdl_wait();
    pdl_trigger();
    float best = -FLT_MAX;
    uint32_t tok = 0xffffffffu;
    for (int64_t g = threadIdx.x; g < G; g += blockDim.x) {
        const float s = ps[m * G + g];
        const uint32_t t = pt[m * G + g];
        if (better(s, t, best, tok)) {
            best = s;
            tok = t;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float s = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t t = __shfl_xor_sync(0xffffffffu, tok, o);
        if (better(s, t, best, tok)) {
            best = s;
            tok = t;
        }
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        ss[warp] = best;
        st[warp] = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int nw = blockDim.x >> 5;
        for (int w = 1; w < nw; ++w)
            if (better(ss[w], st[w], best, tok)) {
                best = ss[w];
                tok = st[w];
            }
        next_token[m] = static_cast<int64_t>(tok);
        uint32_t is_done = 0;
        for (int64_t e = 0; e < E; ++e)
            if (static_cast<int64_t>(tok) == eos[e]) is_done = 1;
        done[m] = is_done;
    }
}

__global__ void token_store_kernel(const int64_t *__restrict__ next_token, const uint32_t *__restrict__ done,
                                   int64_t *__restrict__ gen, uint32_t *__restrict__ gen_len, uint32_t *__restrict__ stopped,
                                   int64_t B, int64_t G, int32_t index_value, const int32_t *__restrict__ index_dev,
                                   int stop_on_eos) {
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b >= B) return;
    pdl_wait();
    pdl_trigger();
    const int64_t index = index_dev ? index_dev[0] : index_value;
    if (index < 0 || index >= G) return;
    if (stop_on_eos && stopped[b]) return;
    gen[b * G + index] = next_token[b];
    gen_len[b] = static_cast<uint32_t>(index + 1);
    if (stop_on_eos && done[b]) stopped[b] = 1u;
}

__global__ void advance_kernel(int32_t *positions, int64_t B, int32_t *token_index) {
    pdl_wait();
    pdl_trigger();
    const int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (b < B) positions[b] += 1;
    if (b == 0 && token_index) token_index[0] += 1;
}

template <typename Kernel, typename... Args>
int launch(Kernel kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

// Launch with a (cluster, 1, 1) thread-block cluster and programmatic stream
// serialization; the dynamic shared-memory limit is raised once per device.
template <typename Kernel, typename... Args>
int launch_cluster(Kernel kernel, bool &configured, dim3 grid, dim3 block, size_t smem, unsigned cluster,
                   cudaStream_t stream, Args... args) {
    if (!configured) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return set_error(T2C_ECUDA, "cluster launch: cudaFuncSetAttribute failed");
        configured = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "cluster launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

int current_device_slot() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    return dev;
}

bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Split partials (max, sum, 2 pad words, acc[D]) for every (b, head, split),
// then one arrival counter per (b, head) in the last B * NH words.
int64_t attn_decode_fused_workspace(int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t splits) {
    (void)NK;
    return splits > kCaMaxSplits ? B * NH * splits * (D + 4) + B * NH : 0;
}

}  // namespace

cudaError_t status_decode(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c

using namespace t2c;

extern "C" int t2c_rms_norm(const void *x, const float *w, void *y, int64_t rows, int64_t cols, float eps, void *stream) {
    if (!x || !w || !y) return set_error(T2C_EINVAL, "rms_norm: NULL pointer");
    if (rows <= 0 || cols <= 0 || cols % 4) return set_error(T2C_EINVAL, "rms_norm: cols must be a positive multiple of 4");
    if (!aligned(x, 8) || !aligned(y, 8) || !aligned(w, 16)) return set_error(T2C_EINVAL, "rms_norm: misaligned operand");
    if (cols % 8 == 0 && cols <= 8 * kRnThreads * kRnVec && aligned(x, 16) && aligned(y, 16))
        return launch(rms_norm_row_kernel, dim3(static_cast<unsigned>(rows)), dim3(kRnThreads), 0, as_stream(stream),
                      static_cast<const __half *>(x), w, static_cast<__half *>(y), static_cast<int>(cols), eps);
    const int warps = 8;
    return launch(rms_norm_kernel, dim3(static_cast<unsigned>((rows + warps - 1) / warps)), dim3(warps * 32), 0,
                  as_stream(stream), static_cast<const __half *>(x), w, static_cast<__half *>(y), rows,
                  static_cast<int>(cols), eps);
}

extern "C" int t2c_qk_norm_rope_cache(const void *q_in, const void *k_in, const void *v_in, const float *q_w,
                                      const float *k_w, void *q_out, void *k_cache, void *v_cache,
                                      const int32_t *positions, int64_t B, int64_t T, int64_t NH, int64_t NK,
                                      int64_t D, int64_t cb, int64_t cs, int64_t ch, const float *inv_freq, float eps,
                                      void *stream) {
    if (!q_in || !k_in || !v_in || !q_w || !k_w || !q_out || !k_cache || !v_cache || !positions || !inv_freq)
        return set_error(T2C_EINVAL, "qk_norm_rope_cache: NULL pointer");
    if (B <= 0 || T <= 0 || NH <= 0 || NK <= 0 || NH % NK) return set_error(T2C_EINVAL, "qk_norm_rope_cache: bad heads");
    const int64_t vecs = B * T * (NH + 2 * NK);
    const int warps = 8;
    const dim3 grid(static_cast<unsigned>((vecs + warps - 1) / warps)), block(warps * 32);
    const cudaStream_t s = as_stream(stream);
#define T2C_QKR(E)                                                                                                   \
    return launch(qk_norm_rope_cache_kernel<E>, grid, block, 0, s, static_cast<const __half *>(q_in),                  \
                  static_cast<const __half *>(k_in), static_cast<const __half *>(v_in), q_w, k_w,                     \
                  static_cast<__half *>(q_out), static_cast<__half *>(k_cache), static_cast<__half *>(v_cache),       \
                  positions, static_cast<int>(B), static_cast<int>(T), static_cast<int>(NH), static_cast<int>(NK),    \
                  cb, cs, ch, inv_freq, eps)
    switch (D) {
        case 64: T2C_QKR(2);
        case 128: T2C_QKR(4);
        case 256: T2C_QKR(8);
        default: return set_error(T2C_EUNSUPPORTED, "qk_norm_rope_cache: D=%lld", (long long)D);
    }
#undef T2C_QKR
}

extern "C" int t2c_attn_decode(const void *q, const void *k_cache, const void *v_cache, void *out,
                               const int32_t *positions, int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t max_len,
                               int64_t cb, int64_t cs, int64_t ch, int64_t splits, float *workspace,
                               int64_t workspace_floats, void *stream) {
    if (!q || !k_cache || !v_cache || !out || !positions) return set_error(T2C_EINVAL, "attn_decode: NULL pointer");
    if (B <= 0 || NH <= 0 || NK <= 0 || NH % NK || max_len <= 0 || max_len > INT32_MAX || splits <= 0)
        return set_error(T2C_EINVAL, "attn_decode: bad shape");
    const int G = static_cast<int>(NH / NK);
    if (G > kMaxGroup) return set_error(T2C_EUNSUPPORTED, "attn_decode: group %d > %d", G, kMaxGroup);
    if (splits > kMaxSplits) return set_error(T2C_EUNSUPPORTED, "attn_decode: splits %lld > %d", (long long)splits, kMaxSplits);
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || cs % 8 || cb % 8 || ch % 8)
        return set_error(T2C_EINVAL, "attn_decode: cache rows must be 16-byte aligned");
    if (splits > 1) {
        const int64_t need = B * NH * splits * (D + 2);
        if (!workspace || workspace_floats < need)
            return set_error(T2C_ESCRATCH, "attn_decode: workspace needs %lld floats", (long long)need);
    }
    const int chunk = static_cast<int>((max_len + splits - 1) / splits);
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    const cudaStream_t s = as_stream(stream);
    const dim3 grid(static_cast<unsigned>(B * NK * splits)), block(kAttnWarps * 32);
    int rc = T2C_OK;
#define T2C_ATT(E, GG)                                                                                           \
    rc = launch(attn_decode_kernel<E, GG, false>, grid, block, 0, s, static_cast<const __half *>(q),               \
                static_cast<const __half *>(k_cache), static_cast<const __half *>(v_cache), static_cast<__half *>(out), \
                positions, static_cast<int>(NH), static_cast<int>(NK), cb, cs, ch, static_cast<int>(max_len), chunk, \
                static_cast<int>(splits), workspace, scale, static_cast<const int32_t *>(nullptr), int64_t(0), 0, 0)
    if (D == 128) {
        switch (G) {
            case 1: T2C_ATT(4, 1); break;
            case 2: T2C_ATT(4, 2); break;
            case 4: T2C_ATT(4, 4); break;
            case 8: T2C_ATT(4, 8); break;
            default: return set_error(T2C_EUNSUPPORTED, "attn_decode: group %d", G);
        }
    } else if (D == 64) {
        switch (G) {
            case 1: T2C_ATT(2, 1); break;
            case 2: T2C_ATT(2, 2); break;
            case 4: T2C_ATT(2, 4); break;
            case 8: T2C_ATT(2, 8); break;
            default: return set_error(T2C_EUNSUPPORTED, "attn_decode: group %d", G);
        }
    } else {
        return set_error(T2C_EUNSUPPORTED, "attn_decode: D=%lld", (long long)D);
    }
#undef T2C_ATT
    if (rc != T2C_OK || splits == 1) return rc;
    if (D == 128)
        return launch(attn_combine_kernel<4>, dim3(static_cast<unsigned>(B * NH)), dim3(128), 0, s,
                      static_cast<const float *>(workspace), static_cast<__half *>(out), static_cast<int>(B),
                      static_cast<int>(NH), static_cast<int>(splits));
    return launch(attn_combine_kernel<2>, dim3(static_cast<unsigned>(B * NH)), dim3(64), 0, s,
                  static_cast<const float *>(workspace), static_cast<__half *>(out), static_cast<int>(B),
                  static_cast<int>(NH), static_cast<int>(splits));
}

extern "C" int t2c_attn_decode_fused(const void *q_in, const void *k_in, const void *v_in, int64_t q_sb, int64_t k_sb,
                                     int64_t v_sb, const float *q_w, const float *k_w, const float *inv_freq, float eps,
                                     void *k_cache, void *v_cache, int64_t cb, int64_t cs, int64_t ch, void *out,
                                     int64_t o_sb, const int32_t *positions, int64_t B, int64_t NH, int64_t NK,
                                     int64_t D, int64_t max_len, int64_t splits, float *workspace,
                                     int64_t workspace_floats, void *stream) {
    if (!q_in || !k_in || !v_in || !q_w || !k_w || !inv_freq || !k_cache || !v_cache || !out || !positions)
        return set_error(T2C_EINVAL, "attn_decode_fused: NULL pointer");
    if (B <= 0 || NH <= 0 || NK <= 0 || NH % NK || splits <= 0 || max_len <= 0 || max_len > INT32_MAX)
        return set_error(T2C_EINVAL, "attn_decode_fused: bad shape");
    if (D != 128) return set_error(T2C_EUNSUPPORTED, "attn_decode_fused: D=%lld (128 only)", (long long)D);
    const int G = static_cast<int>(NH / NK);
    if (splits > kMaxSplits) return set_error(T2C_EUNSUPPORTED, "attn_decode_fused: splits %lld > %d", (long long)splits, kMaxSplits);
    if (!aligned(k_cache, 16) || !aligned(v_cache, 16) || cs % 8 || cb % 8 || ch % 8)
        return set_error(T2C_EINVAL, "attn_decode_fused: cache rows must be 16-byte aligned");
    if (!aligned(q_in, 8) || !aligned(k_in, 8) || !aligned(v_in, 8) || q_sb % 4 || k_sb % 4 || v_sb % 4 || !aligned(q_w, 16) ||
        !aligned(k_w, 16))
        return set_error(T2C_EINVAL, "attn_decode_fused: q/k/v rows must be 8-byte aligned");
    const float qscale = 1.4426950408889634f / sqrtf(static_cast<float>(D));
    const cudaStream_t s = as_stream(stream);
    if (splits <= kCaMaxSplits) {
        static bool configured[4][64] = {};  // [group 1 / 2 / 4 / 8][device]
        const int dev_slot = current_device_slot();
        const dim3 grid(static_cast<unsigned>(B * NK * splits));
#define T2C_CLUSTER(GG)                                                                                                \
    return launch_cluster(attn_decode_cluster_kernel<GG>, configured[GG == 1 ? 0 : GG == 2 ? 1 : GG == 4 ? 2 : 3][dev_slot], \
                          grid, dim3(kCaWarps * 32), kCaSmem,                                                            \
                          static_cast<unsigned>(splits), s, static_cast<const __half *>(q_in),                           \
                          static_cast<const __half *>(k_in), static_cast<const __half *>(v_in), q_sb, k_sb, v_sb, q_w,   \
                          k_w, inv_freq, eps, static_cast<__half *>(k_cache), static_cast<__half *>(v_cache), cb, cs, ch, \
                          static_cast<__half *>(out), o_sb, positions, static_cast<int>(NK), static_cast<int>(max_len),  \
                          static_cast<int>(splits), qscale)
        switch (G) {
            case 1: T2C_CLUSTER(1);
            case 2: T2C_CLUSTER(2);
            case 4: T2C_CLUSTER(4);
            case 8: T2C_CLUSTER(8);
            default: return set_error(T2C_EUNSUPPORTED, "attn_decode_fused: group %d", G);
        }
#undef T2C_CLUSTER
    }
    int *counters = nullptr;
    {
        const int64_t need = attn_decode_fused_workspace(B, NH, NK, D, splits);
        if (!workspace || workspace_floats < need)
            return set_error(T2C_ESCRATCH, "attn_decode_fused: workspace needs %lld words", (long long)need);
        counters = reinterpret_cast<int *>(workspace + (need - B * NH));
    }
    const dim3 grid(static_cast<unsigned>(B * NK * splits));
#define T2C_FUSED(GG)                                                                                              \
    return launch(attn_decode_fused_kernel<GG>, grid, dim3(GG * 32), 0, s, static_cast<const __half *>(q_in),               \
                  static_cast<const __half *>(k_in), static_cast<const __half *>(v_in), q_sb, k_sb, v_sb, q_w, k_w,  \
                  inv_freq, eps, static_cast<__half *>(k_cache), static_cast<__half *>(v_cache), cb, cs, ch,         \
                  static_cast<__half *>(out), o_sb, positions, static_cast<int>(NK), static_cast<int>(max_len),     \
                  static_cast<int>(splits), workspace, counters, qscale)
    switch (G) {
        case 1: T2C_FUSED(1);
        case 2: T2C_FUSED(2);
        case 4: T2C_FUSED(4);
        case 8: T2C_FUSED(8);
        default: return set_error(T2C_EUNSUPPORTED, "attn_decode_fused: group %d", G);
    }
#undef T2C_FUSED
}

extern "C" int64_t t2c_attn_decode_fused_workspace(int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t splits) {
    return attn_decode_fused_workspace(B, NH, NK, D, splits);
}

extern "C" int t2c_attn_prefill(const void *q, const void *k_cache, const void *v_cache, void *out,
                                const int32_t *positions, int64_t B, int64_t T, int64_t NH, int64_t NK, int64_t D,
                                int64_t cb, int64_t cs, int64_t ch, int64_t qb, int64_t qt, int64_t qh, int64_t ob,
                                int64_t ot, int64_t oh, void *stream) {
    if (!q || !k_cache || !v_cache || !out || !positions) return set_error(T2C_EINVAL, "attn_prefill: NULL pointer");
    if (B <= 0 || T <= 0 || NH <= 0 || NK <= 0 || NH % NK) return set_error(T2C_EINVAL, "attn_prefill: bad shape");
    if (!aligned(k_cache, 16) || cs % 8 || cb % 8 || ch % 8)
        return set_error(T2C_EINVAL, "attn_prefill: cache rows must be 16-byte aligned");
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    if (D == 128) {  // tcgen05 tiles where the operand strides allow them
        const int rc = attn_prefill_umma(q, k_cache, v_cache, out, positions, B, T, NH, NK, cb, cs, ch, qb, qt, qh, ob,
                                         ot, oh, scale, as_stream(stream), nullptr, 0, 0, 0, false);
        if (rc != T2C_EUNSUPPORTED) return rc;
    }
    if (D == 128 && aligned(q, 16) && qb % 8 == 0 && qt % 8 == 0 && qh % 8 == 0 && aligned(out, 4) && ob % 2 == 0 &&
        ot % 2 == 0 && oh % 2 == 0) {
        static bool configured[64] = {};
        const int dev_slot = current_device_slot();
        if (!configured[dev_slot]) {
            if (cudaFuncSetAttribute(attn_prefill_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPtSmem) !=
                cudaSuccess)
                return set_error(T2C_ECUDA, "attn_prefill: cudaFuncSetAttribute failed");
            configured[dev_slot] = true;
        }
        const int64_t tiles = (T + kPtQ - 1) / kPtQ;
        return launch(attn_prefill_tc_kernel<false>, dim3(static_cast<unsigned>(B * NH * tiles)), dim3(128), kPtSmem,
                      as_stream(stream), q, static_cast<const __half *>(k_cache),
                      static_cast<const __half *>(v_cache), out, positions, static_cast<int>(T),
                      static_cast<int>(NH), static_cast<int>(NK), cb, cs, ch, qb, qt, qh, ob, ot, oh,
                      1.4426950408889634f * scale, static_cast<const __half *>(nullptr), int64_t{0},
                      static_cast<const uint32_t *>(nullptr), int64_t{0}, 0, int64_t{0});
    }
    const int64_t qtiles = (T + kPfQ - 1) / kPfQ;
    const dim3 grid(static_cast<unsigned>(B * NH * qtiles)), block(128);
    const cudaStream_t s = as_stream(stream);
    if (D == 128)
        return launch(attn_prefill_kernel<4>, grid, block, 0, s, static_cast<const __half *>(q),
                      static_cast<const __half *>(k_cache), static_cast<const __half *>(v_cache),
                      static_cast<__half *>(out), positions, static_cast<int>(T), static_cast<int>(NH),
                      static_cast<int>(NK), cb, cs, ch, qb, qt, qh, ob, ot, oh, scale);
    if (D == 64)
        return launch(attn_prefill_kernel<2>, grid, block, 0, s, static_cast<const __half *>(q),
                      static_cast<const __half *>(k_cache), static_cast<const __half *>(v_cache),
                      static_cast<__half *>(out), positions, static_cast<int>(T), static_cast<int>(NH),
                      static_cast<int>(NK), cb, cs, ch, qb, qt, qh, ob, ot, oh, scale);
    return set_error(T2C_EUNSUPPORTED, "attn_prefill: D=%lld", (long long)D);
}

extern "C" int t2c_attn_prefill_masked_f32(const float *q, const void *k_cache, const void *v_cache, const void *mask,
                                           const uint32_t *mask_opt, float *out, int64_t B, int64_t T, int64_t S,
                                           int64_t NH, int64_t NK, int64_t D, int64_t mask_row_stride,
                                           int64_t mask_opt_row_stride, float scale, void *stream) {
    if (!q || !k_cache || !v_cache || !mask || !out) return set_error(T2C_EINVAL, "attn_prefill_masked_f32: NULL pointer");
    if (B <= 0 || T <= 0 || S <= 0 || NH <= 0 || NK <= 0 || NH % NK || T > INT32_MAX || S > INT32_MAX ||
        mask_row_stride < S)
        return set_error(T2C_EINVAL, "attn_prefill_masked_f32: bad shape");
    if (D != 128) return set_error(T2C_EUNSUPPORTED, "attn_prefill_masked_f32: D=%lld (128 only)", (long long)D);
    if (!aligned(q, 16) || !aligned(out, 8) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
        return set_error(T2C_EINVAL, "attn_prefill_masked_f32: alignment");
    if (mask_opt != nullptr && mask_opt_row_stride < (S + 1023) / 1024)
        return set_error(T2C_EINVAL, "attn_prefill_masked_f32: mask_opt rows need %lld words", (long long)((S + 1023) / 1024));
    {  // tcgen05 tiles (the mask read directly; the classifier's tile skipping is the mma.sync kernel's)
        const int rc = attn_prefill_umma(q, k_cache, v_cache, out, nullptr, B, T, NH, NK, S * NK * D, NK * D, D,
                                         T * NH * D, NH * D, D, T * NH * D, NH * D, D, scale, as_stream(stream), mask, 0,
                                         mask_row_stride, S, true);
        if (rc != T2C_EUNSUPPORTED) return rc;
    }
    static bool configured[64] = {};
    const int dev_slot = current_device_slot();
    if (!configured[dev_slot]) {
        if (cudaFuncSetAttribute(attn_prefill_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPtSmem) !=
            cudaSuccess)
            return set_error(T2C_ECUDA, "attn_prefill_masked_f32: cudaFuncSetAttribute failed");
        configured[dev_slot] = true;
    }
    // token-major q / out [B, T, NH, D] and caches [B, S, NK, D]
    const int64_t tiles = (T + kPtQ - 1) / kPtQ;
    return launch(attn_prefill_tc_kernel<true>, dim3(static_cast<unsigned>(B * NH * tiles)), dim3(128), kPtSmem,
                  as_stream(stream), static_cast<const void *>(q), static_cast<const __half *>(k_cache),
                  static_cast<const __half *>(v_cache), static_cast<void *>(out),
                  static_cast<const int32_t *>(nullptr), static_cast<int>(T), static_cast<int>(NH),
                  static_cast<int>(NK), S * NK * D, NK * D, D, T * NH * D, NH * D, D, T * NH * D, NH * D, D,
                  1.4426950408889634f * scale, static_cast<const __half *>(mask), mask_row_stride, mask_opt,
                  mask_opt_row_stride, static_cast<int>(S), int64_t(0));
}

extern "C" int t2c_attn_masked_gqa(const void *q, const void *k, const void *v, const void *mask, void *out,
                                   int64_t B, int64_t T, int64_t S, int64_t NH, int64_t NK, int64_t D,
                                   const int64_t *q_strides, const int64_t *kv_strides, const int64_t *o_strides,
                                   int64_t mask_b_stride, int64_t mask_row_stride, float scale, void *stream) {
    if (!q || !k || !v || !mask || !out || !q_strides || !kv_strides || !o_strides)
        return set_error(T2C_EINVAL, "attn_masked_gqa: NULL pointer");
    if (B <= 0 || T <= 0 || S <= 0 || NH <= 0 || NK <= 0 || NH % NK || T > INT32_MAX || S > INT32_MAX ||
        mask_row_stride < S || mask_b_stride < 0)
        return set_error(T2C_EINVAL, "attn_masked_gqa: bad shape");
    if (D != 128) return set_error(T2C_EUNSUPPORTED, "attn_masked_gqa: D=%lld (128 only)", (long long)D);
    for (int i = 0; i < 3; ++i)
        if (q_strides[i] % 8 || kv_strides[i] % 8 || o_strides[i] % 2)
            return set_error(T2C_EINVAL, "attn_masked_gqa: q / k / v rows must be 16-byte aligned, out rows 4-byte");
    if (!aligned(q, 16) || !aligned(out, 4) || !aligned(k, 16) || !aligned(v, 16))
        return set_error(T2C_EINVAL, "attn_masked_gqa: alignment");
    {
        const int rc = attn_prefill_umma(q, k, v, out, nullptr, B, T, NH, NK, kv_strides[0], kv_strides[1],
                                         kv_strides[2], q_strides[0], q_strides[1], q_strides[2], o_strides[0],
                                         o_strides[1], o_strides[2], scale, as_stream(stream), mask, mask_b_stride,
                                         mask_row_stride, S, false);
        if (rc != T2C_EUNSUPPORTED) return rc;
    }
    static bool configured[64] = {};
    const int dev_slot = current_device_slot();
    if (!configured[dev_slot]) {
        if (cudaFuncSetAttribute(attn_prefill_tc_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kPtSmem) != cudaSuccess)
            return set_error(T2C_ECUDA, "attn_masked_gqa: cudaFuncSetAttribute failed");
        configured[dev_slot] = true;
    }
    const int64_t tiles = (T + kPtQ - 1) / kPtQ;
    return launch(attn_prefill_tc_kernel<true, false>, dim3(static_cast<unsigned>(B * NH * tiles)), dim3(128),
                  kPtSmem, as_stream(stream), q, static_cast<const __half *>(k), static_cast<const __half *>(v), out,
                  static_cast<const int32_t *>(nullptr), static_cast<int>(T), static_cast<int>(NH),
                  static_cast<int>(NK), kv_strides[0], kv_strides[1], kv_strides[2], q_strides[0], q_strides[1],
                  q_strides[2], o_strides[0], o_strides[1], o_strides[2], 1.4426950408889634f * scale,
                  static_cast<const __half *>(mask), mask_row_stride, static_cast<const uint32_t *>(nullptr),
                  int64_t{0}, static_cast<int>(S), mask_b_stride);
}

extern "C" int t2c_embedding(int wtype, const void *weight, const int64_t *ids, void *out, int64_t n_ids,
                             int64_t vocab, int64_t H, void *stream) {
    if (!weight || !ids || !out) return set_error(T2C_EINVAL, "embedding: NULL pointer");
    if (n_ids <= 0 || vocab <= 0 || H <= 0) return set_error(T2C_EINVAL, "embedding: bad shape");
    const cudaStream_t s = as_stream(stream);
    if (wtype == T2C_F16) {
        if (H % 8 || !aligned(weight, 16) || !aligned(out, 16)) return set_error(T2C_EINVAL, "embedding: alignment");
        return launch(embedding_f16_kernel, dim3(static_cast<unsigned>(n_ids)), dim3(128), 0, s,
                      static_cast<const __half *>(weight), ids, static_cast<__half *>(out), n_ids, vocab,
                      static_cast<int>(H));
    }
    if (wtype == T2C_Q4_K) {
        if (H % 256) return set_error(T2C_EINVAL, "embedding: Q4_K needs H %% 256 == 0");
        return launch(embedding_q4k_kernel<__half>, dim3(static_cast<unsigned>(n_ids)), dim3(256), 0, s,
                      static_cast<const uint8_t *>(weight), ids, static_cast<__half *>(out), n_ids, vocab,
                      static_cast<int>(H));
    }
    return set_error(T2C_EUNSUPPORTED, "embedding: weight type %d", wtype);
}

extern "C" int t2c_embedding_f32(int wtype, const void *weight, const int64_t *ids, float *out, int64_t n_ids,
                                 int64_t vocab, int64_t H, void *stream) {
    if (!weight || !ids || !out) return set_error(T2C_EINVAL, "embedding_f32: NULL pointer");
    if (n_ids <= 0 || vocab <= 0 || H <= 0 || H > INT32_MAX) return set_error(T2C_EINVAL, "embedding_f32: bad shape");
    if (wtype != T2C_Q4_K) return set_error(T2C_EUNSUPPORTED, "embedding_f32: weight type %d", wtype);
    if (H % 256) return set_error(T2C_EINVAL, "embedding_f32: Q4_K needs H %% 256 == 0");
    return launch(embedding_q4k_kernel<float>, dim3(static_cast<unsigned>(n_ids)), dim3(256), 0, as_stream(stream),
                  static_cast<const uint8_t *>(weight), ids, out, n_ids, vocab, static_cast<int>(H));
}

extern "C" int t2c_add(const void *x, const void *r, void *y, int64_t n, void *stream) {
    if (!x || !r || !y || n < 0) return set_error(T2C_EINVAL, "add: bad argument");
    if (n == 0) return T2C_OK;
    if (!aligned(x, 8) || !aligned(r, 8) || !aligned(y, 8)) return set_error(T2C_EINVAL, "add: misaligned");
    const int64_t threads = (n + 3) / 4;
    return launch(add_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, as_stream(stream),
                  static_cast<const __half *>(x), static_cast<const __half *>(r), static_cast<__half *>(y), n);
}

extern "C" int t2c_swiglu(const void *g, const void *u, void *y, int64_t n, void *stream) {
    if (!g || !u || !y || n < 0) return set_error(T2C_EINVAL, "swiglu: bad argument");
    if (n == 0) return T2C_OK;
    if (!aligned(g, 8) || !aligned(u, 8) || !aligned(y, 8)) return set_error(T2C_EINVAL, "swiglu: misaligned");
    const int64_t threads = (n + 3) / 4;
    return launch(swiglu_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, as_stream(stream),
                  static_cast<const __half *>(g), static_cast<const __half *>(u), static_cast<__half *>(y), n);
}

extern "C" int t2c_token_select(const float *partial_scores, const uint32_t *partial_tokens, int64_t M, int64_t G,
                                const int64_t *eos_ids, int64_t E, int64_t *next_token, uint32_t *done, void *stream) {
    if (!partial_scores || !partial_tokens || !next_token || !done || (E > 0 && !eos_ids))
        return set_error(T2C_EINVAL, "token_select: NULL pointer");
    if (M <= 0 || G <= 0 || E < 0) return set_error(T2C_EINVAL, "token_select: bad shape");
    return launch(token_select_kernel, dim3(static_cast<unsigned>(M)), dim3(1024), 0, as_stream(stream), partial_scores,
                  partial_tokens, G, eos_ids, E, next_token, done);
}

extern "C" int t2c_token_store(const int64_t *next_token, const uint32_t *done, int64_t *generated_tokens,
                               uint32_t *generated_length, uint32_t *stopped, int64_t B, int64_t G, int32_t token_index,
                               const int32_t *token_index_dev, int stop_on_eos, void *stream) {
    if (!next_token || !done || !generated_tokens || !generated_length || !stopped)
        return set_error(T2C_EINVAL, "token_store: NULL pointer");
    if (B <= 0 || G <= 0) return set_error(T2C_EINVAL, "token_store: bad shape");
    return launch(token_store_kernel, dim3(static_cast<unsigned>((B + 127) / 128)), dim3(128), 0, as_stream(stream),
                  next_token, done, generated_tokens, generated_length, stopped, B, G, token_index, token_index_dev,
                  stop_on_eos);
}

extern "C" int t2c_advance_positions(int32_t *positions, int64_t B, int32_t *token_index, void *stream) {
    if (!positions || B <= 0) return set_error(T2C_EINVAL, "advance_positions: bad argument");
    return launch(advance_kernel, dim3(static_cast<unsigned>((B + 127) / 128)), dim3(128), 0, as_stream(stream),
                  positions, B, token_index);
}

static int page_log2_of(int64_t page_size) {
    if (page_size <= 0 || page_size > (1 << 20) || (page_size & (page_size - 1))) return -1;
    int l = 0;
    while ((int64_t(1) << l) < page_size) ++l;
    return l;
}

extern "C" int t2c_attn_decode_paged(const void *q, const void *k_pages, const void *v_pages, void *out,
                                     const int32_t *positions, const int32_t *block_table, int64_t bt_stride,
                                     int64_t num_pages, int64_t page_size, int64_t page_stride, int64_t row_stride, int64_t head_stride,
                                     int64_t B, int64_t NH, int64_t NK, int64_t D, int64_t splits, float *workspace,
                                     int64_t workspace_floats, void *stream) {
    if (!q || !k_pages || !v_pages || !out || !positions || !block_table)
        return set_error(T2C_EINVAL, "attn_decode_paged: NULL pointer");
    const int pl = page_log2_of(page_size);
    if (pl < 0) return set_error(T2C_EINVAL, "attn_decode_paged: page_size %lld is not a power of two", (long long)page_size);
    if (B <= 0 || NH <= 0 || NK <= 0 || NH % NK || bt_stride <= 0 || splits <= 0 || bt_stride * page_size > INT32_MAX ||
        num_pages <= 0 || num_pages > INT32_MAX)
        return set_error(T2C_EINVAL, "attn_decode_paged: bad shape");
    const int G = static_cast<int>(NH / NK);
    if (G > kMaxGroup || (G & (G - 1))) return set_error(T2C_EUNSUPPORTED, "attn_decode_paged: group %d", G);
    if (D != 128 && D != 64) return set_error(T2C_EUNSUPPORTED, "attn_decode_paged: D=%lld", (long long)D);
    if (splits > kMaxSplits)
        return set_error(T2C_EUNSUPPORTED, "attn_decode_paged: splits %lld > %d", (long long)splits, kMaxSplits);
    if (!aligned(k_pages, 16) || !aligned(v_pages, 16) || page_stride % 8 || row_stride % 8 || head_stride % 8)
        return set_error(T2C_EINVAL, "attn_decode_paged: page rows must be 16-byte aligned");
    if (splits > 1) {
        const int64_t need = B * NH * splits * (D + 2);
        if (!workspace || workspace_floats < need)
            return set_error(T2C_ESCRATCH, "attn_decode_paged: workspace needs %lld floats", (long long)need);
    }
    const int64_t max_len = bt_stride * page_size;
    const int chunk = static_cast<int>((max_len + splits - 1) / splits);
    const float scale = 1.0f / sqrtf(static_cast<float>(D));
    const cudaStream_t s = as_stream(stream);
    const dim3 grid(static_cast<unsigned>(B * NK * splits)), block(kAttnWarps * 32);
    int rc = T2C_OK;
#define T2C_ATTP(E, GG)                                                                                          \
    rc = launch(attn_decode_kernel<E, GG, true>, grid, block, 0, s, static_cast<const __half *>(q),                \
                static_cast<const __half *>(k_pages), static_cast<const __half *>(v_pages), static_cast<__half *>(out), \
                positions, static_cast<int>(NH), static_cast<int>(NK), page_stride, row_stride, head_stride,         \
                static_cast<int>(max_len), chunk, static_cast<int>(splits), workspace, scale, block_table, bt_stride, pl,     \
                static_cast<int>(num_pages))
    switch (G * 1000 + static_cast<int>(D)) {
        case 1128: T2C_ATTP(4, 1); break;
        case 2128: T2C_ATTP(4, 2); break;
        case 4128: T2C_ATTP(4, 4); break;
        case 8128: T2C_ATTP(4, 8); break;
        case 1064: T2C_ATTP(2, 1); break;
        case 2064: T2C_ATTP(2, 2); break;
        case 4064: T2C_ATTP(2, 4); break;
        default: T2C_ATTP(2, 8); break;
    }
#undef T2C_ATTP
    if (rc != T2C_OK || splits == 1) return rc;
    if (D == 128)
        return launch(attn_combine_kernel<4>, dim3(static_cast<unsigned>(B * NH)), dim3(128), 0, s,
                      static_cast<const float *>(workspace), static_cast<__half *>(out), static_cast<int>(B),
                      static_cast<int>(NH), static_cast<int>(splits));
    return launch(attn_combine_kernel<2>, dim3(static_cast<unsigned>(B * NH)), dim3(64), 0, s,
                  static_cast<const float *>(workspace), static_cast<__half *>(out), static_cast<int>(B),
                  static_cast<int>(NH), static_cast<int>(splits));
}

extern "C" int t2c_kv_cache_write_paged(void *pages, const void *src, int64_t src_b_stride, int64_t src_t_stride,
                                        const int32_t *positions, const int32_t *block_table, int64_t bt_stride,
                                        int64_t num_pages, int64_t page_size, int64_t page_stride, int64_t row_stride,
                                        int64_t head_stride, int64_t B, int64_t T, int64_t NK, int64_t D, void *stream) {
    if (!pages || !src || !positions || !block_table) return set_error(T2C_EINVAL, "kv_cache_write_paged: NULL pointer");
    const int pl = page_log2_of(page_size);
    if (pl < 0) return set_error(T2C_EINVAL, "kv_cache_write_paged: page_size %lld is not a power of two", (long long)page_size);
    if (B <= 0 || T <= 0 || NK <= 0 || D <= 0 || D % 8 || bt_stride <= 0 || bt_stride * page_size > INT32_MAX ||
        num_pages <= 0 || num_pages > INT32_MAX)
        return set_error(T2C_EINVAL, "kv_cache_write_paged: bad shape");
    if (!aligned(pages, 16) || !aligned(src, 16) || page_stride % 8 || row_stride % 8 || head_stride % 8 ||
        src_b_stride % 8 || src_t_stride % 8)
        return set_error(T2C_EINVAL, "kv_cache_write_paged: rows must be 16-byte aligned");
    const int64_t total = B * T * NK * (D / 8);
    const int64_t blocks_needed = (total + 255) / 256;
    const int blocks = static_cast<int>(blocks_needed < 4096 ? blocks_needed : 4096);
    return launch(kv_write_paged_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, as_stream(stream),
                  static_cast<__half *>(pages), static_cast<const __half *>(src), src_b_stride, src_t_stride, positions,
                  block_table, bt_stride, pl, page_stride, row_stride, head_stride, static_cast<int>(B),
                  static_cast<int>(T), static_cast<int>(NK), static_cast<int>(D), static_cast<int>(bt_stride * page_size),
                  static_cast<int>(num_pages));
}

// ------------------------------------------------ decode attention, no allocation
// Fixed scratch for t2c_attn_decode_static: a file-scope device array that
// every GPU which loads this library holds until the process exits.
static constexpr int64_t kStaticAttnScratchFloats = 4 * 1024 * 1024;  // 16 MiB
static __device__ __align__(256) float g_static_attn_scratch[kStaticAttnScratchFloats];

// Device address of the array per device ordinal, resolved once.  It belongs
// to the device's primary context (the one the runtime API uses); after that
// context is destroyed (cudaDeviceReset) a process must not call
// t2c_attn_decode_static on that device again.
namespace {
std::mutex g_static_scratch_mutex;
float *g_static_scratch_ptr[64] = {nullptr};
}  // namespace

extern "C" int t2c_attn_decode_static(const void *q, const void *k_cache, const void *v_cache, void *out,
                                      const int32_t *positions, int64_t B, int64_t NH, int64_t NK, int64_t D,
                                      int64_t max_len, int64_t cb, int64_t cs, int64_t ch, int64_t splits,
                                      void *stream) {
    // Shape checks first, so that an unsupported split count is reported as
    // such and the scratch product below cannot overflow.
    if (B <= 0 || NH <= 0 || NK <= 0 || NH % NK || max_len <= 0 || splits <= 0)
        return set_error(T2C_EINVAL, "attn_decode_static: bad shape");
    if (D != 64 && D != 128) return set_error(T2C_EUNSUPPORTED, "attn_decode_static: head_dim %lld", (long long)D);
    if (splits > kMaxSplits)
        return set_error(T2C_EUNSUPPORTED, "attn_decode_static: splits %lld > %d", (long long)splits, kMaxSplits);
    if (B > kStaticAttnScratchFloats || NH > kStaticAttnScratchFloats || B * NH > kStaticAttnScratchFloats)
        return set_error(T2C_ESCRATCH, "attn_decode_static: B*NH = %lld*%lld exceeds the fixed scratch", (long long)B,
                         (long long)NH);
    const int64_t need = splits > 1 ? B * NH * splits * (D + 2) : 0;
    if (need > kStaticAttnScratchFloats) {
        return set_error(T2C_ESCRATCH,
                         "attn_decode_static: B*NH*splits*(D+2) = %lld floats exceeds the fixed scratch of %lld floats "
                         "(16 MiB); lower splits or use t2c_attn_decode with a caller workspace",
                         (long long)need, (long long)kStaticAttnScratchFloats);
    }
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "attn_decode_static: cudaGetDevice: %s", cudaGetErrorString(err));
    if (device < 0 || device >= 64) return set_error(T2C_EINVAL, "attn_decode_static: device %d out of range", device);
    float *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
        if (g_static_scratch_ptr[device] == nullptr) {
            // One-time set-up on this device (the device is current): the
            // host-side symbol is only a stand-in, so fetch the device address.
            void *ptr = nullptr;
            err = cudaGetSymbolAddress(&ptr, g_static_attn_scratch);
            if (err != cudaSuccess)
                return set_error(T2C_ECUDA, "attn_decode_static: cudaGetSymbolAddress: %s", cudaGetErrorString(err));
            g_static_scratch_ptr[device] = static_cast<float *>(ptr);
        }
        scratch = g_static_scratch_ptr[device];
    }
    return t2c_attn_decode(q, k_cache, v_cache, out, positions, B, NH, NK, D, max_len, cb, cs, ch, splits, scratch,
                           kStaticAttnScratchFloats, stream);
}

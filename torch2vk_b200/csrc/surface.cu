// Kernels that serve the remaining torch2vk shader contracts of the exported
// (unfused) Qwen3 graph: strided 4-D copies (slice / cat / transpose /
// contiguous views), broadcasting 4-D elementwise ops (add / mul / neg /
// silu), the RoPE cos/sin table, table-driven RMSNorm + RoPE, KV-cache
// writes at given positions, and the chunked greedy-select reduction.
#include <float.h>

#include "common.cuh"

namespace t2c {
namespace {

struct Shape4 {
    int64_t n[4];
    int64_t a[4];  // strides of operand a / src (elements)
    int64_t b[4];  // strides of operand b
    int64_t o[4];  // strides of the output / dst
};

__device__ __forceinline__ void unravel(int64_t i, const int64_t n[4], int64_t idx[4]) {
    idx[3] = i % n[3];
    i /= n[3];
    idx[2] = i % n[2];
    i /= n[2];
    idx[1] = i % n[1];
    idx[0] = i / n[1];
}

template <typename T>
__global__ void copy4d_kernel(const T *__restrict__ src, T *__restrict__ dst, Shape4 s, int64_t total) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t idx[4];
        unravel(i, s.n, idx);
        const int64_t si = idx[0] * s.a[0] + idx[1] * s.a[1] + idx[2] * s.a[2] + idx[3] * s.a[3];
        const int64_t di = idx[0] * s.o[0] + idx[1] * s.o[1] + idx[2] * s.o[2] + idx[3] * s.o[3];
        dst[di] = src[si];
    }
}

__device__ __forceinline__ float ld_f(const void *p, int64_t i, int f32) {
    return f32 ? static_cast<const float *>(p)[i] : __half2float(static_cast<const __half *>(p)[i]);
}
__device__ __forceinline__ void st_f(void *p, int64_t i, float v, int f32) {
    if (f32) {
        static_cast<float *>(p)[i] = v;
    } else {
        static_cast<__half *>(p)[i] = __float2half_rn(v);
    }
}

enum { EW_ADD = 0, EW_MUL = 1, EW_NEG = 2, EW_SILU = 3 };

__global__ void elementwise4d_kernel(int op, int f32, const void *__restrict__ a, const void *__restrict__ b,
                                     void *__restrict__ out, Shape4 s, int64_t total) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t idx[4];
        unravel(i, s.n, idx);
        const float x = ld_f(a, idx[0] * s.a[0] + idx[1] * s.a[1] + idx[2] * s.a[2] + idx[3] * s.a[3], f32);
        float r;
        if (op == EW_ADD || op == EW_MUL) {
            const float y = ld_f(b, idx[0] * s.b[0] + idx[1] * s.b[1] + idx[2] * s.b[2] + idx[3] * s.b[3], f32);
            r = op == EW_ADD ? x + y : x * y;
        } else if (op == EW_NEG) {
            r = -x;
        } else {
            r = x / (1.0f + __expf(-x));
        }
        st_f(out, idx[0] * s.o[0] + idx[1] * s.o[1] + idx[2] * s.o[2] + idx[3] * s.o[3], r, f32);
    }
}

// cos/sin [B, T, D] fp16: angle = (start + t) * theta^(-2 (d mod D/2) / D), times attention_scaling
// (src/torch2vk/runtime/rope_table.py:31-121 arithmetic); start read from start_dev when non-NULL.
template <typename OT>
__global__ void rope_table_kernel(OT *__restrict__ cos_out, OT *__restrict__ sin_out, int64_t B, int T, int D,
                                  float theta, int64_t start, const int64_t *__restrict__ start_dev, float scaling) {
    pdl_wait();
    pdl_trigger();
    if (start_dev) start = *start_dev;
    // grid-stride: the launch helper caps the grid
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < B * T * D;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t td = i % (static_cast<int64_t>(T) * D);
        const int t = static_cast<int>(td / D);
        const int d = static_cast<int>(td - static_cast<int64_t>(t) * D);
        const int f = d % (D / 2);
        const float exponent = (2.0f * static_cast<float>(f)) / static_cast<float>(D);
        const float inv_freq = powf(theta, -exponent);
        const float angle = static_cast<float>(start + t) * inv_freq;
        float sn, cs;
        sincosf(angle, &sn, &cs);
        cos_out[i] = static_cast<OT>(cs * scaling);
        sin_out[i] = static_cast<OT>(sn * scaling);
    }
}

// One warp per (b, t, g) row of D values: RMSNorm with fp32 weight, then
// rotate-half RoPE with fp16 cos/sin tables [B, T, D]; output addressed by
// strides (b, g, t) so head-major [B, G, T, D] or token-major layouts work.
template <int E, typename XT = __half, typename OT = __half>
__global__ void rms_norm_rope_kernel(const XT *__restrict__ x, const float *__restrict__ w,
                                     const __half *__restrict__ cos_t, const __half *__restrict__ sin_t,
                                     OT *__restrict__ out, int B, int T, int G, int64_t ob, int64_t og,
                                     int64_t ot, float eps) {
    constexpr int D = E * 32;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= static_cast<int64_t>(B) * T * G) return;
    pdl_wait();
    pdl_trigger();
    const int g = static_cast<int>(row % G);
    const int t = static_cast<int>((row / G) % T);
    const int b = static_cast<int>(row / (static_cast<int64_t>(G) * T));
    const int d0 = lane * E;
    float v[E];
    float ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        v[e] = static_cast<float>(x[row * D + d0 + e]);
        ss += v[e] * v[e];
    }
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / static_cast<float>(D) + eps);
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = v[e] * inv * w[d0 + e];
    const int64_t trow = (static_cast<int64_t>(b) * T + t) * D;
    OT *o = out + b * ob + g * og + t * ot;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        const float c = __half2float(cos_t[trow + d0 + e]), s = __half2float(sin_t[trow + d0 + e]);
        o[d0 + e] = static_cast<OT>(lane < 16 ? v[e] * c - partner * s : v[e] * c + partner * s);
    }
}

// Mixed-precision elementwise steps of an unfused RMSNorm chain (the exported ASR text norm):
// POW2 a*a, RSQRT 1/sqrt(a), ADD_SCALAR a + scalar, MUL_ROW a[i] * b[i / H], MUL_COL a[i] * b[i % H].
// Operand / output dtypes by flag (1 = fp16, 0 = fp32); arithmetic in fp32.
enum { EM_POW2 = 0, EM_RSQRT = 1, EM_ADD_SCALAR = 2, EM_MUL_ROW = 3, EM_MUL_COL = 4 };
__global__ void ew_misc_kernel(int op, const void *__restrict__ a, int a16, const void *__restrict__ b, int b16,
                               void *__restrict__ out, int o16, int64_t n, int64_t H, float scalar) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float x = ld_f(a, i, !a16);
        float r;
        switch (op) {
            case EM_POW2: r = x * x; break;
            case EM_RSQRT: r = rsqrtf(x); break;
            case EM_ADD_SCALAR: r = x + scalar; break;
            case EM_MUL_ROW: r = x * ld_f(b, i / H, !b16); break;
            default: r = x * ld_f(b, i % H, !b16); break;
        }
        st_f(out, i, r, !o16);
    }
}

// out[r] = mean of row r of x [rows, cols] (fp32), one warp per row
__global__ void row_mean_f32_kernel(const float *__restrict__ x, float *__restrict__ out, int64_t rows, int64_t cols) {
    pdl_wait();
    pdl_trigger();
    const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    float sum = 0.0f;
    for (int64_t c = lane; c < cols; c += 32) sum += x[r * cols + c];
    sum = warp_sum(sum);
    if (lane == 0) out[r] = sum / static_cast<float>(cols);
}

// ------------------------------------------- fp32-activation prefill programs
// y = x * rsqrt(mean(x^2) + eps) * w, fp32 in and out, one CTA of 256 threads per row
// (rms_norm_mul_f32.py: fp32 sum of squares, fp32 output).
__global__ void rms_norm_f32_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ y,
                                    int H, float eps) {
    __shared__ float part[8];
    pdl_wait();
    pdl_trigger();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * H;
    const bool vec = (H % 4) == 0;
    float ss = 0.0f;
    if (vec) {
        for (int h = threadIdx.x * 4; h < H; h += 1024) {
            const float4 v = *reinterpret_cast<const float4 *>(x + base + h);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
    } else {
        for (int h = threadIdx.x; h < H; h += 256) ss = fmaf(x[base + h], x[base + h], ss);
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) total += part[i];
    const float inv = rsqrtf(total / static_cast<float>(H) + eps);
    if (vec) {
        for (int h = threadIdx.x * 4; h < H; h += 1024) {
            const float4 v = *reinterpret_cast<const float4 *>(x + base + h);
            const float4 g = *reinterpret_cast<const float4 *>(w + h);
            *reinterpret_cast<float4 *>(y + base + h) = make_float4(v.x * inv * g.x, v.y * inv * g.y, v.z * inv * g.z, v.w * inv * g.w);
        }
    } else {
        for (int h = threadIdx.x; h < H; h += 256) y[base + h] = x[base + h] * inv * w[h];
    }
}

enum { BIN_ADD = 0, BIN_SWIGLU = 1 };

// out = a + b, or silu(a) * b (= a / (1 + exp(-a)) * b), fp32, 4 values per thread
__global__ void binary_f32_kernel(int op, const float *__restrict__ a, const float *__restrict__ b,
                                  float *__restrict__ out, int64_t n) {
    pdl_wait();
    pdl_trigger();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x * 4;
    for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n; i += stride) {
        if (i + 4 <= n) {
            const float4 x = *reinterpret_cast<const float4 *>(a + i);
            const float4 y = *reinterpret_cast<const float4 *>(b + i);
            float4 r;
            if (op == BIN_ADD) {
                r = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
            } else {
                r = make_float4(x.x / (1.0f + expf(-x.x)) * y.x, x.y / (1.0f + expf(-x.y)) * y.y,
                                x.z / (1.0f + expf(-x.z)) * y.z, x.w / (1.0f + expf(-x.w)) * y.w);
            }
            *reinterpret_cast<float4 *>(out + i) = r;
        } else {
            for (int64_t j = i; j < n; ++j)
                out[j] = op == BIN_ADD ? a[j] + b[j] : a[j] / (1.0f + expf(-a[j])) * b[j];
        }
    }
}

template <typename S, typename D>
__global__ void cast_kernel(const S *__restrict__ x, D *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = static_cast<D>(static_cast<float>(x[i]));
}

// out[b, 0, h] = fp16(x[b, S - 1, h])
__global__ void slice_last_f32_kernel(const float *__restrict__ x, __half *__restrict__ out, int B, int64_t S, int H) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = static_cast<int64_t>(B) * H;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / H, h = i % H;
        out[i] = __float2half_rn(x[(b * S + (S - 1)) * H + h]);
    }
}

// Token-major value caches [B, S_c, H, D] (up to 3) receive fp16(src[b, t, h, d]) at row
// positions[t]; a cache whose extent S_c does not reach that row is skipped (as the reference).
struct CacheSet {
    __half *c[3];
    int64_t S[3];
    int n;
};
__global__ void value_cache_write_f32_kernel(const float *__restrict__ src, const int64_t *__restrict__ positions,
                                             CacheSet cs, int B, int T, int H, int D) {
    pdl_wait();
    pdl_trigger();
    const int64_t total = static_cast<int64_t>(B) * T * H * D;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t r = i;
        const int d = static_cast<int>(r % D);
        r /= D;
        const int h = static_cast<int>(r % H);
        r /= H;
        const int t = static_cast<int>(r % T);
        const int64_t b = r / T;
        const int64_t pos = positions[t];
        const __half v = __float2half_rn(src[i]);
        for (int k = 0; k < cs.n; ++k)
            if (pos >= 0 && pos < cs.S[k]) cs.c[k][((b * cs.S[k] + pos) * H + h) * D + d] = v;
    }
}

// Flash-attention mask classifier (fa_mask_opt_f16.py): for the 16 blocks of 16 rows x 64
// columns that output word (row block r, word w) covers, 2 bits each: 1 = every value
// <= -FLT_MAX / 2 (or the block lies outside the mask), 2 = every value == 0.
__global__ void fa_mask_opt_kernel(const __half *__restrict__ mask, uint32_t *__restrict__ out, int T, int64_t S,
                                   int64_t row_stride, int64_t out_row_stride) {
    pdl_wait();
    pdl_trigger();
    const int word = blockIdx.x, rb = blockIdx.y;
    const float big = 1.7014117e38f;
    __shared__ float smin[4], smax[4];
    uint32_t result = 0;
    for (int bx = 0; bx < 16; ++bx) {
        float mn = big, mx = -big;
        for (int idx = threadIdx.x; idx < 16 * 64; idx += blockDim.x) {
            const int64_t col = (idx & 63) + (static_cast<int64_t>(word) * 16 + bx) * 64;
            const int row = (idx >> 6) + rb * 16;
            if (col < S && row < T) {
                const float v = __half2float(mask[row * row_stride + col]);
                mn = fminf(mn, v);
                mx = fmaxf(mx, v);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        }
        if ((threadIdx.x & 31) == 0) {
            smin[threadIdx.x >> 5] = mn;
            smax[threadIdx.x >> 5] = mx;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) {
                mn = fminf(mn, smin[i]);
                mx = fmaxf(mx, smax[i]);
            }
            if (mx <= -big) result |= 1u << (2 * bx);
            if (mn == 0.0f && mx == 0.0f) result |= 2u << (2 * bx);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) out[static_cast<int64_t>(rb) * out_row_stride + word] = result;
}

// cache[b, pos_t, h, :] = src[b, t, h, :] with pos_t = positions[t] (int64) or `position` + t.
__global__ void kv_write_kernel(__half *__restrict__ cache, const __half *__restrict__ src,
                                const int64_t *__restrict__ positions, int64_t position, int B, int H, int T, int D,
                                int64_t cb, int64_t cs, int64_t ch, int64_t sb, int64_t st, int64_t sh, int64_t S) {
    pdl_wait();
    pdl_trigger();
    // grid-stride: the launch helper caps the grid
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < static_cast<int64_t>(B) * H * T * D;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(i % D);
        int64_t r = i / D;
        const int t = static_cast<int>(r % T);
        r /= T;
        const int h = static_cast<int>(r % H);
        const int b = static_cast<int>(r / H);
        const int64_t pos = positions ? positions[t] : position + t;
        if (pos < 0 || pos >= S) {
            report_device_error(T2C_EINVAL);
            continue;
        }
        cache[b * cb + pos * cs + h * ch + d] = src[b * sb + t * st + h * sh + d];
    }
}

__device__ __forceinline__ bool better(float s, uint32_t t, float bs, uint32_t bt) {
    return s > bs || (s == bs && t < bt);
}

// One CTA of 1024 threads per chunk of 1024 partials
// (qwen3_token_select_reduce_f32.py:21-148 chunk stage).
__global__ void __launch_bounds__(1024) select_chunks_kernel(const float *__restrict__ scores,
                                                             const uint32_t *__restrict__ tokens, int64_t G,
                                                             float *__restrict__ cs, uint32_t *__restrict__ ct) {
    __shared__ float ss[32];
    __shared__ uint32_t st[32];
    pdl_wait();
    pdl_trigger();
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 1024 + threadIdx.x;
    float best = i < G ? scores[i] : -FLT_MAX;
    uint32_t tok = i < G ? tokens[i] : 0xffffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float s = __shfl_xor_sync(0xffffffffu, best, o);
        const uint32_t t = __shfl_xor_sync(0xffffffffu, tok, o);
        if (better(s, t, best, tok)) {
            best = s;
            tok = t;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        ss[threadIdx.x >> 5] = best;
        st[threadIdx.x >> 5] = tok;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 32; ++w)
            if (better(ss[w], st[w], best, tok)) {
                best = ss[w];
                tok = st[w];
            }
        cs[blockIdx.x] = best;
        ct[blockIdx.x] = tok;
    }
}

template <typename Kernel, typename... Args>
int launch(Kernel kernel, int64_t threads_total, int block, cudaStream_t stream, Args... args) {
    int64_t grid = (threads_total + block - 1) / block;
    if (grid < 1) grid = 1;
    if (grid > 148LL * 64) grid = 148LL * 64;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(block);
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

int fill_shape(Shape4 &s, const int64_t *shape, const int64_t *a, const int64_t *b, const int64_t *o, int64_t &total) {
    total = 1;
    for (int i = 0; i < 4; ++i) {
        if (shape[i] < 0) return set_error(T2C_EINVAL, "negative extent");
        s.n[i] = shape[i] > 0 ? shape[i] : 1;
        s.a[i] = a ? a[i] : 0;
        s.b[i] = b ? b[i] : 0;
        s.o[i] = o[i];
        total *= shape[i];
    }
    return T2C_OK;
}

}  // namespace

cudaError_t status_surface(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c

using namespace t2c;

extern "C" int t2c_copy4d(int elem_bytes, const void *src, const int64_t *src_strides, void *dst,
                          const int64_t *dst_strides, const int64_t *shape, void *stream) {
    if (!src || !dst || !src_strides || !dst_strides || !shape) return set_error(T2C_EINVAL, "copy4d: NULL pointer");
    Shape4 s;
    int64_t total = 0;
    int rc = fill_shape(s, shape, src_strides, nullptr, dst_strides, total);
    if (rc) return rc;
    if (total == 0) return T2C_OK;
    const cudaStream_t st = as_stream(stream);
    switch (elem_bytes) {
        case 2: return launch(copy4d_kernel<uint16_t>, total, 256, st, static_cast<const uint16_t *>(src),
                              static_cast<uint16_t *>(dst), s, total);
        case 4: return launch(copy4d_kernel<uint32_t>, total, 256, st, static_cast<const uint32_t *>(src),
                              static_cast<uint32_t *>(dst), s, total);
        case 8: return launch(copy4d_kernel<uint64_t>, total, 256, st, static_cast<const uint64_t *>(src),
                              static_cast<uint64_t *>(dst), s, total);
        case 1: return launch(copy4d_kernel<uint8_t>, total, 256, st, static_cast<const uint8_t *>(src),
                              static_cast<uint8_t *>(dst), s, total);
        default: return set_error(T2C_EUNSUPPORTED, "copy4d: element size %d", elem_bytes);
    }
}

extern "C" int t2c_elementwise4d(int op, int is_f32, const void *a, const int64_t *a_strides, const void *b,
                                 const int64_t *b_strides, void *out, const int64_t *out_strides, const int64_t *shape,
                                 void *stream) {
    if (!a || !out || !a_strides || !out_strides || !shape) return set_error(T2C_EINVAL, "elementwise4d: NULL pointer");
    if (op < EW_ADD || op > EW_SILU) return set_error(T2C_EINVAL, "elementwise4d: op %d", op);
    if ((op == EW_ADD || op == EW_MUL) && (!b || !b_strides)) return set_error(T2C_EINVAL, "elementwise4d: b is NULL");
    Shape4 s;
    int64_t total = 0;
    int rc = fill_shape(s, shape, a_strides, b_strides, out_strides, total);
    if (rc) return rc;
    if (total == 0) return T2C_OK;
    return launch(elementwise4d_kernel, total, 256, as_stream(stream), op, is_f32, a, b, out, s, total);
}

extern "C" int t2c_rope_table(void *cos_out, void *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                              int64_t start_position, float attention_scaling, void *stream) {
    if (!cos_out || !sin_out || B <= 0 || T <= 0 || D <= 0 || D % 2) return set_error(T2C_EINVAL, "rope_table: bad arguments");
    return launch(rope_table_kernel<__half>, B * T * D, 256, as_stream(stream), static_cast<__half *>(cos_out),
                  static_cast<__half *>(sin_out), B, static_cast<int>(T), static_cast<int>(D), theta, start_position,
                  static_cast<const int64_t *>(nullptr), attention_scaling);
}

extern "C" int t2c_rms_norm_rope(const void *x, const float *w, const void *cos_t, const void *sin_t, void *out,
                                 int64_t B, int64_t T, int64_t G, int64_t D, int64_t out_b_stride, int64_t out_g_stride,
                                 int64_t out_t_stride, float eps, void *stream) {
    if (!x || !w || !cos_t || !sin_t || !out) return set_error(T2C_EINVAL, "rms_norm_rope: NULL pointer");
    if (B <= 0 || T <= 0 || G <= 0) return set_error(T2C_EINVAL, "rms_norm_rope: bad shape");
    const int64_t rows = B * T * G;
    const int warps = 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((rows + warps - 1) / warps));
    cfg.blockDim = dim3(warps * 32);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err;
    const __half *xp = static_cast<const __half *>(x);
    const __half *cp = static_cast<const __half *>(cos_t);
    const __half *sp = static_cast<const __half *>(sin_t);
    __half *op = static_cast<__half *>(out);
    if (D == 128) {
        err = cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<4>, xp, w, cp, sp, op, static_cast<int>(B), static_cast<int>(T),
                                 static_cast<int>(G), out_b_stride, out_g_stride, out_t_stride, eps);
    } else if (D == 64) {
        err = cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<2>, xp, w, cp, sp, op, static_cast<int>(B), static_cast<int>(T),
                                 static_cast<int>(G), out_b_stride, out_g_stride, out_t_stride, eps);
    } else {
        return set_error(T2C_EUNSUPPORTED, "rms_norm_rope: D=%lld", (long long)D);
    }
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "rms_norm_rope: %s", cudaGetErrorString(err));
    return T2C_OK;
}

extern "C" int t2c_kv_cache_write(void *cache, const void *src, const int64_t *positions, int64_t position, int64_t B,
                                  int64_t H, int64_t T, int64_t D, int64_t S, int64_t cache_b_stride,
                                  int64_t cache_s_stride, int64_t cache_h_stride, int64_t src_b_stride,
                                  int64_t src_t_stride, int64_t src_h_stride, void *stream) {
    if (!cache || !src) return set_error(T2C_EINVAL, "kv_cache_write: NULL pointer");
    if (B <= 0 || H <= 0 || T <= 0 || D <= 0 || S <= 0) return set_error(T2C_EINVAL, "kv_cache_write: bad shape");
    if (!positions && (position < 0 || position + T > S))
        return set_error(T2C_EINVAL, "kv_cache_write: position %lld + %lld outside cache of %lld", (long long)position,
                         (long long)T, (long long)S);
    return launch(kv_write_kernel, B * H * T * D, 256, as_stream(stream), static_cast<__half *>(cache),
                  static_cast<const __half *>(src), positions, position, static_cast<int>(B), static_cast<int>(H),
                  static_cast<int>(T), static_cast<int>(D), cache_b_stride, cache_s_stride, cache_h_stride,
                  src_b_stride, src_t_stride, src_h_stride, S);
}

extern "C" int t2c_token_select_chunks(const float *scores, const uint32_t *tokens, int64_t G, float *chunk_scores,
                                       uint32_t *chunk_tokens, void *stream) {
    if (!scores || !tokens || !chunk_scores || !chunk_tokens || G <= 0)
        return set_error(T2C_EINVAL, "token_select_chunks: bad arguments");
    const int64_t chunks = (G + 1023) / 1024;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(chunks));
    cfg.blockDim = dim3(1024);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err = cudaLaunchKernelEx(&cfg, select_chunks_kernel, scores, tokens, G, chunk_scores, chunk_tokens);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "token_select_chunks: %s", cudaGetErrorString(err));
    return T2C_OK;
}

extern "C" int t2c_rms_norm_f32(const float *x, const float *w, float *y, int64_t rows, int64_t H, float eps,
                                void *stream) {
    if (!x || !w || !y) return set_error(T2C_EINVAL, "rms_norm_f32: NULL pointer");
    if (rows <= 0 || H <= 0 || H > INT32_MAX) return set_error(T2C_EINVAL, "rms_norm_f32: bad shape");
    if (H % 4 == 0 && (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16 ||
                       reinterpret_cast<uintptr_t>(w) % 16))
        return set_error(T2C_EINVAL, "rms_norm_f32: rows must be 16-byte aligned");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(rows));
    cfg.blockDim = dim3(256);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, rms_norm_f32_kernel, x, w, y, static_cast<int>(H), eps);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "rms_norm_f32: %s", cudaGetErrorString(err));
    return T2C_OK;
}

extern "C" int t2c_rms_norm_rope_f32(const float *x, const float *w, const void *cos_t, const void *sin_t, void *out,
                                     int out_f32, int64_t B, int64_t T, int64_t G, int64_t D, float eps, void *stream) {
    if (!x || !w || !cos_t || !sin_t || !out) return set_error(T2C_EINVAL, "rms_norm_rope_f32: NULL pointer");
    if (B <= 0 || T <= 0 || G <= 0) return set_error(T2C_EINVAL, "rms_norm_rope_f32: bad shape");
    if (D != 128 && D != 64) return set_error(T2C_EUNSUPPORTED, "rms_norm_rope_f32: D=%lld", (long long)D);
    const int64_t rows = B * T * G;
    const int warps = 8;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((rows + warps - 1) / warps));
    cfg.blockDim = dim3(warps * 32);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // token-major output [B, T, G, D]
    const int64_t ob = T * G * D, og = D, ot = G * D;
    const __half *cp = static_cast<const __half *>(cos_t);
    const __half *sp = static_cast<const __half *>(sin_t);
    const int b = static_cast<int>(B), t = static_cast<int>(T), g = static_cast<int>(G);
    cudaError_t err;
    if (D == 128) {
        err = out_f32 ? cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<4, float, float>, x, w, cp, sp,
                                           static_cast<float *>(out), b, t, g, ob, og, ot, eps)
                      : cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<4, float, __half>, x, w, cp, sp,
                                           static_cast<__half *>(out), b, t, g, ob, og, ot, eps);
    } else {
        err = out_f32 ? cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<2, float, float>, x, w, cp, sp,
                                           static_cast<float *>(out), b, t, g, ob, og, ot, eps)
                      : cudaLaunchKernelEx(&cfg, rms_norm_rope_kernel<2, float, __half>, x, w, cp, sp,
                                           static_cast<__half *>(out), b, t, g, ob, og, ot, eps);
    }
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "rms_norm_rope_f32: %s", cudaGetErrorString(err));
    return T2C_OK;
}

extern "C" int t2c_binary_f32(int op, const float *a, const float *b, float *out, int64_t n, void *stream) {
    if (!a || !b || !out || n < 0) return set_error(T2C_EINVAL, "binary_f32: bad arguments");
    if (op != BIN_ADD && op != BIN_SWIGLU) return set_error(T2C_EINVAL, "binary_f32: op %d", op);
    if (reinterpret_cast<uintptr_t>(a) % 16 || reinterpret_cast<uintptr_t>(b) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
        return set_error(T2C_EINVAL, "binary_f32: operands must be 16-byte aligned");
    if (n == 0) return T2C_OK;
    return launch(binary_f32_kernel, (n + 3) / 4, 256, as_stream(stream), op, a, b, out, n);
}

extern "C" int t2c_cast(const void *x, int x_dtype, void *y, int y_dtype, int64_t n, void *stream) {
    if (!x || !y || n < 0) return set_error(T2C_EINVAL, "cast: bad arguments");
    if (n == 0) return T2C_OK;
    const cudaStream_t s = as_stream(stream);
    if (x_dtype == T2C_F32 && y_dtype == T2C_F16)
        return launch(cast_kernel<float, __half>, n, 256, s, static_cast<const float *>(x), static_cast<__half *>(y), n);
    if (x_dtype == T2C_F16 && y_dtype == T2C_F32)
        return launch(cast_kernel<__half, float>, n, 256, s, static_cast<const __half *>(x), static_cast<float *>(y), n);
    return set_error(T2C_EUNSUPPORTED, "cast: dtypes %d -> %d", x_dtype, y_dtype);
}

extern "C" int t2c_slice_last_f32_to_f16(const float *x, void *out, int64_t B, int64_t S, int64_t H, void *stream) {
    if (!x || !out || B <= 0 || S <= 0 || H <= 0 || H > INT32_MAX) return set_error(T2C_EINVAL, "slice_last: bad arguments");
    return launch(slice_last_f32_kernel, B * H, 256, as_stream(stream), x, static_cast<__half *>(out),
                  static_cast<int>(B), S, static_cast<int>(H));
}

extern "C" int t2c_value_cache_write_f32(const float *src, const int64_t *positions, int ncaches, void *const *caches,
                                         const int64_t *cache_lens, int64_t B, int64_t T, int64_t H, int64_t D,
                                         void *stream) {
    if (!src || !positions || !caches || !cache_lens || ncaches < 1 || ncaches > 3)
        return set_error(T2C_EINVAL, "value_cache_write_f32: bad arguments");
    if (B <= 0 || T <= 0 || H <= 0 || D <= 0) return set_error(T2C_EINVAL, "value_cache_write_f32: bad shape");
    CacheSet cs = {};
    cs.n = ncaches;
    for (int i = 0; i < ncaches; ++i) {
        if (!caches[i] || cache_lens[i] <= 0) return set_error(T2C_EINVAL, "value_cache_write_f32: cache %d", i);
        cs.c[i] = static_cast<__half *>(caches[i]);
        cs.S[i] = cache_lens[i];
    }
    return launch(value_cache_write_f32_kernel, B * T * H * D, 256, as_stream(stream), src, positions, cs,
                  static_cast<int>(B), static_cast<int>(T), static_cast<int>(H), static_cast<int>(D));
}

extern "C" int t2c_fa_mask_opt(const void *mask, uint32_t *out, int64_t T, int64_t S, int64_t words, int64_t row_blocks,
                               void *stream) {
    if (!mask || !out || T <= 0 || S <= 0 || words <= 0 || row_blocks <= 0)
        return set_error(T2C_EINVAL, "fa_mask_opt: bad arguments");
    if (words > 65535 || row_blocks > 65535) return set_error(T2C_EINVAL, "fa_mask_opt: grid too large");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(words), static_cast<unsigned>(row_blocks));
    cfg.blockDim = dim3(128);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, fa_mask_opt_kernel, static_cast<const __half *>(mask), out,
                                               static_cast<int>(T), S, S, words);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "fa_mask_opt: %s", cudaGetErrorString(err));
    return T2C_OK;
}

extern "C" int t2c_rope_table_f32(float *cos_out, float *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                                  int64_t start_position, float attention_scaling, void *stream) {
    if (!cos_out || !sin_out || B <= 0 || T <= 0 || D <= 0 || D % 2) return set_error(T2C_EINVAL, "rope_table_f32: bad arguments");
    return launch(rope_table_kernel<float>, B * T * D, 256, as_stream(stream), cos_out, sin_out, B, static_cast<int>(T),
                  static_cast<int>(D), theta, start_position, static_cast<const int64_t *>(nullptr), attention_scaling);
}

extern "C" int t2c_rope_table_dev(void *cos_out, void *sin_out, int64_t B, int64_t T, int64_t D, float theta,
                                  const int64_t *start_position_dev, float attention_scaling, int out_f32,
                                  void *stream) {
    if (!cos_out || !sin_out || !start_position_dev || B <= 0 || T <= 0 || D <= 0 || D % 2)
        return set_error(T2C_EINVAL, "rope_table_dev: bad arguments");
    if (out_f32)
        return launch(rope_table_kernel<float>, B * T * D, 256, as_stream(stream), static_cast<float *>(cos_out),
                      static_cast<float *>(sin_out), B, static_cast<int>(T), static_cast<int>(D), theta, int64_t{0},
                      start_position_dev, attention_scaling);
    return launch(rope_table_kernel<__half>, B * T * D, 256, as_stream(stream), static_cast<__half *>(cos_out),
                  static_cast<__half *>(sin_out), B, static_cast<int>(T), static_cast<int>(D), theta, int64_t{0},
                  start_position_dev, attention_scaling);
}

extern "C" int t2c_ew_misc(int op, const void *a, int a_f16, const void *b, int b_f16, void *out, int out_f16, int64_t n,
                           int64_t H, float scalar, void *stream) {
    if (!a || !out || n < 0 || op < EM_POW2 || op > EM_MUL_COL) return set_error(T2C_EINVAL, "ew_misc: bad arguments");
    if ((op == EM_MUL_ROW || op == EM_MUL_COL) && (!b || H <= 0)) return set_error(T2C_EINVAL, "ew_misc: b / H");
    if (n == 0) return T2C_OK;
    return launch(ew_misc_kernel, n, 256, as_stream(stream), op, a, a_f16, b, b_f16, out, out_f16, n, H, scalar);
}

extern "C" int t2c_row_mean_f32(const float *x, float *out, int64_t rows, int64_t cols, void *stream) {
    if (!x || !out || rows <= 0 || cols <= 0) return set_error(T2C_EINVAL, "row_mean_f32: bad arguments");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((rows + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = as_stream(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, row_mean_f32_kernel, x, out, rows, cols);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "row_mean_f32: %s", cudaGetErrorString(err));
    return T2C_OK;
}

// Kernels of the Qwen3-ASR audio encoder (quantized_qwen3_asr, config 5):
// Q8_0-weight linears and 3x3 stride-2 convolutions as one tensor-core GEMM
// (mma.m16n8k16, fp16 operands, fp32 accumulation, fp32 bias and optional
// GELU in the epilogue), LayerNorm, GELU, row gather and windowed
// (additive-mask) attention.  Activations are fp16 throughout, as in the
// reference's exported encoder (models/quantized_qwen3_asr/dispatch/audio_encoder.py).
#include <float.h>

#include "common.cuh"
#include "qgemm.cuh"

namespace t2c {
namespace {

__device__ __forceinline__ void ldsm4(uint32_t r[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4_t(uint32_t r[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ float4 h4_to_f4_c(uint2 v) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
    return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f)); }

// ------------------------------------------------------- Q8_0 GEMM / conv
// y[m, n] = sum_k A[m, k] * d[n, k/32] * q[n, k] + bias[n]  (optional GELU).
// LINEAR: A = x [M, K] row-major.  CONV: A is the implicit im2col of an NCHW
// input, m = (b, oh, ow), k = (ic, fh, fw), with zero padding; the output is
// written NCHW (n = output channel).  CTA = 4 warps on a 64 x 64 (m, n) tile;
// K advances one Q8_0 block (32 values) at a time through two shared-memory
// buffers (the next block is loaded into registers while the current one is
// multiplied).  Weights are dequantized to fp16 (d * q rounded once).
struct Q8Gemm {
    const __half *x;
    const uint8_t *w;
    const float *bias;
    __half *y;
    int M, N, K, nblk;
    int64_t row_bytes;
    int act;
    int Ci, Hi, Wi, Ho, Wo, kh, kw, sh, sw, ph, pw;
    int out_cl;  // CONV: output [B, Ho, Wo, N] (channels last) instead of [B, N, Ho, Wo]
};
constexpr int kQT = 64;
constexpr int kQRow = 40;  // halves per shared row (80 B: conflict-free ldmatrix rows)

template <bool CONV>
__global__ void __launch_bounds__(128) q8_gemm_kernel(const Q8Gemm p) {
    __shared__ __align__(16) __half As[2][kQT][kQRow];
    __shared__ __align__(16) __half Bs[2][kQT][kQRow];
    __shared__ int pix[kQT][3];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int m0 = blockIdx.x * kQT, n0 = blockIdx.y * kQT;
    const int wm = (warp & 1) * 32, wn = (warp >> 1) * 32;
    pdl_wait();
    pdl_trigger();
    if (CONV) {
        if (tid < kQT) {
            const int m = m0 + tid;
            if (m < p.M) {
                const int hw = p.Ho * p.Wo;
                const int b = m / hw, r = m - b * hw, oh = r / p.Wo, ow = r - oh * p.Wo;
                pix[tid][0] = b * p.Ci * p.Hi * p.Wi;
                pix[tid][1] = oh * p.sh - p.ph;
                pix[tid][2] = ow * p.sw - p.pw;
            } else {
                pix[tid][0] = -1;
            }
        }
        __syncthreads();
    }
    // per-thread register stage of one K block
    uint4 av[2];
    __half ac[16];
    uint32_t bq[8];
    float bd = 0.0f;
    const int brow = tid >> 1, bhf = tid & 1;
    auto load = [&](int kb) {
        const int k0 = kb * 32;
        if (CONV) {
            const int kk = tid & 31, k = k0 + kk;
            const bool kin = k < p.K;
            int ic = 0, fh = 0, fw = 0;
            if (kin) {
                const int khw = p.kh * p.kw;
                ic = k / khw;
                const int rem = k - ic * khw;
                fh = rem / p.kw;
                fw = rem - fh * p.kw;
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int row = (tid >> 5) + 4 * j;
                __half v = __float2half(0.0f);
                const int pb = pix[row][0];
                if (kin && pb >= 0) {
                    const int ih = pix[row][1] + fh, iw = pix[row][2] + fw;
                    if (ih >= 0 && ih < p.Hi && iw >= 0 && iw < p.Wi) v = p.x[pb + (ic * p.Hi + ih) * p.Wi + iw];
                }
                ac[j] = v;
            }
        } else {
            const int m = m0 + brow;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int k = k0 + 16 * bhf + 8 * j;
                av[j] = (m < p.M && k + 8 <= p.K)
                            ? *reinterpret_cast<const uint4 *>(p.x + static_cast<int64_t>(m) * p.K + k)
                            : make_uint4(0u, 0u, 0u, 0u);
            }
        }
        const int n = n0 + brow;
        if (n < p.N) {
            const uint8_t *blk = p.w + static_cast<int64_t>(n) * p.row_bytes + static_cast<int64_t>(kb) * 34;
            bd = half_bits_to_float(*reinterpret_cast<const unsigned short *>(blk));
            const unsigned short *qs = reinterpret_cast<const unsigned short *>(blk + 2 + 16 * bhf);
#pragma unroll
            for (int j = 0; j < 8; ++j) bq[j] = qs[j];
        } else {
            bd = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) bq[j] = 0u;
        }
    };
    auto store = [&](int buf) {
        if (CONV) {
#pragma unroll
            for (int j = 0; j < 16; ++j) As[buf][(tid >> 5) + 4 * j][tid & 31] = ac[j];
        } else {
            *reinterpret_cast<uint4 *>(&As[buf][brow][16 * bhf]) = av[0];
            *reinterpret_cast<uint4 *>(&As[buf][brow][16 * bhf + 8]) = av[1];
        }
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float lo = bd * static_cast<float>(static_cast<int8_t>(bq[j] & 0xffu));
            const float hi = bd * static_cast<float>(static_cast<int8_t>(bq[j] >> 8));
            const __half2 hv = __floats2half2_rn(lo, hi);
            h[j] = *reinterpret_cast<const uint32_t *>(&hv);
        }
        *reinterpret_cast<uint4 *>(&Bs[buf][brow][16 * bhf]) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4 *>(&Bs[buf][brow][16 * bhf + 8]) = make_uint4(h[4], h[5], h[6], h[7]);
    };
    float acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
    load(0);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int kb = 0; kb < p.nblk; ++kb) {
        if (kb + 1 < p.nblk) load(kb + 1);
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t a[2][4], b[2][4];
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) ldsm4(a[mi], &As[buf][wm + 16 * mi + (lane & 15)][16 * ks + 8 * (lane >> 4)]);
#pragma unroll
            for (int np = 0; np < 2; ++np)
                ldsm4(b[np], &Bs[buf][wn + 16 * np + (lane & 7) + 8 * (lane >> 4)][16 * ks + 8 * ((lane >> 3) & 1)]);
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    mma16816(acc[mi][2 * np], a[mi], b[np][0], b[np][1]);
                    mma16816(acc[mi][2 * np + 1], a[mi], b[np][2], b[np][3]);
                }
        }
        if (kb + 1 < p.nblk) store(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m0 + wm + 16 * mi + g + 8 * (e >> 1);
                const int n = n0 + wn + 8 * ni + 2 * t4 + (e & 1);
                if (m >= p.M || n >= p.N) continue;
                float v = acc[mi][ni][e] + (p.bias ? p.bias[n] : 0.0f);
                if (p.act) v = gelu_erf(v);
                if (CONV && !p.out_cl) {
                    const int hw = p.Ho * p.Wo;
                    const int b = m / hw, r = m - b * hw;
                    p.y[(static_cast<int64_t>(b) * p.N + n) * hw + r] = __float2half_rn(v);
                } else {
                    p.y[static_cast<int64_t>(m) * p.N + n] = __float2half_rn(v);
                }
            }
}

// ---------------------------------------------------------------- LayerNorm
// One CTA per row (cols <= 4096, a multiple of 8): y = (x - mean) / sqrt(var + eps) * w + b,
// mean and variance of the fp32 values (two passes over registers).
constexpr int kLnThreads = 256;
__global__ void __launch_bounds__(kLnThreads) layer_norm_kernel(const __half *__restrict__ x, const float *__restrict__ w,
                                                                const float *__restrict__ bias, __half *__restrict__ y,
                                                                int cols, float eps, int y_stride) {
    __shared__ float part[kLnThreads / 32];
    __shared__ float stat;
    const int64_t row = blockIdx.x;
    const int tid = threadIdx.x, nv = cols / 8;
    pdl_wait();
    pdl_trigger();
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * cols);
    float f[2][8];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = tid + i * kLnThreads;
        const uint4 v = c < nv ? xr[c] : make_uint4(0u, 0u, 0u, 0u);
        const float4 a = h4_to_f4_c(make_uint2(v.x, v.y)), b = h4_to_f4_c(make_uint2(v.z, v.w));
        f[i][0] = a.x; f[i][1] = a.y; f[i][2] = a.z; f[i][3] = a.w;
        f[i][4] = b.x; f[i][5] = b.y; f[i][6] = b.z; f[i][7] = b.w;
#pragma unroll
        for (int e = 0; e < 8; ++e) s += f[i][e];
    }
    s = warp_sum(s);
    if ((tid & 31) == 0) part[tid >> 5] = s;
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int i = 0; i < kLnThreads / 32; ++i) t += part[i];
        stat = t / static_cast<float>(cols);
    }
    __syncthreads();
    const float mean = stat;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = tid + i * kLnThreads;
        if (c < nv) {
#pragma unroll
            for (int e = 0; e < 8; ++e) q += (f[i][e] - mean) * (f[i][e] - mean);
        }
    }
    q = warp_sum(q);
    __syncthreads();
    if ((tid & 31) == 0) part[tid >> 5] = q;
    __syncthreads();
    if (tid == 0) {
        float t = 0.0f;
        for (int i = 0; i < kLnThreads / 32; ++i) t += part[i];
        stat = rsqrtf(t / static_cast<float>(cols) + eps);
    }
    __syncthreads();
    const float inv = stat;
    uint4 *yr = reinterpret_cast<uint4 *>(y + row * y_stride);
    // columns cols .. y_stride - 1 of the output row: zeros (the K padding of the next GEMM's input)
    for (int c = nv + tid; c < y_stride / 8; c += kLnThreads) yr[c] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int c = tid + i * kLnThreads;
        if (c >= nv) continue;
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int k = 8 * c + 2 * e;
            const __half2 hv = __floats2half2_rn((f[i][2 * e] - mean) * inv * w[k] + bias[k],
                                                 (f[i][2 * e + 1] - mean) * inv * w[k + 1] + bias[k + 1]);
            h[e] = *reinterpret_cast<const uint32_t *>(&hv);
        }
        yr[c] = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// -------------------------------------------------------------- elementwise
__global__ void gelu_kernel(const __half *__restrict__ x, __half *__restrict__ y, int64_t n) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        y[i] = __float2half_rn(gelu_erf(__half2float(x[i])));
}

// out[o, :] = x[index[o], :]; an index outside [0, rows) writes zeros and sets T2C_EINVAL.
__global__ void index_rows_kernel(const __half *__restrict__ x, const int64_t *__restrict__ index,
                                  __half *__restrict__ out, int64_t O, int64_t H, int64_t rows) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < O * H;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t o = i / H, c = i - o * H;
        const int64_t r = index[o];
        if (r < 0 || r >= rows) {
            if (c == 0) report_device_error(T2C_EINVAL);
            out[i] = __float2half(0.0f);
        } else {
            out[i] = x[r * H + c];
        }
    }
}

// cache[b, index[s], :] = src[b, s, :] (fp16 rows of H; the audio-feature injection into the
// text embeddings).  A destination row outside [0, T) is skipped and sets T2C_EINVAL.
__global__ void index_copy_rows_kernel(__half *__restrict__ cache, const int64_t *__restrict__ index,
                                       const __half *__restrict__ src, int64_t B, int64_t T, int64_t S, int64_t H) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < B * S * H;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t h = i % H, bs = i / H;
        const int64_t s = bs % S, b = bs / S;
        const int64_t t = index[s];
        if (t < 0 || t >= T) {
            if (h == 0) report_device_error(T2C_EINVAL);
            continue;
        }
        cache[(b * T + t) * H + h] = src[i];
    }
}

// out[i, :] = fp16(d * q) of Q8_0 rows ids[i] (embedding_q8_0_f32.py: d fp16, 32 int8 per block)
__global__ void embedding_q8_0_kernel(const uint8_t *__restrict__ w, const int64_t *__restrict__ ids,
                                      __half *__restrict__ out, int64_t n_ids, int64_t vocab, int64_t H) {
    pdl_wait();
    pdl_trigger();
    const int64_t row_bytes = H / 32 * 34;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_ids * H;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / H, c = i - r * H;
        int64_t id = ids[r];
        if (id < 0 || id >= vocab) {
            if (c == 0) report_device_error(T2C_EINVAL);
            id = 0;
        }
        const uint8_t *blk = w + id * row_bytes + (c >> 5) * 34;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
        out[i] = __float2half_rn(d * static_cast<float>(static_cast<int8_t>(blk[2 + (c & 31)])));
    }
}

// OmniVoice input embedding (omnivoice_input_embed_q8_0_f32, quantized_omnivoice/custom_shaders.py:17-181):
// out[b, s, :] = fp16(sum over codebooks c of audio row c * V + ids[b, c, s]) where audio_mask[b, s]
// is set (fp32 sum in codebook order), else fp16(text row ids[b, 0, s]).  Each value d * q of a
// Q8_0 block is exact in fp32.  An id outside its table reads row 0 and reports T2C_EINVAL.
__global__ void omnivoice_input_embed_kernel(const uint8_t *__restrict__ tw, const uint8_t *__restrict__ aw,
                                             const int64_t *__restrict__ ids, const uint32_t *__restrict__ amask,
                                             __half *__restrict__ out, int B, int C, int S, int H, int64_t TV,
                                             int64_t V) {
    pdl_wait();
    pdl_trigger();
    const int64_t row_bytes = H / 32 * 34;
    auto q8 = [&](const uint8_t *w, int64_t row, int h) {
        const uint8_t *blk = w + row * row_bytes + (h >> 5) * 34;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
        return d * static_cast<float>(static_cast<int8_t>(blk[2 + (h & 31)]));
    };
    const int64_t total = static_cast<int64_t>(B) * S * H;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int h = static_cast<int>(i % H);
        const int64_t bs = i / H;
        const int s = static_cast<int>(bs % S), b = static_cast<int>(bs / S);
        if (amask[bs] != 0u) {
            float value = 0.0f;
            for (int c = 0; c < C; ++c) {
                int64_t tok = ids[(static_cast<int64_t>(b) * C + c) * S + s];
                if (tok < 0 || tok >= V) {
                    if (h == 0) report_device_error(T2C_EINVAL);
                    tok = 0;
                }
                value += q8(aw, c * V + tok, h);
            }
            out[i] = __float2half_rn(value);
        } else {
            int64_t tok = ids[static_cast<int64_t>(b) * C * S + s];
            if (tok < 0 || tok >= TV) {
                if (h == 0) report_device_error(T2C_EINVAL);
                tok = 0;
            }
            out[i] = __float2half_rn(q8(tw, tok, h));
        }
    }
}

// ---------------------------------------------------- masked attention
// out[b, h, t, :] = softmax(q k^T * scale + mask[t, s]) v over all S keys
// (non-causal; the additive fp16 mask carries the encoder's block-diagonal
// windows, -inf outside).  CTA = 4 warps on (b, h, 64-query tile); key / value
// tiles of 64 rows in shared memory; mma.m16n8k16 for S = Q K^T and O += P V
// (P split into fp16 high / low parts), online softmax in the log2 domain.
// im2col of a 2-D convolution: cols[(b Ho + oh) Wo + ow][(c kh + i) kw + j] = x[b, c, oh sh - ph + i,
// ow sw - pw + j] (zero outside the image), columns K .. Kp - 1 zero.  x is read through element
// strides (NCHW, or the NHWC rows a GEMM wrote); one thread writes 8 consecutive columns (16 bytes).
__global__ void im2col_kernel(const __half *__restrict__ x, __half *__restrict__ cols, int64_t rows, int Ho, int Wo,
                              int H, int W, int kh, int kw, int sh, int sw, int ph, int pw, int K, int Kp, int64_t xsb,
                              int64_t xsc, int64_t xsh, int64_t xsw) {
    const int groups = Kp / 8;
    const int64_t total = rows * groups;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = e / groups;
        const int k0 = static_cast<int>(e - r * groups) * 8;
        const int ow = static_cast<int>(r % Wo);
        const int64_t t = r / Wo;
        const int oh = static_cast<int>(t % Ho);
        const int64_t b = t / Ho;
        int j = k0 % kw, i = (k0 / kw) % kh, c = k0 / (kw * kh);
        __align__(16) __half v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            __half val = __float2half(0.0f);
            if (k0 + u < K) {
                const int ih = oh * sh - ph + i, iw = ow * sw - pw + j;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W) val = x[b * xsb + c * xsc + ih * xsh + iw * xsw];
            }
            v[u] = val;
            if (++j == kw) {
                j = 0;
                if (++i == kh) {
                    i = 0;
                    ++c;
                }
            }
        }
        *reinterpret_cast<uint4 *>(cols + r * Kp + k0) = *reinterpret_cast<const uint4 *>(v);
    }
}

// The same columns from channels-last x (rows [B, H, W, C], c contiguous, C % 8 == 0) for a 3 x 3
// kernel: one thread per (output pixel, 8 channels) reads the 9 taps as 16-byte vectors and writes
// the 72 columns (c, i, j) of those channels as 9 16-byte stores; one more thread per 8 padding
// columns of a row writes zeros.
__global__ void im2col_cl3_kernel(const __half *__restrict__ x, __half *__restrict__ cols, int64_t rows, int Ho,
                                  int Wo, int H, int W, int C, int sh, int sw, int ph, int pw, int K, int Kp,
                                  int64_t xsb, int64_t xsh, int64_t xsw) {
    const int cg = C / 8, padg = (Kp - K) / 8, per_row = cg + padg;
    const int64_t total = rows * per_row;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < total;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = e / per_row;
        const int q = static_cast<int>(e - r * per_row);
        __half *dst = cols + r * Kp;
        if (q >= cg) {
            *reinterpret_cast<uint4 *>(dst + K + 8 * (q - cg)) = make_uint4(0, 0, 0, 0);
            continue;
        }
        const int ow = static_cast<int>(r % Wo);
        const int64_t t = r / Wo;
        const int oh = static_cast<int>(t % Ho);
        const int64_t b = t / Ho;
        __align__(16) __half tap[9][8];
#pragma unroll
        for (int i = 0; i < 3; ++i)
#pragma unroll
            for (int j = 0; j < 3; ++j) {
                const int ih = oh * sh - ph + i, iw = ow * sw - pw + j;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                    v = *reinterpret_cast<const uint4 *>(x + b * xsb + ih * xsh + iw * xsw + 8 * q);
                *reinterpret_cast<uint4 *>(tap[3 * i + j]) = v;
            }
        // columns 72 q .. 72 q + 71: channel 8 q + u, tap m at 9 u + m
        __align__(16) __half out[72];
#pragma unroll
        for (int u = 0; u < 8; ++u)
#pragma unroll
            for (int m = 0; m < 9; ++m) out[9 * u + m] = tap[m][u];
#pragma unroll
        for (int w16 = 0; w16 < 9; ++w16)
            *reinterpret_cast<uint4 *>(dst + 72 * static_cast<int64_t>(q) + 8 * w16) =
                *reinterpret_cast<const uint4 *>(out + 8 * w16);
    }
}

template <int D>
__global__ void __launch_bounds__(128) attn_masked_kernel(
    const __half *__restrict__ q, const __half *__restrict__ k, const __half *__restrict__ v,
    const __half *__restrict__ mask, __half *__restrict__ out, int H, int T, int S, int64_t q_sb, int64_t q_sh,
    int64_t q_st, int64_t k_sb, int64_t k_sh, int64_t k_ss, int64_t v_sb, int64_t v_sh, int64_t v_ss, int64_t m_sb,
    int64_t m_sh, int64_t m_st, int64_t o_sb, int64_t o_sh, int64_t o_st, float scale_log2) {
    constexpr int R = D + 8;  // halves per shared row
    constexpr int KS = D / 16, NT = D / 8;
    __shared__ __align__(16) __half qs[64][R];
    __shared__ __align__(16) __half ks[64][R];
    __shared__ __align__(16) __half vs[64][R];
    const int qtiles = (T + 63) / 64;
    const int qt = blockIdx.x % qtiles;
    const int h = (blockIdx.x / qtiles) % H;
    const int b = blockIdx.x / (qtiles * H);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t4 = lane & 3;
    pdl_wait();
    pdl_trigger();
    const int q0 = qt * 64;
    for (int i = threadIdx.x; i < 64 * (D / 8); i += 128) {
        const int r = i / (D / 8), c = i - r * (D / 8);
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (q0 + r < T) val = *reinterpret_cast<const uint4 *>(q + b * q_sb + h * q_sh + (q0 + r) * q_st + 8 * c);
        *reinterpret_cast<uint4 *>(&qs[r][8 * c]) = val;
    }
    __syncthreads();
    uint32_t qa[KS][4];
#pragma unroll
    for (int s = 0; s < KS; ++s) ldsm4(qa[s], &qs[16 * w + (lane & 15)][16 * s + 8 * (lane >> 4)]);
    const int t0 = q0 + 16 * w + g, t1 = t0 + 8;
    const __half *mrow0 = mask + b * m_sb + h * m_sh + static_cast<int64_t>(min(t0, T - 1)) * m_st;
    const __half *mrow1 = mask + b * m_sb + h * m_sh + static_cast<int64_t>(min(t1, T - 1)) * m_st;
    float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.0f, 0.0f};
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    for (int s0 = 0; s0 < S; s0 += 64) {
        __syncthreads();
        for (int i = threadIdx.x; i < 64 * (D / 8); i += 128) {
            const int r = i / (D / 8), c = i - r * (D / 8);
            uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
            if (s0 + r < S) {
                kv = *reinterpret_cast<const uint4 *>(k + b * k_sb + h * k_sh + (s0 + r) * k_ss + 8 * c);
                vv = *reinterpret_cast<const uint4 *>(v + b * v_sb + h * v_sh + (s0 + r) * v_ss + 8 * c);
            }
            *reinterpret_cast<uint4 *>(&ks[r][8 * c]) = kv;
            *reinterpret_cast<uint4 *>(&vs[r][8 * c]) = vv;
        }
        __syncthreads();
        float sc[8][4];
#pragma unroll
        for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
        for (int s = 0; s < KS; ++s)
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t kb[4];
                ldsm4(kb, &ks[16 * np + (lane & 7) + 8 * (lane >> 4)][16 * s + 8 * ((lane >> 3) & 1)]);
                mma16816(sc[2 * np], qa[s], kb[0], kb[1]);
                mma16816(sc[2 * np + 1], qa[s], kb[2], kb[3]);
            }
        float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = s0 + 8 * n + 2 * t4 + (e & 1);
                const int r = e >> 1;
                float val = -INFINITY;
                if (key < S) {
                    const float mk = __half2float((r ? mrow1 : mrow0)[key]);
                    val = (sc[n][e] * scale_log2) + mk * 1.4426950408889634f;
                }
                sc[n][e] = val;
                mx[r] = fmaxf(mx[r], val);
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
        for (int n = 0; n < NT; ++n) {
            o[n][0] *= corr[0];
            o[n][1] *= corr[0];
            o[n][2] *= corr[1];
            o[n][3] *= corr[1];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float pv[2][4];
#pragma unroll
            for (int hn = 0; hn < 2; ++hn)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p = exp2f(sc[2 * j + hn][e] - m_run[e >> 1]);
                    l_run[e >> 1] += p;
                    pv[hn][e] = p;
                }
            uint32_t ah[4], al[4];
#pragma unroll
            for (int hn = 0; hn < 2; ++hn)
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const __half2 hi = __floats2half2_rn(pv[hn][2 * r], pv[hn][2 * r + 1]);
                    const float2 hf = __half22float2(hi);
                    const __half2 lo = __floats2half2_rn(pv[hn][2 * r] - hf.x, pv[hn][2 * r + 1] - hf.y);
                    ah[2 * hn + r] = *reinterpret_cast<const uint32_t *>(&hi);
                    al[2 * hn + r] = *reinterpret_cast<const uint32_t *>(&lo);
                }
#pragma unroll
            for (int dp = 0; dp < D / 16; ++dp) {
                uint32_t vb[4];
                ldsm4_t(vb, &vs[16 * j + (lane & 7) + 8 * ((lane >> 3) & 1)][16 * dp + 8 * (lane >> 4)]);
                mma16816(o[2 * dp], ah, vb[0], vb[1]);
                mma16816(o[2 * dp], al, vb[0], vb[1]);
                mma16816(o[2 * dp + 1], ah, vb[2], vb[3]);
                mma16816(o[2 * dp + 1], al, vb[2], vb[3]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f, inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        const int d = 8 * n + 2 * t4;
        if (t0 < T)
            *reinterpret_cast<__half2 *>(out + b * o_sb + h * o_sh + static_cast<int64_t>(t0) * o_st + d) =
                __floats2half2_rn(o[n][0] * inv0, o[n][1] * inv0);
        if (t1 < T)
            *reinterpret_cast<__half2 *>(out + b * o_sb + h * o_sh + static_cast<int64_t>(t1) * o_st + d) =
                __floats2half2_rn(o[n][2] * inv1, o[n][3] * inv1);
    }
}

template <typename Kernel, typename... Args>
int launch_asr(Kernel kernel, dim3 grid, dim3 block, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, args...);
    if (err != cudaSuccess) return set_error(T2C_ECUDA, "asr launch: %s", cudaGetErrorString(err));
    return T2C_OK;
}

bool al(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int q8_gemm(Q8Gemm p, bool conv, cudaStream_t s) {
    const dim3 grid(static_cast<unsigned>((p.M + kQT - 1) / kQT), static_cast<unsigned>((p.N + kQT - 1) / kQT));
    return conv ? launch_asr(q8_gemm_kernel<true>, grid, dim3(128), s, p) : launch_asr(q8_gemm_kernel<false>, grid, dim3(128), s, p);
}

}  // namespace

cudaError_t status_asr(unsigned int *bits, int clear, cudaStream_t s) { return read_tu_status(bits, clear, s); }

}  // namespace t2c

using namespace t2c;

extern "C" int t2c_linear_q8_0_bias(const void *x, const void *w, const float *bias, void *y, int64_t M, int64_t N,
                                    int64_t K, int act, void *stream) {
    if (!x || !w || !y) return set_error(T2C_EINVAL, "linear_q8_0_bias: NULL pointer");
    if (M <= 0 || N <= 0 || K <= 0 || M > INT32_MAX || N > INT32_MAX || K > INT32_MAX)
        return set_error(T2C_EINVAL, "linear_q8_0_bias: bad shape");
    if (K % 8 || !al(x, 16) || !al(w, 2)) return set_error(T2C_EINVAL, "linear_q8_0_bias: x rows must be 16-byte aligned (K %% 8 == 0)");
    Q8Gemm p = {};
    p.x = static_cast<const __half *>(x);
    p.w = static_cast<const uint8_t *>(w);
    p.bias = bias;
    p.y = static_cast<__half *>(y);
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.nblk = static_cast<int>((K + 31) / 32);
    p.row_bytes = static_cast<int64_t>(p.nblk) * 34;
    p.act = act;
    if (M > 4 && K % 256 == 0 && al(w, 16)) {
        // whole 256-value groups: the tcgen05 GEMM with the bias / GELU epilogue
        QGemmArgs a = {};
        a.fmt = T2C_Q8_0;
        a.nw = 1;
        a.w[0] = p.w;
        a.N[0] = N;
        a.K = K;
        a.M = M;
        a.x = p.x;
        a.y[0] = p.y;
        a.bias = bias;
        a.act = act;
        const int rc = qgemm(a, as_stream(stream));
        if (rc != T2C_EUNSUPPORTED) return rc;
    }
    return q8_gemm(p, false, as_stream(stream));
}

static int conv2d_q8_0_impl(const void *x, const void *w, const float *bias, void *out, int64_t B, int64_t Ci,
                            int64_t Hi, int64_t Wi, int64_t Co, int64_t Ho, int64_t Wo, int64_t kh, int64_t kw,
                            int64_t sh, int64_t sw, int64_t ph, int64_t pw, int act, int out_cl, void *stream) {
    if (!x || !w || !out) return set_error(T2C_EINVAL, "conv2d_q8_0: NULL pointer");
    if (B <= 0 || Ci <= 0 || Hi <= 0 || Wi <= 0 || Co <= 0 || Ho <= 0 || Wo <= 0 || kh <= 0 || kw <= 0 || sh <= 0 ||
        sw <= 0 || ph < 0 || pw < 0)
        return set_error(T2C_EINVAL, "conv2d_q8_0: bad shape");
    if (B * Ci * Hi * Wi > INT32_MAX || B * Ho * Wo > INT32_MAX || Ci * kh * kw > INT32_MAX)
        return set_error(T2C_EUNSUPPORTED, "conv2d_q8_0: sizes beyond 2^31 elements");
    if ((Ho - 1) * sh - ph + kh - 1 >= Hi + ph || (Wo - 1) * sw - pw + kw - 1 >= Wi + pw)
        return set_error(T2C_EINVAL, "conv2d_q8_0: output extent does not match input, stride and padding");
    if (!al(w, 2)) return set_error(T2C_EINVAL, "conv2d_q8_0: weight must be 2-byte aligned");
    Q8Gemm p = {};
    p.x = static_cast<const __half *>(x);
    p.w = static_cast<const uint8_t *>(w);
    p.bias = bias;
    p.y = static_cast<__half *>(out);
    p.M = static_cast<int>(B * Ho * Wo);
    p.N = static_cast<int>(Co);
    p.K = static_cast<int>(Ci * kh * kw);
    p.nblk = (p.K + 31) / 32;
    p.row_bytes = static_cast<int64_t>(p.nblk) * 34;
    p.act = act;
    p.out_cl = out_cl;
    p.Ci = static_cast<int>(Ci);
    p.Hi = static_cast<int>(Hi);
    p.Wi = static_cast<int>(Wi);
    p.Ho = static_cast<int>(Ho);
    p.Wo = static_cast<int>(Wo);
    p.kh = static_cast<int>(kh);
    p.kw = static_cast<int>(kw);
    p.sh = static_cast<int>(sh);
    p.sw = static_cast<int>(sw);
    p.ph = static_cast<int>(ph);
    p.pw = static_cast<int>(pw);
    return q8_gemm(p, true, as_stream(stream));
}

extern "C" int t2c_layer_norm(const void *x, const float *w, const float *b, void *y, int64_t rows, int64_t cols,
                              float eps, void *stream) {
    if (!x || !w || !b || !y) return set_error(T2C_EINVAL, "layer_norm: NULL pointer");
    if (rows <= 0 || cols <= 0 || cols % 8 || cols > 8 * 2 * kLnThreads)
        return set_error(T2C_EINVAL, "layer_norm: cols must be a multiple of 8 up to %d", 16 * kLnThreads);
    if (!al(x, 16) || !al(y, 16)) return set_error(T2C_EINVAL, "layer_norm: rows must be 16-byte aligned");
    return launch_asr(layer_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kLnThreads), as_stream(stream),
                      static_cast<const __half *>(x), w, b, static_cast<__half *>(y), static_cast<int>(cols), eps,
                      static_cast<int>(cols));
}

extern "C" int t2c_layer_norm_padded(const void *x, const float *w, const float *b, void *y, int64_t rows,
                                     int64_t cols, int64_t y_cols, float eps, void *stream) {
    if (!x || !w || !b || !y) return set_error(T2C_EINVAL, "layer_norm_padded: NULL pointer");
    if (rows <= 0 || cols <= 0 || cols % 8 || cols > 8 * 2 * kLnThreads || y_cols < cols || y_cols % 8 ||
        y_cols > INT32_MAX)
        return set_error(T2C_EINVAL, "layer_norm_padded: cols must be a multiple of 8 up to %d, y_cols >= cols a "
                                     "multiple of 8", 16 * kLnThreads);
    if (!al(x, 16) || !al(y, 16)) return set_error(T2C_EINVAL, "layer_norm_padded: rows must be 16-byte aligned");
    return launch_asr(layer_norm_kernel, dim3(static_cast<unsigned>(rows)), dim3(kLnThreads), as_stream(stream),
                      static_cast<const __half *>(x), w, b, static_cast<__half *>(y), static_cast<int>(cols), eps,
                      static_cast<int>(y_cols));
}

extern "C" int t2c_gelu(const void *x, void *y, int64_t n, void *stream) {
    if (!x || !y || n <= 0) return set_error(T2C_EINVAL, "gelu: bad argument");
    int64_t grid = (n + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    return launch_asr(gelu_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), as_stream(stream),
                      static_cast<const __half *>(x), static_cast<__half *>(y), n);
}

extern "C" int t2c_index_rows(const void *x, const int64_t *index, void *out, int64_t O, int64_t H, int64_t rows,
                              void *stream) {
    if (!x || !index || !out || O <= 0 || H <= 0 || rows <= 0) return set_error(T2C_EINVAL, "index_rows: bad argument");
    int64_t grid = (O * H + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    return launch_asr(index_rows_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), as_stream(stream),
                      static_cast<const __half *>(x), index, static_cast<__half *>(out), O, H, rows);
}

extern "C" int t2c_index_copy_rows(void *cache, const int64_t *index, const void *src, int64_t B, int64_t T, int64_t S,
                                   int64_t H, void *stream) {
    if (!cache || !index || !src || B <= 0 || T <= 0 || S <= 0 || H <= 0)
        return set_error(T2C_EINVAL, "index_copy_rows: bad arguments");
    int64_t grid = (B * S * H + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    return launch_asr(index_copy_rows_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), as_stream(stream),
                      static_cast<__half *>(cache), index, static_cast<const __half *>(src), B, T, S, H);
}

extern "C" int t2c_embedding_q8_0(const void *weight, const int64_t *ids, void *out, int64_t n_ids, int64_t vocab,
                                  int64_t H, void *stream) {
    if (!weight || !ids || !out || n_ids <= 0 || vocab <= 0 || H <= 0 || H % 32)
        return set_error(T2C_EINVAL, "embedding_q8_0: bad arguments (H a multiple of 32)");
    int64_t grid = (n_ids * H + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    return launch_asr(embedding_q8_0_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), as_stream(stream),
                      static_cast<const uint8_t *>(weight), ids, static_cast<__half *>(out), n_ids, vocab, H);
}

extern "C" int t2c_omnivoice_input_embed(const void *text_weight, const void *audio_weight, const int64_t *ids,
                                         const uint32_t *audio_mask, void *out, int64_t B, int64_t C, int64_t S,
                                         int64_t H, int64_t text_vocab, int64_t audio_vocab, void *stream) {
    if (!text_weight || !audio_weight || !ids || !audio_mask || !out)
        return set_error(T2C_EINVAL, "omnivoice_input_embed: NULL pointer");
    if (B <= 0 || C <= 0 || S <= 0 || H <= 0 || H % 32 || text_vocab <= 0 || audio_vocab <= 0 || B * S > INT32_MAX ||
        C > 64)
        return set_error(T2C_EINVAL, "omnivoice_input_embed: bad shape (H a multiple of 32)");
    int64_t grid = (B * S * H + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    return launch_asr(omnivoice_input_embed_kernel, dim3(static_cast<unsigned>(grid)), dim3(256), as_stream(stream),
                      static_cast<const uint8_t *>(text_weight), static_cast<const uint8_t *>(audio_weight), ids,
                      audio_mask, static_cast<__half *>(out), static_cast<int>(B), static_cast<int>(C),
                      static_cast<int>(S), static_cast<int>(H), text_vocab, audio_vocab);
}

extern "C" int t2c_attn_masked(const void *q, const void *k, const void *v, const void *mask, void *out, int64_t B,
                               int64_t H, int64_t T, int64_t S, int64_t D, const int64_t *q_strides,
                               const int64_t *k_strides, const int64_t *v_strides, const int64_t *m_strides,
                               const int64_t *o_strides, float scale, void *stream) {
    if (!q || !k || !v || !mask || !out || !q_strides || !k_strides || !v_strides || !m_strides || !o_strides)
        return set_error(T2C_EINVAL, "attn_masked: NULL pointer");
    if (B <= 0 || H <= 0 || T <= 0 || S <= 0) return set_error(T2C_EINVAL, "attn_masked: bad shape");
    if (D != 64) return set_error(T2C_EUNSUPPORTED, "attn_masked: D=%lld (64 only)", (long long)D);
    const int64_t *st[3] = {q_strides, k_strides, v_strides};
    const void *ptrs[3] = {q, k, v};
    for (int i = 0; i < 3; ++i) {
        if (!al(ptrs[i], 16) || st[i][0] % 8 || st[i][1] % 8 || st[i][2] % 8)
            return set_error(T2C_EINVAL, "attn_masked: q / k / v rows must be 16-byte aligned");
    }
    if (!al(out, 4) || o_strides[0] % 2 || o_strides[1] % 2 || o_strides[2] % 2)
        return set_error(T2C_EINVAL, "attn_masked: out rows must be 4-byte aligned");
    const int64_t qtiles = (T + 63) / 64;
    const dim3 grid(static_cast<unsigned>(B * H * qtiles));
    const float sl2 = 1.4426950408889634f * scale;
#define T2C_AM(DD)                                                                                                    \
    return launch_asr(attn_masked_kernel<DD>, grid, dim3(128), as_stream(stream), static_cast<const __half *>(q),      \
                      static_cast<const __half *>(k), static_cast<const __half *>(v), static_cast<const __half *>(mask), \
                      static_cast<__half *>(out), static_cast<int>(H), static_cast<int>(T), static_cast<int>(S),        \
                      q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1], k_strides[2], v_strides[0],  \
                      v_strides[1], v_strides[2], m_strides[0], m_strides[1], m_strides[2], o_strides[0], o_strides[1], \
                      o_strides[2], sl2)
    T2C_AM(64);
#undef T2C_AM
}

extern "C" int t2c_im2col_f16(const void *x, void *cols, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ho,
                              int64_t Wo, int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                              int64_t Kp, const int64_t *x_strides, int channels_last, void *stream) {
    if (!x || !cols || !x_strides) return set_error(T2C_EINVAL, "im2col: NULL pointer");
    const int64_t K = C * kh * kw;
    if (B <= 0 || C <= 0 || H <= 0 || W <= 0 || Ho <= 0 || Wo <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
        ph < 0 || pw < 0 || Kp < K || Kp % 8)
        return set_error(T2C_EINVAL, "im2col: bad shape (Kp must be >= C*kh*kw and a multiple of 8)");
    if (K > INT32_MAX || Kp > INT32_MAX || H > INT32_MAX || W > INT32_MAX || Ho > INT32_MAX || Wo > INT32_MAX)
        return set_error(T2C_EUNSUPPORTED, "im2col: sizes beyond 2^31");
    if ((Ho - 1) * sh - ph + kh - 1 >= H + ph || (Wo - 1) * sw - pw + kw - 1 >= W + pw)
        return set_error(T2C_EINVAL, "im2col: output extent does not match input, stride and padding");
    if (!al(cols, 16)) return set_error(T2C_EINVAL, "im2col: cols must be 16-byte aligned");
    const int64_t rows = B * Ho * Wo;
    const int64_t total = rows * (Kp / 8);
    int64_t blocks = (total + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    if (channels_last && kh == 3 && kw == 3 && x_strides[1] == 1 && C % 8 == 0 && al(x, 16) && x_strides[0] % 8 == 0 &&
        x_strides[2] % 8 == 0 && x_strides[3] % 8 == 0) {
        const int64_t total3 = rows * (C / 8 + (Kp - K) / 8);
        int64_t blocks3 = (total3 + 255) / 256;
        if (blocks3 > 148 * 32) blocks3 = 148 * 32;
        im2col_cl3_kernel<<<static_cast<unsigned>(blocks3), 256, 0, as_stream(stream)>>>(
            static_cast<const __half *>(x), static_cast<__half *>(cols), rows, static_cast<int>(Ho),
            static_cast<int>(Wo), static_cast<int>(H), static_cast<int>(W), static_cast<int>(C), static_cast<int>(sh),
            static_cast<int>(sw), static_cast<int>(ph), static_cast<int>(pw), static_cast<int>(K),
            static_cast<int>(Kp), x_strides[0], x_strides[2], x_strides[3]);
        return check_launch("im2col");
    }
    im2col_kernel<<<static_cast<unsigned>(blocks), 256, 0, as_stream(stream)>>>(
        static_cast<const __half *>(x), static_cast<__half *>(cols), rows, static_cast<int>(Ho), static_cast<int>(Wo),
        static_cast<int>(H), static_cast<int>(W), static_cast<int>(kh), static_cast<int>(kw), static_cast<int>(sh),
        static_cast<int>(sw), static_cast<int>(ph), static_cast<int>(pw), static_cast<int>(K), static_cast<int>(Kp),
        x_strides[0], x_strides[1], x_strides[2], x_strides[3]);
    return check_launch("im2col");
}

extern "C" int t2c_conv2d_q8_0(const void *x, const void *w, const float *bias, void *out, int64_t B, int64_t Ci,
                               int64_t Hi, int64_t Wi, int64_t Co, int64_t Ho, int64_t Wo, int64_t kh, int64_t kw,
                               int64_t sh, int64_t sw, int64_t ph, int64_t pw, int act, void *stream) {
    return conv2d_q8_0_impl(x, w, bias, out, B, Ci, Hi, Wi, Co, Ho, Wo, kh, kw, sh, sw, ph, pw, act, 0, stream);
}

extern "C" int t2c_conv2d_q8_0_nhwc(const void *x, const void *w, const float *bias, void *out, int64_t B,
                                    int64_t Ci, int64_t Hi, int64_t Wi, int64_t Co, int64_t Ho, int64_t Wo,
                                    int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int act,
                                    void *stream) {
    return conv2d_q8_0_impl(x, w, bias, out, B, Ci, Hi, Wi, Co, Ho, Wo, kh, kw, sh, sw, ph, pw, act, 1, stream);
}

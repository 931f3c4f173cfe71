// GGUF block quantizers (fp32 -> Q8_0 / Q4_K / Q6_K) and block decoders on the
// GPU.  The arithmetic is the reference quantizer's
// (src/torch2vk/quantize/vulkan.py:91-185 Q8_0, :188-419 Q4_K, :422-637 Q6_K):
// IEEE binary32 operations in the shader's order.  This file is compiled with
// --fmad=false so no multiply-add is contracted, which makes the packed bytes
// reproducible bit for bit on any IEEE CPU.  The implementation-defined GLSL
// round() of the Q6_K path is taken as round-half-away-from-zero (roundf).
//
// Work split (one warp = 4 Q4_K super-blocks or 2 Q6_K blocks or 1 Q8_0 block):
//  Q4_K: lane = (super-block, sub-block of 32); each lane runs the weighted
//        least-squares scale/min search of its sub-block, the 8 lanes of a
//        super-block agree on (d, dmin) with shuffles, and pack via shared memory.
//  Q6_K: lane = (block, group of 16); same pattern with the 19-step search.
//  Q8_0: lane = value.
#include "common.cuh"

namespace t2c {
namespace {

constexpr int kQThreads = 128;

__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }
__device__ __forceinline__ uint32_t f16_bits(float v) { return __half_as_ushort(__float2half_rn(v)); }

__device__ __forceinline__ uint32_t code_floor_half(float value, uint32_t max_code) {
    return static_cast<uint32_t>(fminf(fmaxf(floorf(value + 0.5f), 0.0f), static_cast<float>(max_code)));
}

// -------------------------------------------------------------------- Q8_0
__global__ void quantize_q8_0_kernel(const float *__restrict__ x, uint8_t *__restrict__ out, int64_t blocks,
                                     int64_t nb_row, int64_t K) {
    const int lane = threadIdx.x & 31;
    const int64_t blk = (static_cast<int64_t>(blockIdx.x) * kQThreads + threadIdx.x) >> 5;
    if (blk >= blocks) return;
    const int64_t row = blk / nb_row, b = blk - row * nb_row;
    const float v = x[row * K + b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const float scale = amax / 127.0f;
    const float inv = scale == 0.0f ? 0.0f : 1.0f / scale;
    const float t = v * inv;
    const float a = fabsf(t);
    const float fl = floorf(a);
    const float rounded = fl + floorf(2.0f * (a - fl));
    const float sg = t > 0.0f ? 1.0f : (t < 0.0f ? -1.0f : 0.0f);
    int q = static_cast<int>(sg * rounded);
    q = max(-128, min(127, q));
    uint8_t *o = out + blk * 34;
    if (lane == 0) st_u16(o, f16_bits(scale));
    o[2 + lane] = static_cast<uint8_t>(q & 255);
}

// -------------------------------------------------------------------- Q4_K
__device__ float q4k_error(const float *v, float scale, float minimum, float inv_scale, float av_x) {
    float error = 0.0f;
    for (int i = 0; i < 32; ++i) {
        const float weight = av_x + fabsf(v[i]);
        const float level = static_cast<float>(code_floor_half(inv_scale * (v[i] - minimum), 15u));
        const float diff = scale * level + minimum - v[i];
        error += weight * diff * diff;
    }
    return error;
}

__device__ float q4k_search(const float *v, float *min_offset) {
    float lo = v[0], hi = v[0], sum_x2 = 0.0f;
    for (int i = 0; i < 32; ++i) {
        lo = fminf(lo, v[i]);
        hi = fmaxf(hi, v[i]);
        sum_x2 += v[i] * v[i];
    }
    if (lo > 0.0f) lo = 0.0f;
    if (hi == lo) {
        *min_offset = -lo;
        return 0.0f;
    }
    const float av_x = sqrtf(sum_x2 / 32.0f);
    float sum_w = 0.0f, sum_x = 0.0f;
    for (int i = 0; i < 32; ++i) {
        const float weight = av_x + fabsf(v[i]);
        sum_w += weight;
        sum_x += weight * v[i];
    }
    float inv_scale = 15.0f / (hi - lo);
    float best_scale = 1.0f / inv_scale;
    float best_min = lo;
    float best_error = q4k_error(v, best_scale, best_min, inv_scale, av_x);
    for (int step = 0; step <= 20; ++step) {
        inv_scale = (14.0f + 0.1f * static_cast<float>(step)) / (hi - lo);
        float sum_l = 0.0f, sum_l2 = 0.0f, sum_xl = 0.0f;
        for (int i = 0; i < 32; ++i) {
            const float weight = av_x + fabsf(v[i]);
            const float level = static_cast<float>(code_floor_half(inv_scale * (v[i] - lo), 15u));
            sum_l += weight * level;
            sum_l2 += weight * level * level;
            sum_xl += weight * level * v[i];
        }
        const float det = sum_w * sum_l2 - sum_l * sum_l;
        if (det > 0.0f) {
            float cs = (sum_w * sum_xl - sum_x * sum_l) / det;
            float cm = (sum_l2 * sum_x - sum_l * sum_xl) / det;
            if (cm > 0.0f) {
                cm = 0.0f;
                cs = sum_l2 > 0.0f ? sum_xl / sum_l2 : 0.0f;
            }
            const float err = q4k_error(v, cs, cm, inv_scale, av_x);
            if (err < best_error) {
                best_error = err;
                best_scale = cs;
                best_min = cm;
            }
        }
    }
    *min_offset = fmaxf(0.0f, -best_min);
    return fmaxf(0.0f, best_scale);
}

__global__ void __launch_bounds__(kQThreads) quantize_q4_k_kernel(const float *__restrict__ x, uint8_t *__restrict__ out,
                                                                  int64_t blocks, int64_t nb_row, int64_t K) {
    __shared__ uint8_t quants[kQThreads / 8][256];
    __shared__ uint8_t codes[kQThreads / 8][16];
    const int lane = threadIdx.x & 31;
    const int slot = threadIdx.x >> 3;  // super-block slot in this CTA
    const int j = threadIdx.x & 7;      // sub-block
    const int64_t blk = static_cast<int64_t>(blockIdx.x) * (kQThreads / 8) + slot;
    const bool active = blk < blocks;
    float v[32];
    float sub_scale = 0.0f, sub_min = 0.0f;
    if (active) {
        const int64_t row = blk / nb_row, b = blk - row * nb_row;
        const float *src = x + row * K + b * 256 + j * 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = src[i];
        sub_scale = q4k_search(v, &sub_min);
    }
    // max over the 8 sub-blocks of this super-block (lanes slot*8 .. slot*8+7)
    float max_scale = sub_scale, max_min = sub_min;
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        max_scale = fmaxf(max_scale, __shfl_xor_sync(0xffffffffu, max_scale, o));
        max_min = fmaxf(max_min, __shfl_xor_sync(0xffffffffu, max_min, o));
    }
    (void)lane;
    float d_scale = max_scale > 0.0f ? max_scale / 63.0f : 0.0f;
    float d_min = max_min > 0.0f ? max_min / 63.0f : 0.0f;
    const float inv_scale = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
    const float inv_min = max_min > 0.0f ? 63.0f / max_min : 0.0f;
    const uint32_t sc = code_floor_half(sub_scale * inv_scale, 63u);
    const uint32_t mn = code_floor_half(sub_min * inv_min, 63u);
    d_scale = f16_round(d_scale);
    d_min = f16_round(d_min);
    codes[slot][j] = static_cast<uint8_t>(sc);
    codes[slot][8 + j] = static_cast<uint8_t>(mn);
    const float scale = d_scale * static_cast<float>(sc);
    const float minimum = d_min * static_cast<float>(mn);
    if (active) {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            uint32_t q = 0u;
            if (scale > 0.0f) q = code_floor_half((v[i] + minimum) / scale, 15u);
            quants[slot][j * 32 + i] = static_cast<uint8_t>(q);
        }
    }
    __syncwarp();
    if (active) {
        uint8_t *o = out + blk * 144;
        if (j == 0) st_u32(o, f16_bits(d_scale) | (f16_bits(d_min) << 16));
        for (int byte = 4 + j; byte < 144; byte += 8) {
            uint32_t value;
            if (byte < 8) {
                const int i = byte - 4;
                value = (codes[slot][i] & 63u) | ((codes[slot][i + 4] & 48u) << 2);
            } else if (byte < 12) {
                const int i = byte - 8;
                value = (codes[slot][8 + i] & 63u) | ((codes[slot][8 + i + 4] & 48u) << 2);
            } else if (byte < 16) {
                const int i = byte - 12;
                value = (codes[slot][i + 4] & 15u) | ((codes[slot][8 + i + 4] & 15u) << 4);
            } else {
                const int b = byte - 16;
                const int g = b >> 5, l = b & 31;
                value = (quants[slot][g * 64 + l] & 15u) | ((quants[slot][g * 64 + 32 + l] & 15u) << 4);
            }
            o[byte] = static_cast<uint8_t>(value);
        }
    }
}

// -------------------------------------------------------------------- Q6_K
__device__ __forceinline__ int near_int(float v) { return static_cast<int>(roundf(v)); }

__device__ float q6k_search(const float *v, int *levels) {
    float max_value = 0.0f, max_abs = 0.0f;
    for (int i = 0; i < 16; ++i) {
        const float a = fabsf(v[i]);
        if (a > max_abs) {
            max_abs = a;
            max_value = v[i];
        }
    }
    if (max_abs < 1.0e-12f) {
        for (int i = 0; i < 16; ++i) levels[i] = 32;
        return 0.0f;
    }
    float inv_scale = -32.0f / max_value;
    float sum_lx = 0.0f, sum_l2 = 0.0f;
    for (int i = 0; i < 16; ++i) {
        const int level = max(-32, min(31, near_int(inv_scale * v[i])));
        levels[i] = level + 32;
        const float weight = v[i] * v[i];
        sum_lx += weight * v[i] * static_cast<float>(level);
        sum_l2 += weight * static_cast<float>(level * level);
    }
    float scale = sum_l2 > 0.0f ? sum_lx / sum_l2 : 0.0f;
    float best = scale * sum_lx;
    for (int step = -9; step <= 9; ++step) {
        if (step == 0) continue;
        inv_scale = -(32.0f + 0.1f * static_cast<float>(step)) / max_value;
        sum_lx = 0.0f;
        sum_l2 = 0.0f;
        for (int i = 0; i < 16; ++i) {
            const int level = max(-32, min(31, near_int(inv_scale * v[i])));
            const float weight = v[i] * v[i];
            sum_lx += weight * v[i] * static_cast<float>(level);
            sum_l2 += weight * static_cast<float>(level * level);
        }
        if (sum_l2 > 0.0f && sum_lx * sum_lx > best * sum_l2) {
            for (int i = 0; i < 16; ++i) levels[i] = max(-32, min(31, near_int(inv_scale * v[i]))) + 32;
            scale = sum_lx / sum_l2;
            best = scale * sum_lx;
        }
    }
    return scale;
}

__global__ void __launch_bounds__(kQThreads) quantize_q6_k_kernel(const float *__restrict__ x, uint8_t *__restrict__ out,
                                                                  int64_t blocks, int64_t nb_row, int64_t K) {
    __shared__ uint8_t lv[kQThreads / 16][256];
    __shared__ int8_t sc_codes[kQThreads / 16][16];
    const int slot = threadIdx.x >> 4;
    const int g = threadIdx.x & 15;
    const int64_t blk = static_cast<int64_t>(blockIdx.x) * (kQThreads / 16) + slot;
    const bool active = blk < blocks;
    float v[16];
    int levels[16];
    float group_scale = 0.0f;
    if (active) {
        const int64_t row = blk / nb_row, b = blk - row * nb_row;
        const float *src = x + row * K + b * 256 + g * 16;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = src[i];
        group_scale = q6k_search(v, levels);
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            v[i] = 0.0f;
            levels[i] = 32;
        }
    }
    // first group (lowest index) with the largest |scale| (strict > scan order of the shader)
    float best_abs = fabsf(group_scale);
    int best_idx = g;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        const float other_abs = __shfl_xor_sync(0xffffffffu, best_abs, o);
        const int other_idx = __shfl_xor_sync(0xffffffffu, best_idx, o);
        if (other_abs > best_abs || (other_abs == best_abs && other_idx < best_idx)) {
            best_abs = other_abs;
            best_idx = other_idx;
        }
    }
    const int lane_base = threadIdx.x & 16;  // first lane of this 16-lane block within the warp
    const float max_scale = __shfl_sync(0xffffffffu, group_scale, (lane_base + best_idx) & 31);
    float d_scale;
    int code;
    if (best_abs < 1.0e-12f) {
        d_scale = 0.0f;
        code = 0;
    } else {
        const float inv_scale = -128.0f / max_scale;
        d_scale = f16_round(1.0f / inv_scale);
        code = max(-128, min(127, near_int(inv_scale * group_scale)));
    }
    const float d = d_scale * static_cast<float>(code);
    if (d != 0.0f) {
#pragma unroll
        for (int i = 0; i < 16; ++i) levels[i] = max(-32, min(31, near_int(v[i] / d))) + 32;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) lv[slot][g * 16 + i] = static_cast<uint8_t>(levels[i]);
    sc_codes[slot][g] = static_cast<int8_t>(code);
    __syncwarp();
    if (!active) return;
    uint8_t *o = out + blk * 210;
    if (g == 0) st_u16(o + 208, f16_bits(d_scale));
    for (int byte = g; byte < 208; byte += 16) {
        uint32_t value;
        if (byte < 128) {
            const int section = byte >> 6, local = byte & 31, base = section * 128;
            if ((byte & 32) == 0) {
                value = (lv[slot][base + local] & 15u) | ((lv[slot][base + local + 64] & 15u) << 4);
            } else {
                value = (lv[slot][base + local + 32] & 15u) | ((lv[slot][base + local + 96] & 15u) << 4);
            }
        } else if (byte < 192) {
            const int b = byte - 128;
            const int section = b >> 5, local = b & 31, base = section * 128;
            value = (((lv[slot][base + local] & 63u) >> 4) & 3u) | ((((lv[slot][base + local + 32] & 63u) >> 4) & 3u) << 2) |
                    ((((lv[slot][base + local + 64] & 63u) >> 4) & 3u) << 4) |
                    ((((lv[slot][base + local + 96] & 63u) >> 4) & 3u) << 6);
        } else {
            value = static_cast<uint32_t>(static_cast<uint8_t>(sc_codes[slot][byte - 192]));
        }
        o[byte] = static_cast<uint8_t>(value);
    }
}

// ----------------------------------------------------------------- decoders
__global__ void dequant_kernel(int wtype, const uint8_t *__restrict__ w, float *__restrict__ out, int64_t total,
                               int64_t K) {
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int64_t row = idx / K, k = idx - row * K;
    if (wtype == T2C_Q4_K) {
        const uint8_t *blk = w + row * (K / 256) * 144 + (k / 256) * 144;
        const int i = static_cast<int>(k & 255), j = i >> 5;
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
        const uint32_t q = (i & 32) ? (byte >> 4) : (byte & 15u);
        out[idx] = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                             __fmul_rn(dmin, static_cast<float>(m)));
    } else if (wtype == T2C_Q6_K) {
        const uint8_t *blk = w + row * (K / 256) * 210 + (k / 256) * 210;
        const int i = static_cast<int>(k & 255);
        const int s = i >> 7, c = (i >> 5) & 3, l = i & 31;
        const uint8_t qlb = blk[64 * s + 32 * (c & 1) + l];
        const uint32_t lo = (c >> 1) ? (qlb >> 4) : (qlb & 15u);
        const uint32_t hi = (static_cast<uint32_t>(blk[128 + 32 * s + l]) >> (2 * c)) & 3u;
        const int level = static_cast<int>(lo | (hi << 4)) - 32;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[208] | (blk[209] << 8))));
        const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + (i >> 4)]));
        out[idx] = __fmul_rn(__fmul_rn(d, sc), static_cast<float>(level));
    } else {
        const uint8_t *blk = w + row * (K / 32) * 34 + (k / 32) * 34;
        const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
        out[idx] = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(blk[2 + (k & 31)])));
    }
}

}  // namespace
}  // namespace t2c

using namespace t2c;

extern "C" int t2c_quantize(int wtype, const float *x, void *out, int64_t R, int64_t K, void *stream) {
    if (x == nullptr || out == nullptr) return set_error(T2C_EINVAL, "quantize: NULL pointer");
    if (R < 0 || K <= 0) return set_error(T2C_EINVAL, "quantize: bad shape R=%lld K=%lld", (long long)R, (long long)K);
    if (R == 0) return T2C_OK;
    const cudaStream_t s = as_stream(stream);
    uint8_t *o = static_cast<uint8_t *>(out);
    if (wtype == T2C_Q8_0) {
        if (K % 32) return set_error(T2C_EINVAL, "Q8_0 needs K %% 32 == 0");
        const int64_t blocks = R * (K / 32);
        const int64_t grid = (blocks * 32 + kQThreads - 1) / kQThreads;
        quantize_q8_0_kernel<<<static_cast<unsigned>(grid), kQThreads, 0, s>>>(x, o, blocks, K / 32, K);
    } else if (wtype == T2C_Q4_K) {
        if (K % 256) return set_error(T2C_EINVAL, "Q4_K needs K %% 256 == 0");
        const int64_t blocks = R * (K / 256);
        const int64_t grid = (blocks + kQThreads / 8 - 1) / (kQThreads / 8);
        quantize_q4_k_kernel<<<static_cast<unsigned>(grid), kQThreads, 0, s>>>(x, o, blocks, K / 256, K);
    } else if (wtype == T2C_Q6_K) {
        if (K % 256) return set_error(T2C_EINVAL, "Q6_K needs K %% 256 == 0");
        const int64_t blocks = R * (K / 256);
        const int64_t grid = (blocks + kQThreads / 16 - 1) / (kQThreads / 16);
        quantize_q6_k_kernel<<<static_cast<unsigned>(grid), kQThreads, 0, s>>>(x, o, blocks, K / 256, K);
    } else {
        return set_error(T2C_EUNSUPPORTED, "quantize: weight type %d", wtype);
    }
    return check_launch("quantize");
}

extern "C" int t2c_dequantize(int wtype, const void *w, float *out, int64_t R, int64_t K, void *stream) {
    if (w == nullptr || out == nullptr) return set_error(T2C_EINVAL, "dequantize: NULL pointer");
    if (row_bytes(wtype, K) < 0 || wtype == T2C_F16) return set_error(T2C_EINVAL, "dequantize: bad type/K");
    if (R <= 0) return R == 0 ? T2C_OK : set_error(T2C_EINVAL, "dequantize: R < 0");
    const int64_t total = R * K;
    dequant_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, as_stream(stream)>>>(
        wtype, static_cast<const uint8_t *>(w), out, total, K);
    return check_launch("dequantize");
}
